// libredukt_archive.so: the host side of a compressed window, native.
//
// The plugin computes each step's coder CDF on the device; what stays on the host is the range
// coder that turns each step's {symbol, low, high} into bytes, the CRC-32 of the window and the
// archive container.  This file holds those, for n lockstep streams at once, and the synthetic
// text workload the archive benchmark codes (an order-3 Markov source over printable ASCII and a
// byte-level vocabulary learned from it by pair merges, tokenised by greedy longest match).
//
//   CRC-32            src/domain/crc32.rs:6-50 (IEEE 802.3, reflected polynomial 0xEDB88320)
//   range coder       src/domain/coder.rs:114-290 (24-bit normalisation, 64-bit low with carry
//                     propagation, the decoder's clamp of the cumulative frequency to total - 1)
//   Cdf::uniform      src/domain/coder.rs:84-98 (the CDF of a stream's first token)
//   container         docs/api/FORMAT-SPEC.md:182-226, src/application/lockstep.rs:401-412:
//                     RDKT v5 header, the coded stream, the CRC-32 (little-endian) of the bytes
//                     that entered the coder
#include "../../include/redukt_archive.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

// ---- CRC-32 ---------------------------------------------------------------------------------

struct CrcTables {
    uint32_t t[4][256];
    CrcTables() {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c & 1u) ? (c >> 1) ^ 0xEDB88320u : c >> 1;
            t[0][i] = c;
        }
        // slicing by 4: t[k][i] is the CRC of byte i followed by k zero bytes
        for (uint32_t i = 0; i < 256; i++)
            for (int k = 1; k < 4; k++) t[k][i] = (t[k - 1][i] >> 8) ^ t[0][t[k - 1][i] & 0xFFu];
    }
};
const CrcTables kCrc;

// ---- range coder ----------------------------------------------------------------------------

constexpr uint32_t kTop = 1u << 24;

struct Encoder {
    uint64_t low = 0;
    uint32_t range = 0xFFFFFFFFu;
    uint8_t cache = 0;
    uint64_t ff_count = 0;
    bool first = true;
    std::vector<uint8_t> out;

    void shift_low() {
        const uint32_t low32 = (uint32_t)low;
        if (low32 < 0xFF000000u || (low >> 32) != 0) {
            const uint8_t carry = (uint8_t)(low >> 32);
            if (!first) out.push_back((uint8_t)(cache + carry));
            first = false;
            for (uint64_t i = 0; i < ff_count; i++) out.push_back((uint8_t)(0xFFu + carry));
            ff_count = 0;
            cache = (uint8_t)((low >> 24) & 0xFFu);
        } else {
            ff_count++;
        }
        low = (low & 0x00FFFFFFull) << 8;
    }
    // false on a range underflow (total larger than the current range)
    bool encode(uint32_t lo, uint32_t hi, uint32_t total) {
        const uint64_t r = range / total;
        if (r == 0 || lo >= hi || hi > total) return false;
        low += (uint64_t)lo * r;
        range = hi < total ? (uint32_t)(r * (hi - lo)) : range - (uint32_t)(r * lo);
        while (range < kTop) {
            shift_low();
            range <<= 8;
        }
        return true;
    }
    void finish() {
        for (int i = 0; i < 5; i++) shift_low();
        if (!first) {
            out.push_back(cache);
            for (uint64_t i = 0; i < ff_count; i++) out.push_back(0xFF);
        }
        first = true;  // finished: further shifts write nothing
        ff_count = 0;
    }
};

struct Decoder {
    uint32_t low = 0, range = 0xFFFFFFFFu, code = 0;
    std::vector<uint8_t> in;
    size_t pos = 0;

    uint8_t next() { return pos < in.size() ? in[pos++] : 0; }
    void start() {
        low = 0;
        range = 0xFFFFFFFFu;
        code = 0;
        pos = 0;
        for (int i = 0; i < 4; i++) code = (code << 8) | next();
    }
    // UINT32_MAX on a range underflow (a corrupted stream)
    uint32_t get_freq(uint32_t total) const {
        const uint32_t r = range / total;
        if (r == 0) return 0xFFFFFFFFu;
        return std::min((code - low) / r, total - 1);
    }
    bool update(uint32_t lo, uint32_t hi, uint32_t total) {
        const uint32_t r = range / total;
        if (r == 0 || lo >= hi || hi > total) return false;
        low += r * lo;
        range = hi < total ? r * (hi - lo) : range - r * lo;
        while (range < kTop) {
            code = (code << 8) | next();
            low <<= 8;
            range <<= 8;
        }
        return true;
    }
};

struct Coders {
    std::vector<Encoder> enc;
    std::vector<Decoder> dec;
};

// ---- workload: order-3 Markov text over printable ASCII -------------------------------------

uint64_t splitmix(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// The source: an order-3 character model (next byte given the previous three) estimated from a
// training stream of pseudo-words.  A lexicon of 6000 words (lengths 1-12, letters drawn from a
// skewed letter law) is drawn from the model seed; the training stream is 4 MB of Zipf(1.0)-chosen
// words separated by spaces, with a comma, full stop or newline-free line break (". ") now and
// then and capitalised sentence starts.  Text is then sampled from the model's counts, one
// seeded generator per window, so every window is a different sample of the same source.
struct MarkovModel {
    uint64_t seed = ~0ull;
    // context (3 bytes) -> [first, first + len) of `succ` (byte, cumulative count)
    std::unordered_map<uint32_t, std::pair<uint32_t, uint32_t>> ctx;
    std::vector<std::pair<uint8_t, uint32_t>> succ;
};

uint64_t rng_next(uint64_t& st) {
    st = splitmix(st);
    return st;
}

void markov_build(MarkovModel& M, uint64_t seed) {
    uint64_t r = splitmix(seed ^ 0x5EEDull);
    // letter law: weight of letter i ~ 1 / (i + 2)^1.1 over a seeded permutation of a..z
    char letters[26];
    for (int i = 0; i < 26; i++) letters[i] = (char)('a' + i);
    for (int i = 25; i > 0; i--) std::swap(letters[i], letters[rng_next(r) % (uint64_t)(i + 1)]);
    double lw[26], lsum = 0;
    for (int i = 0; i < 26; i++) lsum += (lw[i] = 1.0 / std::pow(i + 2.0, 1.1));
    auto letter = [&]() {
        double u = (rng_next(r) >> 11) * (1.0 / 9007199254740992.0) * lsum;
        for (int i = 0; i < 26; i++)
            if ((u -= lw[i]) < 0) return letters[i];
        return letters[25];
    };
    std::vector<std::string> lex;
    for (int w = 0; w < 6000; w++) {
        const int len = 1 + (int)(rng_next(r) % 4) + (int)(rng_next(r) % 5) + (int)(rng_next(r) % 4);
        std::string s;
        for (int i = 0; i < len; i++) s.push_back(letter());
        lex.push_back(s);
    }
    std::vector<double> zc(lex.size());
    double z = 0;
    for (size_t i = 0; i < lex.size(); i++) zc[i] = (z += 1.0 / (double)(i + 1));
    std::string train;
    train.reserve(4 << 20);
    bool cap = true;
    while (train.size() < (4u << 20)) {
        const double u = (rng_next(r) >> 11) * (1.0 / 9007199254740992.0) * z;
        const size_t wi = (size_t)(std::lower_bound(zc.begin(), zc.end(), u) - zc.begin());
        std::string w = lex[std::min(wi, lex.size() - 1)];
        if (cap) w[0] = (char)(w[0] - 32);
        cap = false;
        train += w;
        const uint64_t p = rng_next(r) % 100;
        if (p < 6) train += ", ";
        else if (p < 11) {
            train += ". ";
            cap = true;
        } else train += " ";
    }
    std::unordered_map<uint32_t, std::vector<uint32_t>> cnt;  // context -> counts of 128 bytes
    for (size_t i = 3; i < train.size(); i++) {
        const uint32_t c = ((uint32_t)(uint8_t)train[i - 3] << 16) | ((uint32_t)(uint8_t)train[i - 2] << 8) |
                           (uint8_t)train[i - 1];
        auto& v = cnt[c];
        if (v.empty()) v.assign(128, 0);
        v[(uint8_t)train[i] & 0x7F]++;
    }
    std::vector<uint32_t> keys;
    for (auto& kv : cnt) keys.push_back(kv.first);
    std::sort(keys.begin(), keys.end());  // deterministic layout
    for (uint32_t k : keys) {
        const auto& v = cnt[k];
        const uint32_t first = (uint32_t)M.succ.size();
        uint32_t cum = 0;
        for (int b = 0; b < 128; b++)
            if (v[b]) M.succ.push_back({(uint8_t)b, cum += v[b]});
        M.ctx[k] = {first, (uint32_t)M.succ.size() - first};
    }
    M.seed = seed;
}

// ---- workload: vocabulary and greedy tokenizer ----------------------------------------------

// Byte trie of the vocabulary; edges in one hash table keyed by (node, byte).
struct Trie {
    std::unordered_map<uint64_t, int32_t> edge;
    std::vector<int32_t> token{-1};  // token ending at each node (-1: none); node 0 is the root
    int32_t next(int32_t node, uint8_t byte) const {
        auto it = edge.find(((uint64_t)node << 8) | byte);
        return it == edge.end() ? -1 : it->second;
    }
    void add(const uint8_t* s, size_t len, int32_t id) {
        int32_t cur = 0;
        for (size_t i = 0; i < len; i++) {
            const uint64_t key = ((uint64_t)cur << 8) | s[i];
            auto it = edge.find(key);
            if (it == edge.end()) {
                const int32_t nx = (int32_t)token.size();
                token.push_back(-1);
                edge.emplace(key, nx);
                cur = nx;
            } else {
                cur = it->second;
            }
        }
        token[cur] = id;
    }
};

struct Tokenizer {
    std::vector<uint8_t> blob;
    std::vector<uint32_t> off;  // token i = blob[off[i] .. off[i + 1])
    Trie trie;
    uint32_t vocab = 0;

    // Greedy longest match: at each position the longest vocabulary entry that matches.
    size_t encode(const uint8_t* text, size_t n, uint32_t* ids, size_t cap) const {
        size_t k = 0, i = 0;
        while (i < n) {
            int32_t cur = 0, best = -1;
            size_t best_len = 0;
            for (size_t j = i; j < n; j++) {
                cur = trie.next(cur, text[j]);
                if (cur < 0) break;
                if (trie.token[cur] >= 0) {
                    best = trie.token[cur];
                    best_len = j - i + 1;
                }
            }
            if (best < 0) return (size_t)-1;  // a byte outside the vocabulary (cannot happen: 256 byte tokens)
            if (ids) {
                if (k >= cap) return (size_t)-1;
                ids[k] = (uint32_t)best;
            }
            k++;
            i += best_len;
        }
        return k;
    }
};

}  // namespace

extern "C" {

uint32_t rk_crc32_update(uint32_t state, const uint8_t* data, size_t n) {
    uint32_t c = state;
    size_t i = 0;
    for (; i + 4 <= n; i += 4) {
        c ^= (uint32_t)data[i] | ((uint32_t)data[i + 1] << 8) | ((uint32_t)data[i + 2] << 16) |
             ((uint32_t)data[i + 3] << 24);
        c = kCrc.t[3][c & 0xFFu] ^ kCrc.t[2][(c >> 8) & 0xFFu] ^ kCrc.t[1][(c >> 16) & 0xFFu] ^ kCrc.t[0][c >> 24];
    }
    for (; i < n; i++) c = (c >> 8) ^ kCrc.t[0][(c ^ data[i]) & 0xFFu];
    return c;
}

uint32_t rk_crc32(const uint8_t* data, size_t n) { return rk_crc32_update(0xFFFFFFFFu, data, n) ^ 0xFFFFFFFFu; }

void* rk_coders_new(uint32_t n) {
    Coders* c = new (std::nothrow) Coders();
    if (!c) return nullptr;
    c->enc.resize(n);
    c->dec.resize(n);
    return c;
}

void rk_coders_free(void* h) { delete static_cast<Coders*>(h); }

int32_t rk_enc_uniform(void* h, uint32_t n, const uint32_t* streams, const uint32_t* symbols, uint32_t alphabet) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || alphabet == 0 || alphabet > kTop) return RK_ARC_INVALID;
    const uint32_t f = kTop / alphabet, total = f * alphabet;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = streams ? streams[i] : i, y = symbols[i];
        if (s >= c->enc.size() || y >= alphabet) return RK_ARC_INVALID;
        if (!c->enc[s].encode(y * f, (y + 1) * f, total)) return RK_ARC_CORRUPT;
    }
    return RK_ARC_OK;
}

int32_t rk_enc_batch(void* h, uint32_t n, const uint32_t* streams, const uint32_t* query, uint32_t total) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || total == 0) return RK_ARC_INVALID;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = streams ? streams[i] : i;
        if (s >= c->enc.size()) return RK_ARC_INVALID;
        if (!c->enc[s].encode(query[3 * i + 1], query[3 * i + 2], total)) return RK_ARC_CORRUPT;
    }
    return RK_ARC_OK;
}

int64_t rk_enc_finish(void* h, uint32_t stream, uint8_t* out, size_t cap) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || stream >= c->enc.size()) return -1;
    Encoder& e = c->enc[stream];
    if (!out) {
        e.finish();
        return (int64_t)e.out.size();
    }
    if (cap < e.out.size()) return -1;
    std::memcpy(out, e.out.data(), e.out.size());
    const int64_t len = (int64_t)e.out.size();
    e = Encoder();  // ready for the next window
    return len;
}

int32_t rk_dec_start(void* h, uint32_t stream, const uint8_t* data, size_t len) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || stream >= c->dec.size() || (!data && len)) return RK_ARC_INVALID;
    Decoder& d = c->dec[stream];
    d.in.assign(data, data + len);
    d.start();
    return RK_ARC_OK;
}

int32_t rk_dec_uniform(void* h, uint32_t n, const uint32_t* streams, uint32_t alphabet, uint32_t* symbols) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || alphabet == 0 || alphabet > kTop) return RK_ARC_INVALID;
    const uint32_t f = kTop / alphabet, total = f * alphabet;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = streams ? streams[i] : i;
        if (s >= c->dec.size()) return RK_ARC_INVALID;
        Decoder& d = c->dec[s];
        const uint32_t cum = d.get_freq(total);
        if (cum == 0xFFFFFFFFu) return RK_ARC_CORRUPT;
        const uint32_t y = std::min(cum / f, alphabet - 1);  // Cdf::lookup on the uniform table
        if (!d.update(y * f, (y + 1) * f, total)) return RK_ARC_CORRUPT;
        symbols[i] = y;
    }
    return RK_ARC_OK;
}

int32_t rk_dec_freq_batch(void* h, uint32_t n, const uint32_t* streams, uint32_t total, uint32_t* cum) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || total == 0) return RK_ARC_INVALID;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = streams ? streams[i] : i;
        if (s >= c->dec.size()) return RK_ARC_INVALID;
        cum[i] = c->dec[s].get_freq(total);
        if (cum[i] == 0xFFFFFFFFu) return RK_ARC_CORRUPT;
    }
    return RK_ARC_OK;
}

int32_t rk_dec_update_batch(void* h, uint32_t n, const uint32_t* streams, const uint32_t* query, uint32_t total) {
    Coders* c = static_cast<Coders*>(h);
    if (!c || total == 0) return RK_ARC_INVALID;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t s = streams ? streams[i] : i;
        if (s >= c->dec.size()) return RK_ARC_INVALID;
        if (query[3 * i + 1] == 0xFFFFFFFFu || !c->dec[s].update(query[3 * i + 1], query[3 * i + 2], total))
            return RK_ARC_CORRUPT;
    }
    return RK_ARC_OK;
}

int64_t rk_arc_pack(const RkArcHeader* hdr, const uint8_t* stream, size_t stream_len, uint32_t crc, uint8_t* out,
                    size_t cap) {
    if (!hdr || (!stream && stream_len)) return -1;
    const bool reset = hdr->reset_log2 != 0;
    const size_t need = 8 + 4 + 1 + 1 + (reset ? 1 : 0) + 1 + stream_len + 4;
    if (!out) return (int64_t)need;
    if (cap < need) return -1;
    size_t o = 0;
    static const uint8_t magic[8] = {'R', 'D', 'K', 'T', 5, 0, 0, 0};
    std::memcpy(out, magic, 8);
    o = 8;
    for (int i = 0; i < 4; i++) out[o++] = (uint8_t)(hdr->total_bytes >> (8 * i));
    out[o++] = 0x40;  // FLAGS: a BACKBONE byte follows (v4 flag bit 6); no other optional field
    out[o++] = (uint8_t)((hdr->profile & 0xBFu) | (reset ? 0x40u : 0u));
    if (reset) out[o++] = hdr->reset_log2;
    out[o++] = hdr->backbone;
    if (stream_len) std::memcpy(out + o, stream, stream_len);
    o += stream_len;
    for (int i = 0; i < 4; i++) out[o++] = (uint8_t)(crc >> (8 * i));
    return (int64_t)o;
}

int32_t rk_arc_unpack(const uint8_t* buf, size_t len, RkArcHeader* hdr, size_t* stream_off, size_t* stream_len,
                      uint32_t* crc) {
    if (!buf || !hdr || !stream_off || !stream_len || !crc) return RK_ARC_INVALID;
    if (len < 8 + 4 + 1 + 1 + 4 || std::memcmp(buf, "RDKT\x05\x00\x00\x00", 8) != 0) return RK_ARC_FORMAT;
    size_t o = 8;
    hdr->total_bytes = (uint32_t)buf[8] | ((uint32_t)buf[9] << 8) | ((uint32_t)buf[10] << 16) | ((uint32_t)buf[11] << 24);
    o = 12;
    const uint8_t flags = buf[o++];
    if (flags != 0x40) return RK_ARC_FORMAT;  // only the plugin layout this library writes
    const uint8_t profile = buf[o++];
    if (profile & 0x80u) return RK_ARC_FORMAT;
    hdr->profile = profile;
    hdr->reset_log2 = 0;
    if (profile & 0x40u) {
        hdr->reset_log2 = buf[o++];
        if (hdr->reset_log2 < 8 || hdr->reset_log2 > 20) return RK_ARC_FORMAT;
    }
    if (o + 1 + 4 > len) return RK_ARC_FORMAT;
    hdr->backbone = buf[o++];
    *stream_off = o;
    *stream_len = len - o - 4;
    *crc = (uint32_t)buf[len - 4] | ((uint32_t)buf[len - 3] << 8) | ((uint32_t)buf[len - 2] << 16) |
           ((uint32_t)buf[len - 1] << 24);
    return RK_ARC_OK;
}

size_t rk_markov_text(uint64_t model_seed, uint64_t seed, uint8_t* out, size_t n) {
    static MarkovModel M;  // built once per model seed (not thread-safe)
    if (M.seed != model_seed) {
        M = MarkovModel();
        markov_build(M, model_seed);
    }
    uint64_t r = splitmix(seed ^ 0xC0FFEEull);
    uint32_t c = ((uint32_t)'e' << 16) | ((uint32_t)'s' << 8) | (uint32_t)' ';  // a context the model has
    for (size_t i = 0; i < n; i++) {
        auto it = M.ctx.find(c);
        uint8_t b = ' ';
        if (it != M.ctx.end()) {
            const uint32_t first = it->second.first, len = it->second.second;
            const uint32_t tot = M.succ[first + len - 1].second;
            const uint32_t x = (uint32_t)(rng_next(r) % tot);
            uint32_t lo = 0, hi = len - 1;  // first entry whose cumulative count exceeds x
            while (lo < hi) {
                const uint32_t mid = (lo + hi) / 2;
                if (M.succ[first + mid].second > x) hi = mid;
                else lo = mid + 1;
            }
            b = M.succ[first + lo].first;
        }
        out[i] = b;
        c = ((c << 8) | b) & 0xFFFFFFu;
    }
    return n;
}

void* rk_tok_new(const uint8_t* blob, const uint32_t* offsets, uint32_t vocab) {
    if (!blob || !offsets || vocab < 256) return nullptr;
    Tokenizer* t = new (std::nothrow) Tokenizer();
    if (!t) return nullptr;
    t->blob.assign(blob, blob + offsets[vocab]);
    t->off.assign(offsets, offsets + vocab + 1);
    t->vocab = vocab;
    for (uint32_t i = 0; i < vocab; i++)
        if (offsets[i + 1] > offsets[i]) t->trie.add(blob + offsets[i], offsets[i + 1] - offsets[i], (int32_t)i);
    return t;
}

void rk_tok_free(void* h) { delete static_cast<Tokenizer*>(h); }

int64_t rk_tok_encode(void* h, const uint8_t* text, size_t n, uint32_t* ids, size_t cap) {
    const Tokenizer* t = static_cast<const Tokenizer*>(h);
    if (!t || (!text && n)) return -1;
    const size_t k = t->encode(text, n, ids, cap);
    return k == (size_t)-1 ? -1 : (int64_t)k;
}

int64_t rk_tok_decode(void* h, const uint32_t* ids, size_t n, uint8_t* out, size_t cap) {
    const Tokenizer* t = static_cast<const Tokenizer*>(h);
    if (!t || (!ids && n)) return -1;
    size_t o = 0;
    for (size_t i = 0; i < n; i++) {
        if (ids[i] >= t->vocab) return -1;
        const uint32_t a = t->off[ids[i]], b = t->off[ids[i] + 1];
        if (out) {
            if (o + (b - a) > cap) return -1;
            std::memcpy(out + o, t->blob.data() + a, b - a);
        }
        o += b - a;
    }
    return (int64_t)o;
}

int64_t rk_vocab_learn(const uint8_t* text, size_t n, uint32_t vocab, uint32_t per_round, uint32_t max_len,
                       uint8_t* blob, size_t blob_cap, uint32_t* offsets) {
    if (!text || vocab < 256 || !offsets || per_round == 0) return -1;
    std::vector<std::vector<uint8_t>> toks;
    for (int i = 0; i < 256; i++) toks.push_back({(uint8_t)i});
    std::unordered_map<std::string, uint32_t> have;
    for (int i = 0; i < 256; i++) have.emplace(std::string(1, (char)i), (uint32_t)i);
    std::vector<uint32_t> ids(n);
    while (toks.size() < vocab) {
        // tokenise with the current vocabulary, count adjacent pairs, add the most frequent
        Tokenizer t;
        std::vector<uint8_t> bl;
        std::vector<uint32_t> of{0};
        for (auto& s : toks) {
            bl.insert(bl.end(), s.begin(), s.end());
            of.push_back((uint32_t)bl.size());
        }
        t.blob = bl;
        t.off = of;
        t.vocab = (uint32_t)toks.size();
        for (uint32_t i = 0; i < t.vocab; i++) t.trie.add(bl.data() + of[i], of[i + 1] - of[i], (int32_t)i);
        const size_t k = t.encode(text, n, ids.data(), ids.size());
        if (k == (size_t)-1 || k < 2) break;
        std::unordered_map<uint64_t, uint32_t> cnt;
        cnt.reserve(k);
        for (size_t i = 0; i + 1 < k; i++) cnt[((uint64_t)ids[i] << 32) | ids[i + 1]]++;
        std::vector<std::pair<uint32_t, uint64_t>> top;
        top.reserve(cnt.size());
        for (auto& kv : cnt) top.push_back({kv.second, kv.first});
        std::sort(top.begin(), top.end(), [](const std::pair<uint32_t, uint64_t>& x, const std::pair<uint32_t, uint64_t>& y) {
            return x.first != y.first ? x.first > y.first : x.second < y.second;  // count, then pair: deterministic
        });
        uint32_t added = 0;
        for (auto& p : top) {
            if (toks.size() >= vocab || added >= per_round || p.first < 2) break;
            std::vector<uint8_t> s = toks[p.second >> 32];
            const auto& r = toks[p.second & 0xFFFFFFFFu];
            s.insert(s.end(), r.begin(), r.end());
            if (s.size() > max_len) continue;
            std::string key(s.begin(), s.end());
            if (have.count(key)) continue;
            have.emplace(key, (uint32_t)toks.size());
            toks.push_back(s);
            added++;
        }
        if (added == 0) break;
    }
    // pad with distinct byte strings that printable text never contains (a NUL, then the index in
    // bytes >= 0x80) so the vocabulary has exactly `vocab` entries
    uint64_t filler = 0;
    while (toks.size() < vocab) {
        std::vector<uint8_t> s{0x00};
        uint64_t f = filler++;
        do {
            s.push_back((uint8_t)(0x80 | (f & 0x7F)));
            f >>= 7;
        } while (f);
        toks.push_back(s);
    }
    size_t o = 0;
    offsets[0] = 0;
    for (uint32_t i = 0; i < vocab; i++) {
        if (blob) {
            if (o + toks[i].size() > blob_cap) return -1;
            std::memcpy(blob + o, toks[i].data(), toks[i].size());
        }
        o += toks[i].size();
        offsets[i + 1] = (uint32_t)o;
    }
    return (int64_t)o;
}

}  // extern "C"
