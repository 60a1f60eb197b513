// rk_cdf.cuh -- the coder's 24-bit CDF of one row of logits, computed on the device.
//
// Same result, bit for bit, as the reference host code that turns a logit row into the range
// coder's frequency table under numeric contract fmath-v1:
//   cdf_from_logits_with   src/application/codec.rs:785-798
//   exp_f64 (musl exp)     src/domain/fmath.rs:343-429
//   Cdf::from_probs        src/domain/coder.rs:43-82
//   Cdf::lookup            src/domain/coder.rs:100-114
//
// One CTA per row.  The row's two sequential binary64 sums (sum of exps; sum of the f32
// probabilities widened to f64) are reproduced exactly without a sequential chain:
//
//   While the running sum s lies in the binade [2^E, 2^(E+1)), it is a multiple of
//   u = 2^(E-52), and for a term x >= 0 with s + x < 2^(E+1) the IEEE sum is s + round_u(x),
//   where round_u rounds x to a multiple of u.  In units of u, with x/u = f + r (f integer,
//   0 <= r < 1), the increment is f, or f + 1 when r > 1/2, or, when r == 1/2 (a tie, common
//   for tiny f32 probabilities), f plus the one unit that makes the new sum even.  The
//   increment therefore depends only on the parity of the running sum, so each term is a map
//   {input parity -> (increment, output parity)}; such maps compose associatively, and a
//   block-wide scan of them gives every partial sum of a run exactly.  The scan finds the
//   first term whose rounded partial sum reaches 2^(E+1) (the binade changes, and with it u);
//   everything before it is added at once, that term by one IEEE addition, and the scan
//   resumes with the new binade.  Terms are >= 0, so s never decreases and leaves each binade
//   once: a row of 50,280 terms takes about (terms / 4096) + (binades crossed) scan rounds
//   instead of 50,280 dependent additions.
//
// Every floating-point operation is an explicit round-to-nearest intrinsic (__dmul_rn,
// __dadd_rn, ...), so the compiler cannot contract a multiply and an add into an FMA.
#pragma once

#include <cstdint>

#include "rk_exp_table.h"

namespace cdf {

constexpr int kThreads = 512;
constexpr int kPer = 8;                       // consecutive terms per thread in one chunk
constexpr int kChunk = kThreads * kPer;       // 4096 terms per scan round
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kTotal = 1u << 24;         // coder.rs:12 (TOP)
// The first kHead terms of each sum are added one by one by a single thread: there the running
// sum is still small and crosses a binade every few terms, and each crossing would cost a scan
// round over the whole chunk.
constexpr int kHead = 512;
// Rows of up to this many logits keep their per-symbol workspace (f32 probabilities, then
// frequencies) in dynamic shared memory; longer rows use the output row itself.
constexpr int kSmemVocab = 53248;   // 208 KB
static_assert(kPer == 8, "the shared-workspace paths move kPer words as two 16-byte vectors");

__device__ __forceinline__ double dbits(uint64_t u) { return __longlong_as_double((long long)u); }
__device__ __forceinline__ uint64_t bitsd(double x) { return (uint64_t)__double_as_longlong(x); }

// musl exp_data.c constants (N = 128), fmath.rs:110-119: 128/ln2, -ln2/128 as hi + lo, the
// 1.5 * 2^52 rounding shift, and the polynomial coefficients C2..C5.
constexpr uint64_t kInvLn2N = 0x40671547652b82feull;
constexpr uint64_t kNegLn2HiN = 0xbf762e42fefa0000ull;
constexpr uint64_t kNegLn2LoN = 0xbd0cf79abc9e3b3aull;
constexpr uint64_t kShift = 0x4338000000000000ull;
constexpr uint64_t kC2 = 0x3fdffffffffffdbdull, kC3 = 0x3fc555555555543cull;
constexpr uint64_t kC4 = 0x3fa55555cf172b91ull, kC5 = 0x3f81111167a4d017ull;

__device__ const uint64_t g_exp_tab[256] = {RK_EXP_TABLE_WORDS};

// fmath.rs:359-381 (overflow / subnormal tail of exp).
__device__ __noinline__ double exp_special(double tmp, uint64_t sbits, uint64_t ki) {
    if ((ki & 0x80000000ull) == 0) {
        double scale = dbits(sbits - (1009ull << 52));
        return __dmul_rn(dbits((uint64_t)(1009 + 1023) << 52), __dadd_rn(scale, __dmul_rn(scale, tmp)));
    }
    double scale = dbits(sbits + (1022ull << 52));
    double y = __dadd_rn(scale, __dmul_rn(scale, tmp));
    if (y < 1.0) {
        double lo = __dadd_rn(__dsub_rn(scale, y), __dmul_rn(scale, tmp));
        double hi = __dadd_rn(1.0, y);
        lo = __dadd_rn(__dadd_rn(__dsub_rn(1.0, hi), y), lo);
        y = __dsub_rn(__dadd_rn(hi, lo), 1.0);
        if (y == 0.0) y = 0.0;
    }
    return __dmul_rn(dbits(1ull << 52), y);
}

// fmath.rs:383-429: e^x, the reference's portable binary64 exp; tab is the 256-word table in
// shared memory.
__device__ __forceinline__ double exp_f64(double x, const uint64_t* tab) {
    uint32_t abstop = (uint32_t)(bitsd(x) >> 52) & 0x7ff;
    if (abstop - 0x3c9u >= 0x408u - 0x3c9u) {
        if (abstop - 0x3c9u >= 0x80000000u) return __dadd_rn(1.0, x);
        if (abstop >= 0x409u) {
            if (bitsd(x) == 0xfff0000000000000ull) return 0.0;
            if (abstop >= 0x7ffu) return __dadd_rn(1.0, x);
            return (bitsd(x) >> 63) ? 0.0 : dbits(0x7ff0000000000000ull);
        }
        abstop = 0;
    }
    double z = __dmul_rn(dbits(kInvLn2N), x);
    double kd = __dadd_rn(z, dbits(kShift));
    uint64_t ki = bitsd(kd);
    kd = __dsub_rn(kd, dbits(kShift));
    double r = __dadd_rn(__dadd_rn(x, __dmul_rn(kd, dbits(kNegLn2HiN))), __dmul_rn(kd, dbits(kNegLn2LoN)));
    uint32_t idx = 2u * (uint32_t)(ki & 127);
    uint64_t top = ki << 45;
    double tail = dbits(tab[idx]);
    uint64_t sbits = tab[idx + 1] + top;
    double r2 = __dmul_rn(r, r);
    double p23 = __dmul_rn(r2, __dadd_rn(dbits(kC2), __dmul_rn(r, dbits(kC3))));
    double p45 = __dmul_rn(__dmul_rn(r2, r2), __dadd_rn(dbits(kC4), __dmul_rn(r, dbits(kC5))));
    double tmp = __dadd_rn(__dadd_rn(__dadd_rn(tail, r), p23), p45);
    if (abstop == 0) return exp_special(tmp, sbits, ki);
    double scale = dbits(sbits);
    return __dadd_rn(scale, __dmul_rn(scale, tmp));
}

struct Smem {
    uint64_t tab[256];
    unsigned long long wtot[kWarps];
    unsigned long long wi0[kWarps], wi1[kWarps];   // per-warp parity maps of a scan round
    uint32_t wpar[kWarps];
    unsigned long long xi0[kWarps], xi1[kWarps];   // their exclusive prefixes, and the total
    uint32_t xpar[kWarps];
    unsigned long long ti0, ti1;
    uint32_t tpar;
    unsigned long long wsum[kWarps];
    int wmin[kWarps];
    uint32_t wfreq[kWarps];
    int widx[kWarps];
    float wmax[kWarps];
    double xv;                 // the term at the first break of a scan round
    unsigned long long pbefore;  // rounded partial sum (units of u) just before it
    double head[kHead];        // the first kHead terms of a sum, added by one thread
    double hs;
};

// Exclusive block scan of one u64 per thread; returns the thread's offset, total in *tot.
// Ends with a barrier after the last read of sm.wtot.
__device__ __forceinline__ unsigned long long block_scan(unsigned long long v, Smem& sm,
                                                         unsigned long long* tot) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    unsigned long long inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) sm.wtot[w] = inc;
    __syncthreads();
    unsigned long long before = 0, all = 0;
#pragma unroll
    for (int i = 0; i < kWarps; i++) {
        unsigned long long t = sm.wtot[i];
        before += i < w ? t : 0ull;
        all += t;
    }
    __syncthreads();
    *tot = all;
    return before + inc - v;
}

__device__ __forceinline__ int block_min(int v, Smem& sm) {
    v = __reduce_min_sync(0xffffffffu, v);
    if ((threadIdx.x & 31) == 0) sm.wmin[threadIdx.x >> 5] = v;
    __syncthreads();
    int m = sm.wmin[0];
#pragma unroll
    for (int i = 1; i < kWarps; i++) m = min(m, sm.wmin[i]);
    __syncthreads();
    return m;
}

// A run of terms as a function of the running sum's parity p (in units of u): the run adds
// i0 (p = 0) or i1 (p = 1) and leaves the parity bit (par >> p) & 1.
struct PMap {
    unsigned long long i0, i1;
    uint32_t par;   // bit 0: output parity for input 0; bit 1: for input 1
};

__device__ __forceinline__ PMap pm_identity() { return {0ull, 0ull, 2u}; }

// a, then b
__device__ __forceinline__ PMap pm_then(const PMap& a, const PMap& b) {
    const uint32_t a0 = a.par & 1u, a1 = (a.par >> 1) & 1u;
    PMap r;
    r.i0 = a.i0 + (a0 ? b.i1 : b.i0);
    r.i1 = a.i1 + (a1 ? b.i1 : b.i0);
    r.par = ((b.par >> a0) & 1u) | (((b.par >> a1) & 1u) << 1);
    return r;
}

// Warp-shuffle form of a map: i0 and one word holding i1 - i0 + 1 (i1 - i0 is -1, 0 or 1: two
// running sums that start one unit apart stay at most two units apart under round-to-even) and
// the parity bits.
__device__ __forceinline__ PMap pm_shfl_up(const PMap& m, int o) {
    const uint32_t meta = (uint32_t)(m.i1 - m.i0 + 1ull) | (m.par << 2);
    PMap r;
    r.i0 = __shfl_up_sync(0xffffffffu, m.i0, o);
    const uint32_t mt = __shfl_up_sync(0xffffffffu, meta, o);
    r.i1 = r.i0 + (unsigned long long)(mt & 3u) - 1ull;
    r.par = mt >> 2;
    return r;
}

// Exclusive block scan of one map per thread (in thread order); returns the composition of all
// earlier threads' maps and the whole block's in *all.  Ends with a barrier after the last
// read of the per-warp slots.
__device__ __forceinline__ PMap block_scan_maps(const PMap& v, Smem& sm, PMap* all) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    PMap inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const PMap t = pm_shfl_up(inc, o);
        if (lane >= o) inc = pm_then(t, inc);
    }
    PMap ex = pm_shfl_up(inc, 1);   // exclusive within the warp
    if (lane == 0) ex = pm_identity();
    if (lane == 31) { sm.wi0[w] = inc.i0; sm.wi1[w] = inc.i1; sm.wpar[w] = inc.par; }
    __syncthreads();
    if (w == 0) {   // one warp scans the per-warp maps
        PMap t = lane < kWarps ? PMap{sm.wi0[lane], sm.wi1[lane], sm.wpar[lane]} : pm_identity();
        PMap c = t;
#pragma unroll
        for (int o = 1; o < kWarps; o <<= 1) {
            const PMap u = pm_shfl_up(c, o);
            if (lane >= o) c = pm_then(u, c);
        }
        PMap e = pm_shfl_up(c, 1);
        if (lane == 0) e = pm_identity();
        __syncwarp();
        if (lane < kWarps) { sm.xi0[lane] = e.i0; sm.xi1[lane] = e.i1; sm.xpar[lane] = e.par; }
        if (lane == kWarps - 1) { sm.ti0 = c.i0; sm.ti1 = c.i1; sm.tpar = c.par; }
    }
    __syncthreads();
    const PMap before = {sm.xi0[w], sm.xi1[w], sm.xpar[w]};
    *all = PMap{sm.ti0, sm.ti1, sm.tpar};
    __syncthreads();
    return pm_then(before, ex);
}

// Adds this thread's kPer terms x[] (chunk-local indices threadIdx.x * kPer + k, in order
// across the block) to the block-uniform running sum s, exactly as the sequential loop
// `for x in chunk { s += x }` would.  Terms must be >= 0 or NaN.
__device__ void chain_chunk(const double (&x)[kPer], double& s, Smem& sm, int pos = 0) {
    const int j0 = threadIdx.x * kPer;
    while (pos < kChunk) {
        if (s != s) return;                          // NaN absorbs the rest
        const bool zero = s == 0.0;
        const bool tiny = !zero && s < 0x1p-900;     // outside the scaled-integer range: one term per round
        double up = 0.0, u = 0.0;
        unsigned long long su = 0, thr = 0;
        if (!zero && !tiny) {
            const int e = (int)((bitsd(s) >> 52) & 0x7ff) - 1023;
            up = dbits((uint64_t)(1023 + 52 - e) << 52);   // 2^(52-E)
            u = dbits((uint64_t)(1023 - 52 + e) << 52);    // 2^(E-52)
            su = (unsigned long long)__dmul_rn(s, up);     // s / u, an integer in [2^52, 2^53)
            thr = (1ull << 53) - su;
        }
        // per term: the increment in units of u (f, or f + 1 past a half), with a tie flag and
        // the parity of f, or a break
        unsigned long long inc[kPer];
        uint32_t brk = 0, tie = 0, odd = 0;            // bit k: term k
        const bool live = j0 + kPer > pos;             // has terms at or after pos
        unsigned long long mine = 0;
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int j = j0 + k;
            inc[k] = 0;
            if (live && j >= pos) {
                if (zero || tiny) {
                    if (x[k] != 0.0) brk |= 1u << k;      // s + 0 = s: zeros never break
                } else {
                    const double t = __dmul_rn(x[k], up);  // exact: scaling by a power of two
                    if (!(t < 0x1p53)) {                   // leaves the binade on its own (or NaN)
                        inc[k] = 1ull << 53;
                        brk |= 1u << k;
                    } else {
                        const double f = floor(t);
                        const double fr = __dsub_rn(t, f);   // exact
                        const unsigned long long fi = (unsigned long long)f;
                        inc[k] = fi + (fr > 0.5 ? 1ull : 0ull);
                        if (fr == 0.5) tie |= 1u << k;
                        odd |= (uint32_t)(fi & 1ull) << k;
                    }
                }
            }
            mine += inc[k];
        }
        // a tie adds one more unit when the running sum would otherwise end odd: for running
        // parity 0 when f is odd, for parity 1 when f is even
        const uint32_t p_start = (uint32_t)(su & 1ull);
        unsigned long long run, total;
        uint32_t par = 0;
        const bool ties = __syncthreads_or(tie != 0);
        if (ties) {
            PMap m_all = pm_identity();
#pragma unroll
            for (int k = 0; k < kPer; k++) {
                if (!live) break;
                const unsigned long long a0 = inc[k] + ((tie & odd) >> k & 1u);
                const unsigned long long a1 = inc[k] + ((tie & ~odd) >> k & 1u);
                const PMap m = {a0, a1, (uint32_t)(a0 & 1ull) | (uint32_t)(((1ull + a1) & 1ull) << 1)};
                m_all = pm_then(m_all, m);
            }
            PMap all;
            const PMap pre = block_scan_maps(m_all, sm, &all);
            run = p_start ? pre.i1 : pre.i0;          // units of u added before this thread
            par = (pre.par >> p_start) & 1u;
            total = p_start ? all.i1 : all.i0;
        } else {                                       // no tie: increments do not depend on parity
            run = block_scan(mine, sm, &total);
        }
        int first = kChunk;
        double my_x = 0.0;
        unsigned long long my_pb = 0;
        if (live) {
#pragma unroll
            for (int k = 0; k < kPer; k++) {
                const int j = j0 + k;
                const unsigned long long pb = run;
                const unsigned long long d =
                    inc[k] + ((tie >> k) & 1u & (((odd >> k) & 1u) ^ par));   // tie: even result
                run += d;
                par = (uint32_t)((par + d) & 1ull);
                const bool over = !zero && !tiny && run >= thr;
                if (first == kChunk && j >= pos && (((brk >> k) & 1u) || over)) {
                    first = j;
                    my_x = x[k];
                    my_pb = pb;
                }
            }
        }
        const int fb = block_min(first, sm);
        if (fb == kChunk) {
            if (!zero && !tiny) s = __dmul_rn((double)(su + total), u);
            return;
        }
        if (first == fb) {     // the one thread that owns the block's first break
            sm.xv = my_x;
            sm.pbefore = my_pb;
        }
        __syncthreads();
        // the next write of xv/pbefore comes after two more barriers (in block_scan), by which
        // time every thread has read these
        if (!zero && !tiny) s = __dmul_rn((double)(su + sm.pbefore), u);
        s = __dadd_rn(s, sm.xv);
        pos = fb + 1;
    }
}

// Adds the chunk's first kHead terms to s (block-uniform) one by one, as the sequential loop
// would; the caller continues the chunk at kHead.
__device__ __forceinline__ void add_head(const double (&x)[kPer], double& s, Smem& sm) {
#pragma unroll
    for (int k = 0; k < kPer; k++) {
        const int j = threadIdx.x * kPer + k;
        if (j < kHead) sm.head[j] = x[k];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = s;
#pragma unroll 16
        for (int j = 0; j < kHead; j++) a = __dadd_rn(a, sm.head[j]);
        sm.hs = a;
    }
    __syncthreads();
    s = sm.hs;
    __syncthreads();   // sm.hs and sm.head are free again
}

// One CTA per row.  cdf row: vocab + 1 words (cdf[0] = 0, cdf[vocab] = 2^24); rows longer than
// kSmemVocab also use it as their workspace.  Launch with vocab * 4 bytes of dynamic shared memory
// when vocab <= kSmemVocab (cdf_dyn_smem).  Optional per-row queries, three words each in q_out:
//   symbols  (encoder): {symbol, cdf[symbol], cdf[symbol + 1]}, or {symbol, ~0u, ~0u} when
//                       symbol >= vocab;
//   cum_freqs (decoder): {lookup(cum), cdf[sym], cdf[sym + 1]} with Cdf::lookup's binary search;
//                       sym == vocab (and ~0u, ~0u) when cum >= the total.
__global__ void __launch_bounds__(kThreads, 1)
k_cdf_rows(const float* __restrict__ logits, int vocab, int ld_logits, uint32_t* __restrict__ cdf_all,
           int ld_cdf, const uint32_t* __restrict__ symbols, const uint32_t* __restrict__ cum_freqs,
           uint32_t* __restrict__ q_out) {
    __shared__ Smem sm;
    extern __shared__ __align__(16) uint32_t dyn_ws[];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const float* L = logits + (size_t)row * ld_logits;
    uint32_t* c = cdf_all + (size_t)row * ld_cdf;
    uint32_t* ws = vocab <= kSmemVocab ? dyn_ws : c + 1;   // ws[i]: symbol i's probability, then frequency
    for (int i = tid; i < 256; i += kThreads) sm.tab[i] = g_exp_tab[i];

    // max_l = fold(-inf, f64::max): f32 max is the same value, NaN ignored (codec.rs:787)
    float m = -INFINITY;
    for (int i = tid; i < vocab; i += kThreads) m = fmaxf(m, __ldg(L + i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm.wmax[w] = m;
    __syncthreads();
    m = sm.wmax[0];
#pragma unroll
    for (int i = 1; i < kWarps; i++) m = fmaxf(m, sm.wmax[i]);
    const double max_l = (double)m;

    // sum of e = exp(l - max) in index order (codec.rs:789-793)
    double s = 0.0;
    for (int base = 0; base < vocab; base += kChunk) {
        double x[kPer];
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int i = base + tid * kPer + k;
            x[k] = i < vocab ? exp_f64(__dsub_rn((double)__ldg(L + i), max_l), sm.tab) : 0.0;
        }
        if (base == 0) add_head(x, s, sm);
        chain_chunk(x, s, sm, base == 0 ? kHead : 0);
    }
    const double inv_sum = __ddiv_rn(1.0, s);

    // p = (e * inv_sum) as f32 (codec.rs:795), kept in ws; sum_p in index order (coder.rs:52)
    const bool vec = ws == dyn_ws;   // shared workspace: 16-byte aligned, kPer words per thread at once
    double sp = 0.0;
    for (int base = 0; base < vocab; base += kChunk) {
        double x[kPer];
        uint32_t pb[kPer];
        const int i0 = base + tid * kPer;
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int i = i0 + k;
            pb[k] = 0;
            if (i < vocab) {
                const double e = exp_f64(__dsub_rn((double)__ldg(L + i), max_l), sm.tab);
                const float p = __double2float_rn(__dmul_rn(e, inv_sum));
                pb[k] = __float_as_uint(p);
                x[k] = (double)p;
            } else {
                x[k] = 0.0;
            }
        }
        if (vec && i0 + kPer <= vocab) {
            reinterpret_cast<uint4*>(ws + i0)[0] = make_uint4(pb[0], pb[1], pb[2], pb[3]);
            reinterpret_cast<uint4*>(ws + i0)[1] = make_uint4(pb[4], pb[5], pb[6], pb[7]);
        } else {
#pragma unroll
            for (int k = 0; k < kPer; k++)
                if (i0 + k < vocab) ws[i0 + k] = pb[k];
        }
        if (base == 0) add_head(x, sp, sm);
        chain_chunk(x, sp, sm, base == 0 ? kHead : 0);
    }

    // freqs = 1 + round(p * inv * remaining) (coder.rs:53-63); extra_used; last maximum
    const uint32_t remaining = kTotal - (uint32_t)vocab;
    const double inv = sp > 0.0 ? __ddiv_rn(1.0, sp) : 0.0;
    const double rem_d = (double)remaining;
    unsigned long long used = 0;
    uint32_t best_f = 0;
    int best_i = -1;
    for (int i = tid; i < vocab; i += kThreads) {
        const float p = __uint_as_float(ws[i]);
        const double t = __dadd_rn(__dmul_rn(__dmul_rn((double)p, inv), rem_d), 0.5);
        unsigned long long extra = 0;
        if (t == t && t > 0.0) extra = t >= 0x1p64 ? ~0ull : __double2ull_rz(t);   // Rust `as u64`
        const uint32_t f = 1u + (uint32_t)extra;
        ws[i] = f;
        used += extra;
        if (f >= best_f) { best_f = f; best_i = i; }   // i increases: ties keep the later index
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        used += __shfl_xor_sync(0xffffffffu, used, o);
        const uint32_t of = __shfl_xor_sync(0xffffffffu, best_f, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (of > best_f || (of == best_f && oi > best_i)) { best_f = of; best_i = oi; }
    }
    if (lane == 0) { sm.wsum[w] = used; sm.wfreq[w] = best_f; sm.widx[w] = best_i; }
    __syncthreads();
    if (tid == 0) {
        unsigned long long u_all = 0;
        uint32_t bf = 0;
        int bi = -1;
        for (int i = 0; i < kWarps; i++) {
            u_all += sm.wsum[i];
            if (sm.wfreq[i] > bf || (sm.wfreq[i] == bf && sm.widx[i] > bi)) { bf = sm.wfreq[i]; bi = sm.widx[i]; }
        }
        const long long diff = (long long)remaining - (long long)u_all;   // coder.rs:66-72
        if (diff != 0 && bi >= 0) ws[bi] = (uint32_t)((long long)bf + diff);
        c[0] = 0;
    }
    __syncthreads();

    // cdf[i + 1] = freqs[0] + ... + freqs[i] (wrapping u32, coder.rs:74-80)
    uint32_t carry = 0;
    for (int base = 0; base < vocab; base += kChunk) {
        uint32_t f[kPer];
        uint32_t acc = 0;
        const int i0 = base + tid * kPer;
        if (vec && i0 + kPer <= vocab) {
            const uint4 a = reinterpret_cast<const uint4*>(ws + i0)[0];
            const uint4 b = reinterpret_cast<const uint4*>(ws + i0)[1];
            f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
        } else {
#pragma unroll
            for (int k = 0; k < kPer; k++) f[k] = i0 + k < vocab ? ws[i0 + k] : 0u;
        }
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            acc += f[k];
            f[k] = acc;
        }
        unsigned long long tot = 0;
        const uint32_t off = (uint32_t)block_scan(acc, sm, &tot);
#pragma unroll
        for (int k = 0; k < kPer; k++) {
            const int i = base + tid * kPer + k;
            if (i < vocab) c[i + 1] = carry + off + f[k];
        }
        carry += (uint32_t)tot;
    }
    if (!q_out) return;
    __syncthreads();           // the last chunk's cdf writes, before thread 0 reads them
    if (tid != 0) return;
    uint32_t* q = q_out + (size_t)row * 3;
    if (symbols) {
        const uint32_t sym = symbols[row];
        q[0] = sym;
        q[1] = sym < (uint32_t)vocab ? c[sym] : ~0u;
        q[2] = sym < (uint32_t)vocab ? c[sym + 1] : ~0u;
    } else if (cum_freqs) {
        const uint32_t cum = cum_freqs[row];
        uint32_t lo = 0, hi = (uint32_t)vocab;   // coder.rs:100-114
        while (lo < hi) {
            const uint32_t mid = (lo + hi) / 2;
            if (c[mid + 1] <= cum) lo = mid + 1;
            else hi = mid;
        }
        q[0] = lo;
        q[1] = lo < (uint32_t)vocab ? c[lo] : ~0u;
        q[2] = lo < (uint32_t)vocab ? c[lo + 1] : ~0u;
    }
}

__host__ __device__ constexpr size_t cdf_dyn_smem(int vocab) {
    return vocab <= kSmemVocab ? (size_t)vocab * sizeof(uint32_t) : 0;
}

}  // namespace cdf
