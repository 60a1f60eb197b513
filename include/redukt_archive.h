/*
 * redukt_archive.h -- C ABI of libredukt_archive.so: the host side of a compressed window.
 *
 * With redukt_b200_forward_batch_cdf the device returns, for each lockstep stream and step, the
 * coder's {symbol, low, high} (encoding) or {symbol, low, high} of a cumulative frequency
 * (decoding).  This library turns those into bytes and back: the reference's range coder, its
 * CRC-32 and its archive container, for n streams at once.  It also generates the synthetic text
 * workload of the archive benchmark.  Plain C types only.  Not thread-safe per handle.
 */
#ifndef REDUKT_ARCHIVE_H
#define REDUKT_ARCHIVE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { RK_ARC_OK = 0, RK_ARC_INVALID = 1, RK_ARC_CORRUPT = 2, RK_ARC_FORMAT = 3 };

/* CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320): src/domain/crc32.rs:6-50.  _update takes
 * and returns the raw state (start with 0xFFFFFFFF, finish with ^ 0xFFFFFFFF). */
uint32_t rk_crc32_update(uint32_t state, const uint8_t* data, size_t n);
uint32_t rk_crc32(const uint8_t* data, size_t n);

/* n range encoders and n range decoders (src/domain/coder.rs:114-290), one per lockstep stream.
 * `streams` lists which coder each batch entry uses (NULL = entry i uses coder i).  query is
 * [n][3] {symbol, low, high} as redukt_b200_forward_batch_cdf writes it; total is the CDF total
 * (2^24).  CORRUPT: an interval the coder cannot take (empty, past total, or a range underflow of a
 * corrupted stream). */
void* rk_coders_new(uint32_t n);
void rk_coders_free(void* coders);
/* A stream's first token is coded with Cdf::uniform(alphabet) (src/domain/coder.rs:84-98). */
int32_t rk_enc_uniform(void* coders, uint32_t n, const uint32_t* streams, const uint32_t* symbols, uint32_t alphabet);
int32_t rk_enc_batch(void* coders, uint32_t n, const uint32_t* streams, const uint32_t* query, uint32_t total);
/* out == NULL: finish the stream and return its byte count; then call again with a buffer to take
 * the bytes (the encoder is reset for the next window).  -1 on a bad stream or a short buffer. */
int64_t rk_enc_finish(void* coders, uint32_t stream, uint8_t* out, size_t cap);
int32_t rk_dec_start(void* coders, uint32_t stream, const uint8_t* data, size_t len);
int32_t rk_dec_uniform(void* coders, uint32_t n, const uint32_t* streams, uint32_t alphabet, uint32_t* symbols);
int32_t rk_dec_freq_batch(void* coders, uint32_t n, const uint32_t* streams, uint32_t total, uint32_t* cum_freqs);
int32_t rk_dec_update_batch(void* coders, uint32_t n, const uint32_t* streams, const uint32_t* query, uint32_t total);

/* RDKT v5 container of one window (docs/api/FORMAT-SPEC.md:182-226, src/application/lockstep.rs:401-412):
 * MAGIC "RDKT\5\0\0\0", TOTAL_BYTES (LE u32), FLAGS = 0x40 (a BACKBONE byte follows), PROFILE
 * (bit 6 set when RESET_LOG2 follows), [RESET_LOG2], BACKBONE_ID, the coded stream, CRC-32 (LE)
 * of the window's bytes.  The reference writes this header for the GPU plugin backbone (ID 3,
 * PROFILE 0x50, RESET_LOG2 12). */
typedef struct {
    uint32_t total_bytes;
    uint8_t profile;     /* bits 0-3 quant, 4-5 numeric contract; bit 6 is set from reset_log2 */
    uint8_t reset_log2;  /* 0 = none, else 8..20 */
    uint8_t backbone;    /* BACKBONE_ID */
} RkArcHeader;
/* out == NULL returns the size needed; -1 on a bad argument or a short buffer. */
int64_t rk_arc_pack(const RkArcHeader* hdr, const uint8_t* stream, size_t stream_len, uint32_t crc, uint8_t* out,
                    size_t cap);
/* FORMAT: not this container (magic, flags, reserved bits, RESET_LOG2 range, too short). */
int32_t rk_arc_unpack(const uint8_t* buf, size_t len, RkArcHeader* hdr, size_t* stream_off, size_t* stream_len,
                      uint32_t* crc);

/* ---- Synthetic workload (benchmark inputs; not part of the coding path) ---- */
/* n bytes sampled (generator seed `seed`) from the order-3 character model `model_seed` over
 * printable ASCII (0x20-0x7E): the model is estimated from a training stream of Zipf-chosen
 * pseudo-words of a seeded lexicon.  Builds the model on the first call for a model seed. */
size_t rk_markov_text(uint64_t model_seed, uint64_t seed, uint8_t* out, size_t n);
/* A byte-level vocabulary of `vocab` entries learned from `text`: the 256 bytes, then rounds of the
 * `per_round` most frequent adjacent token pairs (at most max_len bytes each) under greedy
 * longest-match tokenisation, padded with strings printable text never contains.  Writes
 * offsets[vocab + 1] and, if blob != NULL, the concatenated strings; returns the blob size. */
int64_t rk_vocab_learn(const uint8_t* text, size_t n, uint32_t vocab, uint32_t per_round, uint32_t max_len,
                       uint8_t* blob, size_t blob_cap, uint32_t* offsets);
/* Greedy longest-match tokenizer over a vocabulary (token i = blob[offsets[i] .. offsets[i + 1])). */
void* rk_tok_new(const uint8_t* blob, const uint32_t* offsets, uint32_t vocab);
void rk_tok_free(void* tok);
/* ids == NULL counts; returns the token count, -1 on a short buffer. */
int64_t rk_tok_encode(void* tok, const uint8_t* text, size_t n, uint32_t* ids, size_t cap);
/* out == NULL counts; returns the byte count, -1 on a bad id or a short buffer. */
int64_t rk_tok_decode(void* tok, const uint32_t* ids, size_t n, uint8_t* out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* REDUKT_ARCHIVE_H */
