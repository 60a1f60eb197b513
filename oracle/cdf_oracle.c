/*
 * cdf_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement of the reference's coder-side CDF under numeric contract fmath-v1, used
 * only as the parity checker for the device CDF kernels (tests/) and as the timed CPU leg of
 * bench.py.  Nothing in the redukt_b200 product path links or calls this file.
 *
 *   exp constants and table           src/domain/fmath.rs:110-120
 *   exp_f64 (musl exp, non-FMA path)  src/domain/fmath.rs:343-429
 *   cdf_from_logits_with              src/application/codec.rs:785-798
 *   Cdf::from_probs                   src/domain/coder.rs:43-82
 *   Cdf::lookup                       src/domain/coder.rs:100-114
 *
 * Every operation is a single IEEE-754 binary64 (or binary32) operation in source order;
 * compile with -ffp-contract=off so that no multiply-add is fused (the reference never
 * fuses: src/domain/fmath.rs:18-20).  The 2^(i/128) table is derived from its definition by
 * redukt_b200/csrc/gen_exp_table.py (the same derived words the device kernel uses); the exp
 * is pinned against the reference's 24 golden bit patterns (fmath.rs:525-550) in the tests.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../redukt_b200/csrc/rk_exp_table.h"

static const uint64_t kExpTab[256] = {RK_EXP_TABLE_WORDS};

static inline uint64_t bits_of(double x) { uint64_t u; memcpy(&u, &x, 8); return u; }
static inline double double_of(uint64_t u) { double x; memcpy(&x, &u, 8); return x; }
static inline uint32_t top12(double x) { return (uint32_t)(bits_of(x) >> 52); }

/* musl exp_data.c constants (N = 128): 128/ln2, -ln2/128 split hi/lo, 1.5*2^52, and the
 * degree-5 polynomial coefficients C2..C5 (fmath.rs:110-119). */
#define EXP_INVLN2N   0x40671547652b82feull
#define EXP_NEGLN2HIN 0xbf762e42fefa0000ull
#define EXP_NEGLN2LON 0xbd0cf79abc9e3b3aull
#define EXP_SHIFT     0x4338000000000000ull
static const uint64_t kExpPoly[4] = {0x3fdffffffffffdbdull, 0x3fc555555555543cull,
                                     0x3fa55555cf172b91ull, 0x3f81111167a4d017ull};

/* fmath.rs:359-381: scale * (1 + tmp) near overflow / in the subnormal range. */
static double exp_specialcase(double tmp, uint64_t sbits, uint64_t ki) {
    if ((ki & 0x80000000ull) == 0) {
        double scale = double_of(sbits - (1009ull << 52));
        return double_of((uint64_t)(1009 + 1023) << 52) * (scale + scale * tmp);
    }
    double scale = double_of(sbits + (1022ull << 52));
    double y = scale + scale * tmp;
    if (y < 1.0) {
        double lo = scale - y + scale * tmp;
        double hi = 1.0 + y;
        lo = 1.0 - hi + y + lo;
        y = (hi + lo) - 1.0;
        if (y == 0.0) y = 0.0;
    }
    return double_of(1ull << 52) * y;
}

/* fmath.rs:383-429 (exp_f64 with exp_huge inlined) */
double orc_exp_f64(double x) {
    const uint32_t top_tiny = 0x3c9, top_512 = 0x408, top_1024 = 0x409, top_inf = 0x7ff;
    uint32_t abstop = top12(x) & 0x7ff;
    if (abstop - top_tiny >= top_512 - top_tiny) {
        if (abstop - top_tiny >= 0x80000000u) return 1.0 + x;
        if (abstop >= top_1024) {
            if (bits_of(x) == 0xfff0000000000000ull) return 0.0;
            if (abstop >= top_inf) return 1.0 + x;
            return (bits_of(x) >> 63) ? 0.0 : INFINITY;
        }
        abstop = 0;
    }
    double z = double_of(EXP_INVLN2N) * x;
    double kd = z + double_of(EXP_SHIFT);
    uint64_t ki = bits_of(kd);
    kd = kd - double_of(EXP_SHIFT);
    double r = x + kd * double_of(EXP_NEGLN2HIN) + kd * double_of(EXP_NEGLN2LON);
    uint64_t idx = 2 * (ki & 127);
    uint64_t top = ki << 45;
    double tail = double_of(kExpTab[idx]);
    uint64_t sbits = kExpTab[idx + 1] + top;
    double r2 = r * r;
    double tmp = tail + r + r2 * (double_of(kExpPoly[0]) + r * double_of(kExpPoly[1])) +
                 r2 * r2 * (double_of(kExpPoly[2]) + r * double_of(kExpPoly[3]));
    if (abstop == 0) return exp_specialcase(tmp, sbits, ki);
    double scale = double_of(sbits);
    return scale + scale * tmp;
}

/* coder.rs:43-82 for one row: probs[v] (binary32) -> cdf[v + 1] (24-bit total). */
static void cdf_from_probs_row(const float* probs, uint32_t v, uint32_t* freqs, uint32_t* cdf) {
    const uint32_t total = 1u << 24;
    const uint64_t remaining = (uint64_t)total - v;
    double sum_p = -0.0;
    for (uint32_t i = 0; i < v; i++) sum_p += (double)probs[i];
    double inv = sum_p > 0.0 ? 1.0 / sum_p : 0.0;
    uint64_t extra_used = 0;
    for (uint32_t i = 0; i < v; i++) {
        double t = (double)probs[i] * inv * (double)remaining + 0.5;
        /* Rust `as u64` saturates: NaN and negatives give 0. */
        uint64_t extra = (t != t || t <= 0.0) ? 0 : (t >= 18446744073709551616.0 ? UINT64_MAX : (uint64_t)t);
        freqs[i] = 1u + (uint32_t)extra;
        extra_used += extra;
    }
    int64_t diff = (int64_t)remaining - (int64_t)extra_used;
    if (diff != 0) {
        /* Iterator::max_by_key returns the LAST of equal maxima */
        uint32_t max_i = 0;
        for (uint32_t i = 1; i < v; i++)
            if (freqs[i] >= freqs[max_i]) max_i = i;
        freqs[max_i] = (uint32_t)((int64_t)freqs[max_i] + diff);
    }
    uint32_t cum = 0;
    cdf[0] = 0;
    for (uint32_t i = 0; i < v; i++) {
        cum += freqs[i];
        cdf[i + 1] = cum;
    }
}

/* codec.rs:785-798 for one row: logits[v] -> cdf[v + 1]; scratch holds v doubles + v floats
 * + v uint32. */
static void cdf_from_logits_row(const float* logits, uint32_t v, uint32_t* cdf, void* scratch) {
    double* e = (double*)scratch;
    float* p = (float*)(e + v);
    uint32_t* freqs = (uint32_t*)(p + v);
    double max_l = -INFINITY;
    for (uint32_t i = 0; i < v; i++) max_l = fmax(max_l, (double)logits[i]);
    double sum = 0.0;
    for (uint32_t i = 0; i < v; i++) {
        e[i] = orc_exp_f64((double)logits[i] - max_l);
        sum += e[i];
    }
    double inv_sum = 1.0 / sum;
    for (uint32_t i = 0; i < v; i++) p[i] = (float)(e[i] * inv_sum);
    cdf_from_probs_row(p, v, freqs, cdf);
}

typedef struct {
    const float* logits;
    uint32_t* cdf;
    uint32_t v, ld_logits, ld_cdf, row0, row1;
} CdfJob;

static void* cdf_worker(void* arg) {
    CdfJob* j = (CdfJob*)arg;
    void* scratch = malloc((size_t)j->v * 16);
    if (!scratch) return (void*)1;
    for (uint32_t r = j->row0; r < j->row1; r++)
        cdf_from_logits_row(j->logits + (size_t)r * j->ld_logits, j->v, j->cdf + (size_t)r * j->ld_cdf, scratch);
    free(scratch);
    return NULL;
}

/* Rows are independent, so splitting them over threads never changes a row's arithmetic.
 * Returns 0, or -1 on an invalid argument / allocation failure. */
int orc_cdf_from_logits(const float* logits, uint32_t n_rows, uint32_t vocab, uint32_t ld_logits, uint32_t* cdf,
                        uint32_t ld_cdf, int n_threads) {
    if (vocab == 0 || vocab >= (1u << 24) || ld_logits < vocab || ld_cdf < vocab + 1) return -1;
    if (n_threads < 1) n_threads = 1;
    if ((uint32_t)n_threads > n_rows) n_threads = n_rows ? (int)n_rows : 1;
    CdfJob jobs[256];
    pthread_t tid[256];
    if (n_threads > 256) n_threads = 256;
    int rc = 0;
    for (int t = 0; t < n_threads; t++) {
        jobs[t] = (CdfJob){logits, cdf, vocab, ld_logits, ld_cdf, (uint32_t)((uint64_t)n_rows * t / n_threads),
                           (uint32_t)((uint64_t)n_rows * (t + 1) / n_threads)};
    }
    int started = 1;
    for (; started < n_threads; started++)
        if (pthread_create(&tid[started], NULL, cdf_worker, &jobs[started]) != 0) break;
    for (int t = started; t < n_threads; t++)  /* threads that did not start: run here */
        if (cdf_worker(&jobs[t])) rc = -1;
    if (cdf_worker(&jobs[0])) rc = -1;
    for (int t = 1; t < started; t++) {
        void* ret = NULL;
        pthread_join(tid[t], &ret);
        if (ret) rc = -1;
    }
    return rc;
}

/* coder.rs:43-82 on caller probabilities (the reference's coder unit tests build CDFs this way). */
int orc_cdf_from_probs(const float* probs, uint32_t v, uint32_t* cdf) {
    if (v == 0 || v >= (1u << 24)) return -1;
    uint32_t* freqs = (uint32_t*)malloc((size_t)v * sizeof(uint32_t));
    if (!freqs) return -1;
    cdf_from_probs_row(probs, v, freqs, cdf);
    free(freqs);
    return 0;
}

/* coder.rs:100-114: the symbol whose interval holds cum_freq (binary search, lowest match). */
uint32_t orc_cdf_lookup(const uint32_t* cdf, uint32_t vocab, uint32_t cum_freq) {
    uint32_t lo = 0, hi = vocab;
    while (lo < hi) {
        uint32_t mid = (lo + hi) / 2;
        if (cdf[mid + 1] <= cum_freq) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}
