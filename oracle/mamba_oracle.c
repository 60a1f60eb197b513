/*
 * mamba_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement of the redukt reference CPU path for one Mamba-1 decode step
 * (`MambaModel::forward_into` / `forward_multi`, Kernel::Plain = numeric contract 1),
 * used only as the parity checker (tests/, __graft_entry__.smoke()) and as the timed
 * CPU baseline leg of bench.py.  Nothing in the redukt_b200 product path links or
 * calls this file; the product fails loudly when its CUDA library is missing.
 *
 * Operation order follows the reference's scalar kernels, which the reference documents
 * as bit-identical to its AVX2 kernels (src/domain/gemv.rs:13-21, tensor.rs:1674-1705):
 *   portable_expf            src/domain/tensor.rs:765-794   (Cephes degree-5 polynomial)
 *   portable_lnf             src/domain/tensor.rs:799-837   (musl/FreeBSD logf)
 *   portable_softplus        src/domain/tensor.rs:859-861
 *   lane_expf/lane_sigmoidf  src/domain/tensor.rs:877-885
 *   rms_norm_into            src/domain/tensor.rs:900-908
 *   layer_norm_into          src/domain/tensor.rs:1390-1398
 *   silu_inplace (body/tail) src/domain/tensor.rs:1197-1211
 *   gated_silu_mul           src/domain/tensor.rs:1229-1243
 *   ssm_recurrence_d16       src/domain/tensor.rs:1281-1325 (dt-sparse skip, hsum_ssm tree)
 *   dot_avx2_order           src/domain/tensor.rs:1663-1705 (8 lanes, hsum_f32 tree, tail)
 *   Q8wMatrix::quantize      src/domain/gemv.rs:251-273     (group 64 or per-row)
 *   q8w_rows_scalar          src/domain/gemv.rs:459-502     (group dot, hsum8, group order)
 *   dequant_row_into         src/domain/gemv.rs:284-295
 *   conv_silu_block          src/infrastructure/mamba/model.rs:134-153
 *   scan_block               src/infrastructure/mamba/model.rs:174-190
 *   layer_norm_step          src/infrastructure/mamba/model.rs:193-200
 *   forward_layers_normed    src/infrastructure/mamba/model.rs:635-752
 *   forward_layers_normed_multi / forward_multi  src/infrastructure/mamba/model.rs:773-935
 *   maybe_periodic_reset     src/infrastructure/mamba/model.rs:315-320
 *   softmax_into             src/domain/tensor.rs:1917-1933
 *
 * The x86 AVX2 variants below reproduce the same lane order with separate multiply and
 * add (no FMA), exactly like the reference's AVX2 tier; they exist only so the timed CPU
 * baseline runs at the reference's real speed.  Compile with -ffp-contract=off (the
 * reference never contracts: src/domain/fmath.rs:18-20).
 *
 * Row partitioning over pool threads never changes the arithmetic of a row, so results
 * are bit-identical for any thread count (the reference's par_pool rule, gemv.rs:1-7).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif
#include <pthread.h>
#include <unistd.h>

#define ORC_API __attribute__((visibility("default")))
#define ORC_INTERNAL __attribute__((visibility("hidden")))
#include "oracle_internal.h"

/* ------------------------------------------------------------------------------------
 * Portable transcendentals (tensor.rs:757-915)
 * ---------------------------------------------------------------------------------- */

static inline float f_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* tensor.rs:910-915: round to nearest even through the 2^23 magic constant. */
static inline float portable_roundeven(float x) {
    const float magic = 8388608.0f;
    return x >= 0.0f ? (x + magic) - magic : (x - magic) + magic;
}

ORC_API float orc_expf(float x) {
    const float LOG2E = 1.44269504088896341f;
    const float LN2_HI = 6.93145751953125E-1f;
    const float LN2_LO = 1.42860682030941723212E-6f;
    const float EXP_LO = -87.3365447505531f;
    const float EXP_HI = 88.3762626647949f;
    const float P0 = 1.9875691500E-4f, P1 = 1.3981999507E-3f, P2 = 8.3334519073E-3f;
    const float P3 = 4.1665795894E-2f, P4 = 1.6666665459E-1f, P5 = 5.0000001201E-1f;
    x = x < EXP_LO ? EXP_LO : (x > EXP_HI ? EXP_HI : x);
    float fx = x * LOG2E;
    float nf = portable_roundeven(fx);
    int32_t n = (int32_t)nf;
    float r = (x - nf * LN2_HI) - nf * LN2_LO;
    float r2 = r * r;
    float y = P0;
    y = y * r + P1;
    y = y * r + P2;
    y = y * r + P3;
    y = y * r + P4;
    y = y * r + P5;
    y = (y * r2 + r) + 1.0f;
    float pow2n = f_from_bits(((uint32_t)(n + 127)) << 23);
    return y * pow2n;
}

ORC_API float orc_lnf(float x) {
    const float LN2_HI = 6.9313812256e-01f, LN2_LO = 9.0580006145e-06f;
    const float LG1 = 0.66666662693f, LG2 = 0.40000972152f, LG3 = 0.28498786688f, LG4 = 0.24279078841f;
    uint32_t ix = f_to_bits(x);
    int32_t k = 0;
    if (ix < 0x00800000u || (ix >> 31) != 0) {
        if ((uint32_t)(ix << 1) == 0) return -INFINITY;
        if ((ix >> 31) != 0) return NAN;
        k -= 25;
        ix = f_to_bits(x * f_from_bits(0x4c000000u));
    } else if (ix >= 0x7f800000u) {
        return x;
    } else if (ix == 0x3f800000u) {
        return 0.0f;
    }
    ix = ix + (0x3f800000u - 0x3f3504f3u);
    k += (int32_t)(ix >> 23) - 0x7f;
    ix = (ix & 0x007fffffu) + 0x3f3504f3u;
    float xn = f_from_bits(ix);
    float f = xn - 1.0f;
    float s = f / (2.0f + f);
    float dk = (float)k;
    float z = s * s;
    float w = z * z;
    float t1 = w * (LG2 + w * LG4);
    float t2 = z * (LG1 + w * LG3);
    float r = t2 + t1;
    float hfsq = 0.5f * f * f;
    return s * (hfsq + r) + dk * LN2_LO - hfsq + f + dk * LN2_HI;
}

/* tensor.rs:869-879: one lane of fast_exp_ps (a NaN lane is clamped to EXP_LO). */
ORC_INTERNAL float lane_expf(float x) { return orc_expf(isnan(x) ? -87.3365447505531f : x); }
ORC_API float orc_lane_sigmoidf(float x) { return 1.0f / (1.0f + lane_expf(0.0f - x)); }
ORC_INTERNAL float portable_sigmoidf(float x) { return 1.0f / (1.0f + orc_expf(-x)); }
static inline float portable_silu(float x) { return x * portable_sigmoidf(x); }
ORC_API float orc_softplus(float x) { return x > 20.0f ? x : orc_lnf(1.0f + orc_expf(x)); }

/* tensor.rs:1206-1211: SiLU over a slice, SIMD-body lanes then portable tail. */
static void silu_inplace(float* buf, size_t n) {
    size_t body = n / 8 * 8;
    for (size_t i = 0; i < body; i++) buf[i] *= orc_lane_sigmoidf(buf[i]);
    for (size_t i = body; i < n; i++) buf[i] = portable_silu(buf[i]);
}

/* tensor.rs:1238-1243 */
static void gated_silu_mul(float* out, const float* y, const float* z, size_t n) {
    size_t body = n / 8 * 8;
    for (size_t i = 0; i < body; i++) out[i] = y[i] * (z[i] * orc_lane_sigmoidf(z[i]));
    for (size_t i = body; i < n; i++) out[i] = y[i] * portable_silu(z[i]);
}

/* tensor.rs:900-908 */
static void rms_norm_into(float* x, const float* w, size_t n, float eps) {
    float sum_sq = 0.0f;
    for (size_t i = 0; i < n; i++) sum_sq += x[i] * x[i];
    float rms = sqrtf(sum_sq / (float)n + eps);
    float inv = 1.0f / rms;
    for (size_t i = 0; i < n; i++) x[i] = x[i] * inv * w[i];
}

/* tensor.rs:1390-1398 (Rust's f32 Sum folds sequentially). */
ORC_INTERNAL void layer_norm_into(float* out, const float* x, const float* w, const float* b, size_t n, float eps) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += x[i];
    float mean = sum / (float)n;
    float var = 0.0f;
    for (size_t i = 0; i < n; i++) var += (x[i] - mean) * (x[i] - mean);
    var = var / (float)n;
    float inv_std = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < n; i++) out[i] = (x[i] - mean) * inv_std * w[i] + b[i];
}


/* ------------------------------------------------------------------------------------
 * A small persistent thread pool (the role of the reference's par_pool, par_pool.rs:1-20):
 * it decides WHICH thread computes a row, never HOW, so results do not depend on the
 * thread count.
 * ---------------------------------------------------------------------------------- */


static struct {
    pthread_mutex_t mu;
    pthread_cond_t cv_work, cv_done;
    int nthreads;      /* workers + the caller */
    int started;
    long gen;          /* bumped once per job */
    int pending;       /* workers still running the current job */
    par_fn fn;
    void* ctx;
    long n;
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER, 0, 0, 0, 0, 0, 0, 0};

static void pool_range(int part, int parts, long n, long* b, long* e) {
    *b = n * part / parts;
    *e = n * (part + 1) / parts;
}

static void* pool_worker(void* arg) {
    int id = (int)(long)arg;
    long seen = 0;
    for (;;) {
        pthread_mutex_lock(&g_pool.mu);
        while (g_pool.gen == seen) pthread_cond_wait(&g_pool.cv_work, &g_pool.mu);
        seen = g_pool.gen;
        par_fn fn = g_pool.fn;
        void* ctx = g_pool.ctx;
        long n = g_pool.n;
        int parts = g_pool.nthreads;
        pthread_mutex_unlock(&g_pool.mu);
        long b, e;
        pool_range(id, parts, n, &b, &e);
        if (b < e) fn(ctx, b, e);
        pthread_mutex_lock(&g_pool.mu);
        if (--g_pool.pending == 0) pthread_cond_signal(&g_pool.cv_done);
        pthread_mutex_unlock(&g_pool.mu);
    }
    return NULL;
}

static int g_req_threads = 0;

static void pool_start(void) {
    if (g_pool.started) return;
    int t = g_req_threads;
    if (t <= 0) {
        const char* e = getenv("REDUKT_THREADS");
        t = e ? atoi(e) : 0;
        if (t <= 0) t = (int)sysconf(_SC_NPROCESSORS_ONLN);
    }
    if (t < 1) t = 1;
    if (t > 256) t = 256;
    g_pool.nthreads = t;
    for (int i = 1; i < t; i++) {
        pthread_t th;
        if (pthread_create(&th, NULL, pool_worker, (void*)(long)i) != 0) { g_pool.nthreads = i; break; }
        pthread_detach(th);
    }
    g_pool.started = 1;
}

/* Runs fn over [0, n) split into one contiguous range per thread; serial when small. */
ORC_INTERNAL void par_for(long n, long work, par_fn fn, void* ctx) {
    if (n <= 0) return;
    pool_start();
    if (g_pool.nthreads == 1 || work < 65536 || n < 2) { fn(ctx, 0, n); return; }
    pthread_mutex_lock(&g_pool.mu);
    g_pool.fn = fn;
    g_pool.ctx = ctx;
    g_pool.n = n;
    g_pool.pending = g_pool.nthreads - 1;
    g_pool.gen++;
    pthread_cond_broadcast(&g_pool.cv_work);
    pthread_mutex_unlock(&g_pool.mu);
    long b, e;
    pool_range(0, g_pool.nthreads, n, &b, &e);
    if (b < e) fn(ctx, b, e);
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.pending > 0) pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
}

/* ------------------------------------------------------------------------------------
 * GEMV kernels (gemv.rs, tensor.rs:1663-1705)
 * ---------------------------------------------------------------------------------- */

/* ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) -- hsum_f32_scalar / hsum8_scalar */
static inline float hsum8(const float a[8]) {
    float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
    return (s0 + s2) + (s1 + s3);
}

/* ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)) -- hsum_ssm_scalar (tensor.rs:1285-1294) */
static inline float hsum_ssm(const float a[8]) {
    float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
    return (s0 + s1) + (s2 + s3);
}

static float dot_ref_scalar(const float* w, const float* v, size_t n) {
    size_t body = n / 8 * 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t c = 0; c < body; c += 8)
        for (int l = 0; l < 8; l++) acc[l] += w[c + l] * v[c + l];
    float s = hsum8(acc);
    for (size_t c = body; c < n; c++) s += w[c] * v[c];
    return s;
}

static float group_dot_scalar(const int8_t* q, const float* v, size_t len) {
    size_t chunks = len / 8;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (size_t ch = 0; ch < chunks; ch++)
        for (int l = 0; l < 8; l++) acc[l] += (float)q[ch * 8 + l] * v[ch * 8 + l];
    float s = hsum8(acc);
    for (size_t c = chunks * 8; c < len; c++) s += (float)q[c] * v[c];
    return s;
}

#if defined(__x86_64__)
__attribute__((target("avx2"))) static inline float hsum8_avx(__m256 v) {
    __m128 hi = _mm256_extractf128_ps(v, 1);
    __m128 lo = _mm256_castps256_ps128(v);
    __m128 sum4 = _mm_add_ps(lo, hi);
    __m128 sum2 = _mm_add_ps(sum4, _mm_movehl_ps(sum4, sum4));
    return _mm_cvtss_f32(_mm_add_ss(sum2, _mm_shuffle_ps(sum2, sum2, 1)));
}

__attribute__((target("avx2"))) static float dot_ref_avx2(const float* w, const float* v, size_t n) {
    size_t body = n / 8 * 8;
    __m256 acc = _mm256_setzero_ps();
    for (size_t c = 0; c < body; c += 8)
        acc = _mm256_add_ps(acc, _mm256_mul_ps(_mm256_loadu_ps(w + c), _mm256_loadu_ps(v + c)));
    float s = hsum8_avx(acc);
    for (size_t c = body; c < n; c++) s += w[c] * v[c];
    return s;
}

__attribute__((target("avx2"))) static inline __m256 load_i8x8_ps(const int8_t* p) {
    __m128i b = _mm_loadl_epi64((const __m128i*)p);
    return _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(b));
}

__attribute__((target("avx2"))) static float group_dot_avx2(const int8_t* q, const float* v, size_t len) {
    size_t chunks = len / 8;
    __m256 acc = _mm256_setzero_ps();
    for (size_t ch = 0; ch < chunks; ch++)
        acc = _mm256_add_ps(acc, _mm256_mul_ps(load_i8x8_ps(q + ch * 8), _mm256_loadu_ps(v + ch * 8)));
    float s = hsum8_avx(acc);
    for (size_t c = chunks * 8; c < len; c++) s += (float)q[c] * v[c];
    return s;
}
#endif

static int g_use_avx2 = -1; /* -1 = detect */
ORC_INTERNAL int use_avx2(void) {
#if defined(__x86_64__)
    if (g_use_avx2 < 0) {
        const char* e = getenv("REDUKT_NO_SIMD");
        g_use_avx2 = (e && strcmp(e, "1") == 0) ? 0 : (__builtin_cpu_supports("avx2") ? 1 : 0);
    }
    return g_use_avx2;
#else
    return 0;
#endif
}

ORC_API void orc_set_simd(int on) { g_use_avx2 = on ? 1 : 0; }

ORC_INTERNAL float dot_ref(const float* w, const float* v, size_t n) {
#if defined(__x86_64__)
    if (use_avx2()) return dot_ref_avx2(w, v, n);
#endif
    return dot_ref_scalar(w, v, n);
}

static inline float group_dot(const int8_t* q, const float* v, size_t len) {
#if defined(__x86_64__)
    if (use_avx2()) return group_dot_avx2(q, v, len);
#endif
    return group_dot_scalar(q, v, len);
}

/* A large matrix in the active profile (model.rs:58-117). */
typedef struct {
    uint32_t rows, cols, group; /* group = 0 for F32 */
    float* f;                   /* F32 data, rows*cols */
    int8_t* q;                  /* Q8 data, rows*cols */
    float* scales;              /* Q8 scales, rows*(cols/group) */
} Mat;

/* gemv.rs:256-273; Rust `round` = half away from zero = C roundf. */
static void q8_quantize(const float* w, uint32_t rows, uint32_t cols, uint32_t group, int8_t* q, float* scales) {
    if (!(group > 0 && group % 8 == 0 && cols % group == 0)) group = cols;
    size_t total = (size_t)rows * cols;
    size_t ngroups = total / group;
    for (size_t gi = 0; gi < ngroups; gi++) {
        const float* wg = w + gi * group;
        float amax = 0.0f;
        for (uint32_t i = 0; i < group; i++) {
            float a = fabsf(wg[i]);
            amax = amax > a ? amax : a; /* f32::max(amax, |x|) */
        }
        float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
        float inv = 1.0f / scale;
        for (uint32_t i = 0; i < group; i++) {
            float r = roundf(wg[i] * inv);
            r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
            q[gi * group + i] = (int8_t)r;
        }
        scales[gi] = scale;
    }
}

ORC_API uint32_t orc_q8_effective_group(uint32_t cols, uint32_t group) {
    return (group > 0 && group % 8 == 0 && cols % group == 0) ? group : cols;
}

ORC_API void orc_q8_quantize(const float* w, uint32_t rows, uint32_t cols, uint32_t group, int8_t* q,
                             float* scales) {
    q8_quantize(w, rows, cols, group, q, scales);
}

static inline float q8_row(const Mat* m, size_t r, const float* v) {
    uint32_t cols = m->cols, group = m->group, gpr = cols / group;
    float sum = 0.0f;
    for (uint32_t g = 0; g < gpr; g++) {
        float d = group_dot(m->q + r * cols + (size_t)g * group, v + (size_t)g * group, group);
        sum += d * m->scales[r * gpr + g];
    }
    return sum;
}

static inline float mat_row(const Mat* m, size_t r, const float* v) {
    if (m->group) return q8_row(m, r, v);
    return dot_ref(m->f + r * m->cols, v, m->cols);
}

/* out[s][r] = M[r] . xs[s] for ns streams.  Each (stream,row) is computed by exactly the
 * single-stream row kernel, so any row/stream partition is bit-identical (gemv.rs:135-141). */
typedef struct { const Mat* m; int ns; const float* const* xs; float* const* outs; } GemvJob;

static void gemv_rows(void* ctx, long b, long e) {
    const GemvJob* j = (const GemvJob*)ctx;
    for (long r = b; r < e; r++)
        for (int s = 0; s < j->ns; s++) j->outs[s][r] = mat_row(j->m, (size_t)r, j->xs[s]);
}

static void gemv_multi(const Mat* m, int ns, const float* const* xs, float* const* outs) {
    GemvJob j = {m, ns, xs, outs};
    par_for((long)m->rows, (long)m->rows * m->cols * ns, gemv_rows, &j);
}

ORC_API void orc_gemv_f32(const float* mat, const float* v, uint32_t rows, uint32_t cols, float* out) {
    for (uint32_t r = 0; r < rows; r++) out[r] = dot_ref(mat + (size_t)r * cols, v, cols);
}

ORC_API void orc_gemv_q8(const int8_t* q, const float* scales, uint32_t rows, uint32_t cols, uint32_t group,
                         const float* v, float* out) {
    Mat m = {rows, cols, orc_q8_effective_group(cols, group), NULL, (int8_t*)q, (float*)scales};
    for (uint32_t r = 0; r < rows; r++) out[r] = q8_row(&m, r, v);
}

/* ------------------------------------------------------------------------------------
 * Model, .rbin loader (plugins/redukt-gpu-cuda/README.md:38-70)
 * ---------------------------------------------------------------------------------- */

#define RBIN_MAGIC 0x55504752u
#define FLAG_NORM_BIAS 1u
#define FLAG_UNTIED_HEAD 2u

typedef struct {
    float *norm_w, *norm_b;
    Mat in_proj;
    float *conv_w, *conv_b;
    Mat x_proj;  /* always f32 */
    Mat dt_proj; /* always f32 */
    float *dt_b, *a_log, *d_vec;
    Mat out_proj;
} Layer;

typedef struct OrcModel {
    uint32_t vocab, d, di, ds, dc, dr, nl, flags;
    int profile; /* 0 = F32, 1 = Q8 */
    uint32_t group;
    Mat emb;
    Mat head; /* aliases emb when tied */
    int head_tied;
    float *norm_f_w, *norm_f_b;
    Layer* layers;
} OrcModel;

typedef struct OrcState {
    uint32_t nl, conv_len, ssm_len;
    float* conv; /* nl * conv_len, layout [layer][di][dc-1] like MambaState */
    float* ssm;  /* nl * ssm_len,  layout [layer][di][ds] */
    uint64_t reset_every, since_reset;
} OrcState;

static float* read_f32(FILE* f, size_t n) {
    float* p = (float*)malloc(n * sizeof(float) + 64);
    if (!p) return NULL;
    if (fread(p, sizeof(float), n, f) != n) { free(p); return NULL; }
    return p;
}

static int make_mat(Mat* m, float* data, uint32_t rows, uint32_t cols, int profile, uint32_t group) {
    m->rows = rows;
    m->cols = cols;
    if (profile == 0) {
        m->group = 0;
        m->f = data;
        m->q = NULL;
        m->scales = NULL;
        return 0;
    }
    uint32_t g = orc_q8_effective_group(cols, group);
    m->group = g;
    m->q = (int8_t*)malloc((size_t)rows * cols);
    m->scales = (float*)malloc((size_t)rows * (cols / g) * sizeof(float));
    if (!m->q || !m->scales) return -1;
    q8_quantize(data, rows, cols, g, m->q, m->scales);
    free(data);
    m->f = NULL;
    return 0;
}

static void free_mat(Mat* m) {
    free(m->f);
    free(m->q);
    free(m->scales);
    memset(m, 0, sizeof(*m));
}

ORC_API void orc_model_free(OrcModel* m) {
    if (!m) return;
    for (uint32_t i = 0; m->layers && i < m->nl; i++) {
        Layer* L = &m->layers[i];
        free(L->norm_w); free(L->norm_b); free(L->conv_w); free(L->conv_b);
        free(L->dt_b); free(L->a_log); free(L->d_vec);
        free_mat(&L->in_proj); free_mat(&L->x_proj); free_mat(&L->dt_proj); free_mat(&L->out_proj);
    }
    free(m->layers);
    if (!m->head_tied) free_mat(&m->head);
    free_mat(&m->emb);
    free(m->norm_f_w);
    free(m->norm_f_b);
    free(m);
}

/* profile: 0 = F32, 1 = Q8 weight-only (in_proj, out_proj, embedding/head; model.rs:375-376).
 * group: Q8 columns per scale (64 = the reference's Q8_GROUP, 0 = per-row). */
ORC_API OrcModel* orc_model_load(const char* path, int profile, uint32_t group) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    uint32_t h[11];
    OrcModel* m = NULL;
    if (fread(h, 4, 11, f) != 11 || h[0] != RBIN_MAGIC || (h[1] != 1 && h[1] != 2)) goto fail;
    m = (OrcModel*)calloc(1, sizeof(OrcModel));
    if (!m) goto fail;
    m->vocab = h[2]; m->d = h[3]; m->di = h[4]; m->ds = h[5]; m->dc = h[6]; m->dr = h[7]; m->nl = h[8];
    m->flags = h[9];
    m->profile = profile;
    m->group = profile ? orc_q8_effective_group(m->d, group ? group : 0) : 0;
    if (m->ds != 16 || m->dc < 2 || m->d == 0 || m->di == 0 || m->nl == 0 || m->vocab == 0) goto fail;
    {
        size_t V = m->vocab, d = m->d, di = m->di, ds = m->ds, dc = m->dc, dr = m->dr;
        int nb = (m->flags & FLAG_NORM_BIAS) != 0;
        float* emb = read_f32(f, V * d);
        if (!emb || make_mat(&m->emb, emb, (uint32_t)V, (uint32_t)d, profile, group)) goto fail;
        m->layers = (Layer*)calloc(m->nl, sizeof(Layer));
        if (!m->layers) goto fail;
        for (uint32_t i = 0; i < m->nl; i++) {
            Layer* L = &m->layers[i];
            float* t;
            if (!(L->norm_w = read_f32(f, d))) goto fail;
            if (nb && !(L->norm_b = read_f32(f, d))) goto fail;
            if (!(t = read_f32(f, 2 * di * d)) || make_mat(&L->in_proj, t, (uint32_t)(2 * di), (uint32_t)d, profile, group)) goto fail;
            if (!(L->conv_w = read_f32(f, di * dc))) goto fail;
            if (!(L->conv_b = read_f32(f, di))) goto fail;
            if (!(t = read_f32(f, (dr + 2 * ds) * di)) || make_mat(&L->x_proj, t, (uint32_t)(dr + 2 * ds), (uint32_t)di, 0, 0)) goto fail;
            if (!(t = read_f32(f, di * dr)) || make_mat(&L->dt_proj, t, (uint32_t)di, (uint32_t)dr, 0, 0)) goto fail;
            if (!(L->dt_b = read_f32(f, di))) goto fail;
            if (!(L->a_log = read_f32(f, di * ds))) goto fail;
            if (!(L->d_vec = read_f32(f, di))) goto fail;
            if (!(t = read_f32(f, d * di)) || make_mat(&L->out_proj, t, (uint32_t)d, (uint32_t)di, profile, group)) goto fail;
        }
        if (!(m->norm_f_w = read_f32(f, d))) goto fail;
        if (nb && !(m->norm_f_b = read_f32(f, d))) goto fail;
        if (m->flags & FLAG_UNTIED_HEAD) {
            float* hd = read_f32(f, V * d);
            if (!hd || make_mat(&m->head, hd, (uint32_t)V, (uint32_t)d, profile, group)) goto fail;
            m->head_tied = 0;
        } else {
            m->head = m->emb;
            m->head_tied = 1;
        }
    }
    fclose(f);
    return m;
fail:
    fclose(f);
    if (m) {
        if (m->head_tied) memset(&m->head, 0, sizeof(m->head));
        orc_model_free(m);
    }
    return NULL;
}

/* dims: vocab, d, di, ds, dc, dr, nl, flags, profile, group */
ORC_API void orc_model_dims(const OrcModel* m, uint32_t* out) {
    out[0] = m->vocab; out[1] = m->d; out[2] = m->di; out[3] = m->ds; out[4] = m->dc;
    out[5] = m->dr; out[6] = m->nl; out[7] = m->flags; out[8] = (uint32_t)m->profile; out[9] = m->group;
}

/* Export one quantized matrix: which = 0 emb, 1 head, 2 in_proj(layer), 3 out_proj(layer). */
ORC_API int orc_model_q8(const OrcModel* m, int which, uint32_t layer, int8_t* q, float* scales) {
    const Mat* mt = NULL;
    if (which == 0) mt = &m->emb;
    else if (which == 1) mt = &m->head;
    else if (layer < m->nl) mt = which == 2 ? &m->layers[layer].in_proj : &m->layers[layer].out_proj;
    if (!mt || !mt->group) return -1;
    memcpy(q, mt->q, (size_t)mt->rows * mt->cols);
    memcpy(scales, mt->scales, (size_t)mt->rows * (mt->cols / mt->group) * sizeof(float));
    return 0;
}

ORC_API OrcState* orc_state_new(const OrcModel* m) {
    OrcState* s = (OrcState*)calloc(1, sizeof(OrcState));
    if (!s) return NULL;
    s->nl = m->nl;
    s->conv_len = m->di * (m->dc - 1);
    s->ssm_len = m->di * m->ds;
    s->conv = (float*)calloc((size_t)s->nl * s->conv_len, sizeof(float));
    s->ssm = (float*)calloc((size_t)s->nl * s->ssm_len, sizeof(float));
    if (!s->conv || !s->ssm) { free(s->conv); free(s->ssm); free(s); return NULL; }
    return s;
}

ORC_API void orc_state_free(OrcState* s) {
    if (!s) return;
    free(s->conv);
    free(s->ssm);
    free(s);
}

/* model.rs:298-302 */
ORC_API void orc_state_reset(OrcState* s) {
    memset(s->conv, 0, (size_t)s->nl * s->conv_len * sizeof(float));
    memset(s->ssm, 0, (size_t)s->nl * s->ssm_len * sizeof(float));
    s->since_reset = 0;
}

ORC_API void orc_state_set_reset_every(OrcState* s, uint64_t every) { s->reset_every = every; }

/* Copies the state in the reference layout: conv [layer][di][dc-1], ssm [layer][di][ds]. */
ORC_API void orc_state_export(const OrcState* s, float* conv, float* ssm) {
    if (conv) memcpy(conv, s->conv, (size_t)s->nl * s->conv_len * sizeof(float));
    if (ssm) memcpy(ssm, s->ssm, (size_t)s->nl * s->ssm_len * sizeof(float));
}

/* model.rs:315-320 */
static void maybe_periodic_reset(OrcState* s) {
    if (s->reset_every > 0 && s->since_reset >= s->reset_every) orc_state_reset(s);
    s->since_reset += 1;
}

/* ------------------------------------------------------------------------------------
 * Forward (model.rs:635-752, 773-935)
 * ---------------------------------------------------------------------------------- */

typedef struct {
    float *x, *normed, *xz, *conv_out, *zp, *dt, *y, *gated, *res;
} Scratch;

static int scratch_alloc(Scratch* sc, const OrcModel* m) {
    size_t d = m->d, di = m->di, xr = m->dr + 2 * m->ds;
    sc->x = calloc(d, 4); sc->normed = calloc(d, 4); sc->xz = calloc(2 * di, 4);
    sc->conv_out = calloc(di, 4); sc->zp = calloc(xr, 4); sc->dt = calloc(di, 4);
    sc->y = calloc(di, 4); sc->gated = calloc(di, 4); sc->res = calloc(d, 4);
    return (sc->x && sc->normed && sc->xz && sc->conv_out && sc->zp && sc->dt && sc->y && sc->gated && sc->res) ? 0 : -1;
}

static void scratch_free(Scratch* sc) {
    free(sc->x); free(sc->normed); free(sc->xz); free(sc->conv_out); free(sc->zp);
    free(sc->dt); free(sc->y); free(sc->gated); free(sc->res);
}

/* Embedding row (Q8: dequantize, gemv.rs:284-295). */
static void emb_row(const OrcModel* m, uint32_t tok, float* out) {
    const Mat* e = &m->emb;
    size_t d = m->d;
    if (!e->group) { memcpy(out, e->f + (size_t)tok * d, d * 4); return; }
    uint32_t g = e->group, gpr = (uint32_t)d / g;
    for (uint32_t gi = 0; gi < gpr; gi++) {
        float s = e->scales[(size_t)tok * gpr + gi];
        for (uint32_t c = 0; c < g; c++) out[gi * g + c] = (float)e->q[(size_t)tok * d + gi * g + c] * s;
    }
}

static void layer_norm_step(const OrcModel* m, const Layer* L, Scratch* sc) {
    if (L->norm_b) {
        layer_norm_into(sc->normed, sc->x, L->norm_w, L->norm_b, m->d, 1e-5f);
    } else {
        memcpy(sc->normed, sc->x, m->d * 4);
        rms_norm_into(sc->normed, L->norm_w, m->d, 1e-5f);
    }
}

#define CONV_BLOCK 256
#define SSM_BLOCK 64

/* model.rs:134-153 for channels j0..j0+len of one stream. */
static void conv_silu_block(const OrcModel* m, const Layer* L, size_t j0, size_t len, float* cs, const float* x, float* out) {
    size_t dc = m->dc;
    for (size_t jj = 0; jj < len; jj++) {
        size_t j = j0 + jj;
        float* st = cs + j * (dc - 1);
        const float* w = L->conv_w + j * dc;
        float val = 0.0f;
        for (size_t k = 0; k < dc - 1; k++) val += st[k] * w[k];
        val += x[j] * w[dc - 1];
        val += L->conv_b[j];
        for (size_t k = 0; k + 1 < dc - 1; k++) st[k] = st[k + 1];
        st[dc - 2] = x[j];
        out[j] = val;
    }
    silu_inplace(out + j0, len);
}

/* model.rs:174-190 + tensor.rs:1301-1325 for channels j0..j0+len of one stream. */
static void scan_block(const OrcModel* m, const Layer* L, size_t j0, size_t len, Scratch* sc, float* ss) {
    size_t dr = m->dr, ds = m->ds, di = m->di;
    const float* B = sc->zp + dr;
    const float* C = sc->zp + dr + ds;
    const float* z = sc->xz + di;
    for (size_t jj = 0; jj < len; jj++) {
        size_t j = j0 + jj;
        sc->dt[j] = dot_ref(L->dt_proj.f + j * dr, sc->zp, dr);
    }
    for (size_t jj = 0; jj < len; jj++) {
        size_t j = j0 + jj;
        sc->dt[j] = orc_softplus(sc->dt[j] + L->dt_b[j]);
    }
    for (size_t jj = 0; jj < len; jj++) {
        size_t j = j0 + jj;
        float* st = ss + j * 16;
        float dt = sc->dt[j], xv = sc->conv_out[j];
        if (!(fabsf(dt) < 1e-6f)) {
            float dtx = dt * xv;
            for (int n = 0; n < 16; n++) {
                float a = lane_expf(L->a_log[j * 16 + n]);
                float da = lane_expf(0.0f - dt * a);
                st[n] = da * st[n] + dtx * B[n];
            }
        }
        float lanes[8];
        for (int l = 0; l < 8; l++) lanes[l] = st[l] * C[l] + st[l + 8] * C[l + 8];
        sc->y[j] = hsum_ssm(lanes) + L->d_vec[j] * xv;
    }
    gated_silu_mul(sc->gated + j0, sc->y + j0, z + j0, len);
}

static void final_norm(const OrcModel* m, Scratch* sc) {
    if (m->norm_f_b) {
        memcpy(sc->normed, sc->x, m->d * 4);
        layer_norm_into(sc->x, sc->normed, m->norm_f_w, m->norm_f_b, m->d, 1e-5f);
    } else {
        rms_norm_into(sc->x, m->norm_f_w, m->d, 1e-5f);
    }
}

typedef struct { const OrcModel* m; const Layer* L; uint32_t li; OrcState* const* st; Scratch* sc; } PhaseJob;

static void conv_units(void* ctx, long b, long e) {
    const PhaseJob* p = (const PhaseJob*)ctx;
    size_t di = p->m->di;
    long nblk = (long)((di + CONV_BLOCK - 1) / CONV_BLOCK);
    for (long u = b; u < e; u++) {
        int s = (int)(u / nblk);
        size_t j0 = (size_t)(u % nblk) * CONV_BLOCK;
        size_t len = di - j0 < CONV_BLOCK ? di - j0 : CONV_BLOCK;
        float* cs = p->st[s]->conv + (size_t)p->li * p->st[s]->conv_len;
        conv_silu_block(p->m, p->L, j0, len, cs, p->sc[s].xz, p->sc[s].conv_out);
    }
}

static void scan_units(void* ctx, long b, long e) {
    const PhaseJob* p = (const PhaseJob*)ctx;
    size_t di = p->m->di;
    long sblk = (long)((di + SSM_BLOCK - 1) / SSM_BLOCK);
    for (long u = b; u < e; u++) {
        int s = (int)(u / sblk);
        size_t j0 = (size_t)(u % sblk) * SSM_BLOCK;
        size_t len = di - j0 < SSM_BLOCK ? di - j0 : SSM_BLOCK;
        float* ss = p->st[s]->ssm + (size_t)p->li * p->st[s]->ssm_len;
        scan_block(p->m, p->L, j0, len, &p->sc[s], ss);
    }
}

/* Lockstep step for ns streams (forward_layers_normed_multi + compute_head_multi).  With
 * ns == 1 this is forward_layers_normed + the head: identical arithmetic per stream. */
static void forward_multi(const OrcModel* m, int ns, const uint32_t* tokens, OrcState* const* st, float* logits) {
    size_t d = m->d, di = m->di, dc = m->dc;
    Scratch* sc = (Scratch*)calloc((size_t)ns, sizeof(Scratch));
    const float** xs = (const float**)malloc((size_t)ns * sizeof(float*));
    float** outs = (float**)malloc((size_t)ns * sizeof(float*));
    for (int s = 0; s < ns; s++) scratch_alloc(&sc[s], m);
    for (int s = 0; s < ns; s++) {
        maybe_periodic_reset(st[s]);
        emb_row(m, tokens[s], sc[s].x);
    }
    for (uint32_t li = 0; li < m->nl; li++) {
        const Layer* L = &m->layers[li];
        for (int s = 0; s < ns; s++) layer_norm_step(m, L, &sc[s]);
        for (int s = 0; s < ns; s++) { xs[s] = sc[s].normed; outs[s] = sc[s].xz; }
        gemv_multi(&L->in_proj, ns, xs, outs);
        /* conv phase: units = (stream, 256-channel block) */
        PhaseJob pj = {m, L, li, st, sc};
        long nblk = (long)((di + CONV_BLOCK - 1) / CONV_BLOCK);
        par_for(ns * nblk, (long)ns * (long)di * 64, conv_units, &pj);
        (void)dc;
        for (int s = 0; s < ns; s++) { xs[s] = sc[s].conv_out; outs[s] = sc[s].zp; }
        gemv_multi(&L->x_proj, ns, xs, outs);
        long sblk = (long)((di + SSM_BLOCK - 1) / SSM_BLOCK);
        par_for(ns * sblk, (long)ns * (long)di * 256, scan_units, &pj);
        for (int s = 0; s < ns; s++) { xs[s] = sc[s].gated; outs[s] = sc[s].res; }
        gemv_multi(&L->out_proj, ns, xs, outs);
        for (int s = 0; s < ns; s++)
            for (size_t j = 0; j < d; j++) sc[s].x[j] += sc[s].res[j];
    }
    for (int s = 0; s < ns; s++) final_norm(m, &sc[s]);
    for (int s = 0; s < ns; s++) { xs[s] = sc[s].x; outs[s] = logits + (size_t)s * m->vocab; }
    gemv_multi(&m->head, ns, xs, outs);
    for (int s = 0; s < ns; s++) scratch_free(&sc[s]);
    free(sc);
    free(xs);
    free(outs);
}

ORC_API void orc_forward(const OrcModel* m, uint32_t token, OrcState* st, float* logits) {
    forward_multi(m, 1, &token, &st, logits);
}

ORC_API void orc_forward_multi(const OrcModel* m, uint32_t n, const uint32_t* tokens, OrcState* const* states,
                               float* logits) {
    if (n) forward_multi(m, (int)n, tokens, states, logits);
}

/* tensor.rs:1917-1933 */
ORC_API void orc_softmax(const float* logits, uint32_t n, float* out) {
    float mx = -INFINITY;
    for (uint32_t i = 0; i < n; i++) mx = logits[i] > mx ? logits[i] : (mx != mx ? logits[i] : mx);
    if (mx == -INFINITY) {
        float u = 1.0f / (float)n;
        for (uint32_t i = 0; i < n; i++) out[i] = u;
        return;
    }
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; i++) {
        float e = orc_expf(logits[i] - mx);
        out[i] = e;
        sum += e;
    }
    float denom = sum > 1.1920929e-07f ? sum : 1.1920929e-07f;
    for (uint32_t i = 0; i < n; i++) out[i] /= denom;
}

/* Thread count of the pool; only effective before the first parallel call. */
ORC_API void orc_set_threads(int n) {
    if (!g_pool.started) g_req_threads = n;
}

ORC_API int orc_get_threads(void) {
    pool_start();
    return g_pool.nthreads;
}
