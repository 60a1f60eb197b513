/*
 * rwkv7_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * CPU restatement of the redukt reference's RWKV-7 single-token decode step
 * (`Rwkv7Model::forward_into`, src/infrastructure/rwkv7/model.rs:643-698) with its
 * default W8A8 quantisation (`AUTO_QUANT = Q8`, model.rs:245), used only as the parity
 * checker of the engine's RWKV-7 kernels and as the CPU baseline leg of bench.py.
 *
 * Operation order follows the reference:
 *   forward_into              rwkv7/model.rs:643-698  (LN1 -> time mix -> residual, LN2 -> channel mix)
 *   time_mixing_scratch       rwkv7/model.rs:802-916  (token shift, W8A8 r/k/v, LoRAs, WKV-7 state, GN, bonus)
 *   channel_mixing_scratch    rwkv7/model.rs:919-925
 *   Rwkv7Model::load (HF)     rwkv7/model.rs:249-329  (embedding pre-normalised with ln0 at load)
 *   Rwkv7State::reset         rwkv7/model.rs:136-141
 *   Q8Tensor::from_f32        src/domain/tensor.rs:113-135   (per-row abs-max / 127, round half away, clamp)
 *   quantize_vec_i8_into      src/domain/tensor.rs:1791-1800
 *   q8_mat_vec_mul_*          src/domain/tensor.rs:1819-1867 (exact int32 dot, sum * (scale_r * v_scale))
 *   mat_vec_mul_into (F32)    src/domain/tensor.rs:1602-1705 (8 lanes, hsum, no FMA) -- dot_ref
 *   sub/add_scaled/mul_into   src/domain/tensor.rs:739-755
 *   tanh/sigmoid_inplace      src/domain/tensor.rs:1007-1036 (lane functions on the 8-aligned body, portable tail)
 *   sigmoid_add_into          src/domain/tensor.rs:1040-1058
 *   decay_sigmoid_into        src/domain/tensor.rs:1082-1101
 *   sigmoid_mix_inplace       src/domain/tensor.rs:1128-1150
 *   squared_relu_into         src/domain/tensor.rs:1386-1388
 *   layer_norm_into           src/domain/tensor.rs:1390-1398
 *   group_norm_into           src/domain/tensor.rs:1400-1414
 *   l2_normalize_per_head     src/domain/tensor.rs:1416-1424
 *   outer_product_into        src/domain/tensor.rs:1869-1877
 *   mat_vec_mul_small_into    src/domain/tensor.rs:1892-1898
 *
 * The int32 dots are exact, so the AVX2 int8 dot below gives the scalar loop's bits.
 * Compile with -ffp-contract=off (Rust never contracts a * b + c).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

#define ORC_API __attribute__((visibility("default")))
#include "oracle_internal.h"

#define RW_MAGIC 0x55504752u
#define RW_VERSION 3u
#define RW_FLAG_RWKV7 (1u << 4)
#define RW_FLAG_G1K (1u << 5)

/* ------------------------------------------------------------------------------------
 * Element-wise helpers (tensor.rs:739-755, 1007-1150, 1386-1424)
 * ---------------------------------------------------------------------------------- */

static inline size_t body_len(size_t n) { return n / 8 * 8; }            /* simd_body_len, tensor.rs:895-897 */
static inline float lane_tanhf(float x) { return orc_lane_sigmoidf(x * 2.0f) * 2.0f - 1.0f; } /* tensor.rs:889-891 */
static inline float portable_tanhf(float x) { return 2.0f * portable_sigmoidf(2.0f * x) - 1.0f; } /* tensor.rs:847-849 */

ORC_API void rw_tanh_inplace(float* x, size_t n) {
    size_t body = body_len(n);
    for (size_t i = 0; i < n; i++) x[i] = i < body ? lane_tanhf(x[i]) : portable_tanhf(x[i]);
}

ORC_API void rw_sigmoid_inplace(float* x, size_t n) {
    size_t body = body_len(n);
    for (size_t i = 0; i < n; i++) x[i] = i < body ? orc_lane_sigmoidf(x[i]) : portable_sigmoidf(x[i]);
}

ORC_API void rw_sigmoid_add_into(float* out, const float* base, const float* off, size_t n) {
    size_t body = body_len(n);
    for (size_t i = 0; i < n; i++) {
        float s = base[i] + off[i];
        out[i] = i < body ? orc_lane_sigmoidf(s) : portable_sigmoidf(s);
    }
}

ORC_API void rw_decay_sigmoid_into(float* out, const float* base, const float* off, size_t n) {
    size_t body = body_len(n);
    for (size_t i = 0; i < n; i++) {
        float s = base[i] + off[i];
        out[i] = i < body ? lane_expf(-0.606531f * orc_lane_sigmoidf(s)) : orc_expf(-0.606531f * portable_sigmoidf(s));
    }
}

ORC_API void rw_sigmoid_mix_inplace(float* v_out, const float* v_first, const float* base, const float* off, size_t n) {
    size_t body = body_len(n);
    for (size_t i = 0; i < n; i++) {
        float s = base[i] + off[i];
        float mix = i < body ? orc_lane_sigmoidf(s) : portable_sigmoidf(s);
        v_out[i] += (v_first[i] - v_out[i]) * mix;
    }
}

static void group_norm_into(float* out, const float* x, size_t groups, size_t n, const float* w, const float* b, float eps) {
    size_t gs = n / groups;
    for (size_t g = 0; g < groups; g++) {
        const float* s = x + g * gs;
        float sum = 0.0f;
        for (size_t i = 0; i < gs; i++) sum += s[i];
        float mean = sum / (float)gs;
        float var = 0.0f;
        for (size_t i = 0; i < gs; i++) var += (s[i] - mean) * (s[i] - mean);
        var = var / (float)gs;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (size_t i = g * gs; i < g * gs + gs; i++) out[i] = (x[i] - mean) * inv_std * w[i] + b[i];
    }
}

static void l2_normalize_per_head(float* x, size_t heads, size_t hs) {
    for (size_t h = 0; h < heads; h++) {
        float* s = x + h * hs;
        float sq = 0.0f;
        for (size_t i = 0; i < hs; i++) sq += s[i] * s[i];
        float norm = sqrtf(sq);
        float inv = norm > 1e-12f ? 1.0f / norm : 0.0f;
        for (size_t i = 0; i < hs; i++) s[i] *= inv;
    }
}

/* ------------------------------------------------------------------------------------
 * W8A8 (tensor.rs:105-206, 1790-1867)
 * ---------------------------------------------------------------------------------- */

typedef struct { int8_t* q; float* s; uint32_t rows, cols; } RwQ8;

/* Q8Tensor::from_f32: one scale per row. */
ORC_API void rw_q8_quantize_rows(const float* w, uint32_t rows, uint32_t cols, int8_t* q, float* scales) {
    for (uint32_t r = 0; r < rows; r++) {
        const float* row = w + (size_t)r * cols;
        float amax = 0.0f;
        for (uint32_t c = 0; c < cols; c++) amax = fmaxf(amax, fabsf(row[c]));
        float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
        float inv = 1.0f / scale;
        scales[r] = scale;
        for (uint32_t c = 0; c < cols; c++) {
            float v = roundf(row[c] * inv);
            v = v != v ? 0.0f : (v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v));  /* Rust `as i8`: NaN -> 0 */
            q[(size_t)r * cols + c] = (int8_t)v;
        }
    }
}

/* quantize_vec_i8_into: one scale for the whole activation vector. */
ORC_API float rw_quantize_vec(const float* v, uint32_t n, int8_t* q) {
    float amax = 0.0f;
    for (uint32_t i = 0; i < n; i++) { float a = fabsf(v[i]); if (a > amax) amax = a; }
    float scale = amax > 0.0f ? amax / 127.0f : 1.0f;
    float inv = 1.0f / scale;
    for (uint32_t i = 0; i < n; i++) {
        float x = roundf(v[i] * inv);
        x = x != x ? 0.0f : (x < -127.0f ? -127.0f : (x > 127.0f ? 127.0f : x));
        q[i] = (int8_t)x;
    }
    return scale;
}

static int32_t dot_i8_scalar(const int8_t* a, const int8_t* b, uint32_t n) {
    int32_t s = 0;
    for (uint32_t i = 0; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

#if defined(__x86_64__)
__attribute__((target("avx2"))) static int32_t dot_i8_avx2(const int8_t* a, const int8_t* b, uint32_t n) {
    __m256i acc = _mm256_setzero_si256();
    uint32_t i = 0;
    for (; i + 16 <= n; i += 16) {
        __m256i x = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i)));
        __m256i y = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + i)));
        acc = _mm256_add_epi32(acc, _mm256_madd_epi16(x, y));
    }
    int32_t lanes[8];
    _mm256_storeu_si256((__m256i*)lanes, acc);
    int32_t s = 0;
    for (int l = 0; l < 8; l++) s += lanes[l];
    for (; i < n; i++) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}
#endif

static inline int32_t dot_i8(const int8_t* a, const int8_t* b, uint32_t n) {
#if defined(__x86_64__)
    if (use_avx2()) return dot_i8_avx2(a, b, n);
#endif
    return dot_i8_scalar(a, b, n);
}

/* q8_mat_vec_mul_into: quantise the vector, exact int32 dot per row, one rounding. */
static void q8_mat_vec(const RwQ8* m, const float* v, float* out, int8_t* vq) {
    float vs = rw_quantize_vec(v, m->cols, vq);
    for (uint32_t r = 0; r < m->rows; r++) {
        int32_t sum = dot_i8(m->q + (size_t)r * m->cols, vq, m->cols);
        out[r] = (float)sum * (m->s[r] * vs);
    }
}

ORC_API void rw_gemv_w8a8(const int8_t* q, const float* scales, uint32_t rows, uint32_t cols, const float* v, float* out) {
    int8_t* vq = (int8_t*)malloc(cols ? cols : 1);
    RwQ8 m = {(int8_t*)q, (float*)scales, rows, cols};
    q8_mat_vec(&m, v, out, vq);
    free(vq);
}

/* mat_vec_mul_into for the F32 LoRA matrices ([rows][cols], HF layout). */
static void f32_mat_vec(const float* w, uint32_t rows, uint32_t cols, const float* v, float* out) {
    for (uint32_t r = 0; r < rows; r++) out[r] = dot_ref(w + (size_t)r * cols, v, cols);
}

/* ------------------------------------------------------------------------------------
 * Model and state
 * ---------------------------------------------------------------------------------- */

typedef struct {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
    const float *x_r, *x_w, *x_k, *x_v, *x_a, *x_g;
    const float *w0, *w1, *w2, *a0, *a1, *a2, *v0, *v1, *v2, *g1, *g2;
    const float *k_k, *k_a, *r_k, *ln_x_w, *ln_x_b, *ffn_x_k;
    RwQ8 rq, kq, vq, oq, fk, fv;
} RwLayer;

typedef struct RwModel {
    uint32_t V, D, H, N, F, L, lw, la, lv, lg, g1k;
    uint32_t lmax;   /* max LoRA rank: the length of the reference's lora_tmp scratch (model.rs:625-631) */
    float* blob;     /* every f32 array of the file */
    float* emb;      /* [V][D], pre-normalised by ln0 */
    const float *ln_out_w, *ln_out_b;
    RwLayer* layers;
    RwQ8 head;
    int8_t* qblob;
    float* sblob;
} RwModel;

typedef struct RwState {
    float* x_att;    /* [L][D] */
    float* wkv;      /* [L][H][N][N] */
    float* x_ffn;    /* [L][D] */
    float* v_first;  /* [D] */
    uint64_t since, every;
} RwState;

ORC_API void rw_model_free(RwModel* m) {
    if (!m) return;
    free(m->blob);
    free(m->qblob);
    free(m->sblob);
    free(m->layers);
    free(m);
}

/* Number of f32 values in the file after the header, in file order. */
static size_t rw_float_count(const RwModel* m) {
    size_t D = m->D, F = m->F;
    size_t per_layer = 4 * D + 6 * D + (D + 2 * (size_t)m->lw * D) + (D + 2 * (size_t)m->la * D) +
                       (D + 2 * (size_t)m->lv * D) + 2 * (size_t)m->lg * D + 3 * D + 4 * D * D + 2 * D + D + 2 * F * D;
    return (size_t)m->V * D + 2 * D + per_layer * m->L + 2 * D + (size_t)m->V * D;
}

ORC_API RwModel* rw_model_load(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    uint32_t h[19];
    if (fread(h, 4, 19, f) != 19 || h[0] != RW_MAGIC || h[1] != RW_VERSION || !(h[9] & RW_FLAG_RWKV7)) { fclose(f); return NULL; }
    RwModel* m = (RwModel*)calloc(1, sizeof(RwModel));
    m->V = h[2]; m->D = h[3]; m->F = h[4]; m->N = h[5]; m->H = h[6]; m->L = h[8];
    m->lw = h[11]; m->la = h[12]; m->lv = h[13]; m->lg = h[14];
    m->g1k = (h[9] & RW_FLAG_G1K) ? 1 : 0;
    m->lmax = m->lw;
    if (m->la > m->lmax) m->lmax = m->la;
    if (m->lv > m->lmax) m->lmax = m->lv;
    if (m->lg > m->lmax) m->lmax = m->lg;
    if (m->H * m->N != m->D || !m->V || !m->L || !m->F) { fclose(f); free(m); return NULL; }
    size_t nf = rw_float_count(m);
    m->blob = (float*)malloc(nf * sizeof(float));
    if (!m->blob || fread(m->blob, sizeof(float), nf, f) != nf) { fclose(f); rw_model_free(m); return NULL; }
    fclose(f);

    size_t D = m->D, F = m->F, V = m->V;
    float* p = m->blob;
    m->emb = p; p += V * D;
    const float* ln0_w = p; p += D;
    const float* ln0_b = p; p += D;
    /* Rwkv7Model::load: every embedding row goes through ln0 once, at load (model.rs:266-275). */
    float* tmp = (float*)malloc(D * sizeof(float));
    for (size_t r = 0; r < V; r++) {
        layer_norm_into(tmp, m->emb + r * D, ln0_w, ln0_b, D, 1e-5f);
        memcpy(m->emb + r * D, tmp, D * sizeof(float));
    }
    free(tmp);

    size_t qcount = V * D + (size_t)m->L * (4 * D * D + 2 * F * D);
    size_t scount = V + (size_t)m->L * (4 * D + F + D);
    m->qblob = (int8_t*)malloc(qcount);
    m->sblob = (float*)malloc(scount * sizeof(float));
    m->layers = (RwLayer*)calloc(m->L, sizeof(RwLayer));
    int8_t* qp = m->qblob;
    float* sp = m->sblob;
#define TAKE(n) (p += (n), p - (n))
#define QUANT(dst, rows_, cols_, src) do { (dst).rows = (rows_); (dst).cols = (cols_); (dst).q = qp; (dst).s = sp; \
        rw_q8_quantize_rows((src), (rows_), (cols_), qp, sp); qp += (size_t)(rows_) * (cols_); sp += (rows_); } while (0)
    for (uint32_t l = 0; l < m->L; l++) {
        RwLayer* y = &m->layers[l];
        y->ln1_w = TAKE(D); y->ln1_b = TAKE(D); y->ln2_w = TAKE(D); y->ln2_b = TAKE(D);
        y->x_r = TAKE(D); y->x_w = TAKE(D); y->x_k = TAKE(D); y->x_v = TAKE(D); y->x_a = TAKE(D); y->x_g = TAKE(D);
        y->w0 = TAKE(D); y->w1 = TAKE((size_t)m->lw * D); y->w2 = TAKE(D * m->lw);
        y->a0 = TAKE(D); y->a1 = TAKE((size_t)m->la * D); y->a2 = TAKE(D * m->la);
        y->v0 = TAKE(D); y->v1 = TAKE((size_t)m->lv * D); y->v2 = TAKE(D * m->lv);
        y->g1 = TAKE((size_t)m->lg * D); y->g2 = TAKE(D * m->lg);
        y->k_k = TAKE(D); y->k_a = TAKE(D); y->r_k = TAKE(D);
        const float* wr = TAKE(D * D); const float* wk = TAKE(D * D);
        const float* wv = TAKE(D * D); const float* wo = TAKE(D * D);
        QUANT(y->rq, D, D, wr); QUANT(y->kq, D, D, wk); QUANT(y->vq, D, D, wv); QUANT(y->oq, D, D, wo);
        y->ln_x_w = TAKE(D); y->ln_x_b = TAKE(D);
        y->ffn_x_k = TAKE(D);
        const float* fk = TAKE(F * D); const float* fv = TAKE(D * F);
        QUANT(y->fk, F, D, fk); QUANT(y->fv, D, F, fv);
    }
    m->ln_out_w = TAKE(D); m->ln_out_b = TAKE(D);
    const float* head = TAKE(V * D);
    QUANT(m->head, V, D, head);
#undef TAKE
#undef QUANT
    return m;
}

/* dims: V, D, H, N, F, L, lw, la, lv, lg, g1k */
ORC_API void rw_model_dims(const RwModel* m, uint32_t* out) {
    uint32_t d[11] = {m->V, m->D, m->H, m->N, m->F, m->L, m->lw, m->la, m->lv, m->lg, m->g1k};
    memcpy(out, d, sizeof(d));
}

/* which: 0 r, 1 k, 2 v, 3 o, 4 ffn key, 5 ffn value, 6 head. Returns rows*cols or 0. */
ORC_API size_t rw_model_q8(const RwModel* m, int which, uint32_t layer, int8_t* q, float* scales) {
    const RwQ8* x = NULL;
    if (which == 6) x = &m->head;
    else if (layer < m->L) {
        const RwLayer* y = &m->layers[layer];
        const RwQ8* t[6] = {&y->rq, &y->kq, &y->vq, &y->oq, &y->fk, &y->fv};
        if (which >= 0 && which < 6) x = t[which];
    }
    if (!x) return 0;
    size_t n = (size_t)x->rows * x->cols;
    if (q) memcpy(q, x->q, n);
    if (scales) memcpy(scales, x->s, x->rows * sizeof(float));
    return n;
}

ORC_API const float* rw_model_embedding(const RwModel* m) { return m->emb; }

ORC_API RwState* rw_state_new(const RwModel* m) {
    RwState* s = (RwState*)calloc(1, sizeof(RwState));
    s->x_att = (float*)calloc((size_t)m->L * m->D, sizeof(float));
    s->wkv = (float*)calloc((size_t)m->L * m->H * m->N * m->N, sizeof(float));
    s->x_ffn = (float*)calloc((size_t)m->L * m->D, sizeof(float));
    s->v_first = (float*)calloc(m->D, sizeof(float));
    return s;
}

ORC_API void rw_state_free(RwState* s) {
    if (!s) return;
    free(s->x_att); free(s->wkv); free(s->x_ffn); free(s->v_first); free(s);
}

/* Rwkv7State::reset (model.rs:136-141); also restarts the periodic-reset counter. */
ORC_API void rw_state_reset(const RwModel* m, RwState* s) {
    memset(s->x_att, 0, (size_t)m->L * m->D * sizeof(float));
    memset(s->wkv, 0, (size_t)m->L * m->H * m->N * m->N * sizeof(float));
    memset(s->x_ffn, 0, (size_t)m->L * m->D * sizeof(float));
    memset(s->v_first, 0, m->D * sizeof(float));
    s->since = 0;
}

ORC_API void rw_state_set_reset_every(RwState* s, uint64_t every) { s->every = every; }

ORC_API void rw_state_export(const RwModel* m, const RwState* s, float* x_att, float* wkv, float* x_ffn, float* v_first) {
    if (x_att) memcpy(x_att, s->x_att, (size_t)m->L * m->D * sizeof(float));
    if (wkv) memcpy(wkv, s->wkv, (size_t)m->L * m->H * m->N * m->N * sizeof(float));
    if (x_ffn) memcpy(x_ffn, s->x_ffn, (size_t)m->L * m->D * sizeof(float));
    if (v_first) memcpy(v_first, s->v_first, m->D * sizeof(float));
}

/* ------------------------------------------------------------------------------------
 * Forward (model.rs:643-698, 802-925)
 * ---------------------------------------------------------------------------------- */

typedef struct {
    float *x, *ln, *xx, *xr, *xw, *xk, *xv, *xa, *xg, *r, *k, *v, *lora_tmp, *lora_d, *w, *a, *g;
    float *kk, *k_mod, *v_out, *out_vec, *out_norm, *gated, *tm_out, *cm_out, *ffn, *kk_a, *neg_kk, *out_h, *s_ab;
    int8_t* vq;
    float* mem;
} RwScratch;

static void scratch_init(RwScratch* s, const RwModel* m) {
    size_t D = m->D, F = m->F, N = m->N;
    size_t lmax = m->lmax;
    size_t total = 25 * D + lmax + F + 3 * N + N * N;
    s->mem = (float*)calloc(total, sizeof(float));
    float* p = s->mem;
    float** vecs[] = {&s->x, &s->ln, &s->xx, &s->xr, &s->xw, &s->xk, &s->xv, &s->xa, &s->xg, &s->r, &s->k, &s->v,
                      &s->lora_d, &s->w, &s->a, &s->g, &s->kk, &s->k_mod, &s->v_out, &s->out_vec, &s->out_norm,
                      &s->gated, &s->tm_out, &s->cm_out};
    for (size_t i = 0; i < sizeof(vecs) / sizeof(vecs[0]); i++) { *vecs[i] = p; p += D; }
    s->lora_tmp = p; p += lmax;
    s->ffn = p; p += F;
    s->kk_a = p; p += N;
    s->neg_kk = p; p += N;
    s->out_h = p; p += N;
    s->s_ab = p;
    s->vq = (int8_t*)malloc(F > D ? F : D);
}

static void scratch_free(RwScratch* s) { free(s->mem); free(s->vq); }

static void time_mixing(const RwModel* m, RwScratch* s, uint32_t layer, const float* x_prev, const float* v_first, float* state) {
    const RwLayer* w = &m->layers[layer];
    size_t D = m->D, H = m->H, N = m->N;
    /* Step 1: token shift */
    for (size_t i = 0; i < D; i++) s->xx[i] = x_prev[i] - s->ln[i];
    for (size_t i = 0; i < D; i++) {
        s->xr[i] = s->ln[i] + s->xx[i] * w->x_r[i];
        s->xw[i] = s->ln[i] + s->xx[i] * w->x_w[i];
        s->xk[i] = s->ln[i] + s->xx[i] * w->x_k[i];
        s->xv[i] = s->ln[i] + s->xx[i] * w->x_v[i];
        s->xa[i] = s->ln[i] + s->xx[i] * w->x_a[i];
        s->xg[i] = s->ln[i] + s->xx[i] * w->x_g[i];
    }
    /* Step 2: W8A8 projections */
    q8_mat_vec(&w->rq, s->xr, s->r, s->vq);
    q8_mat_vec(&w->kq, s->xk, s->k, s->vq);
    q8_mat_vec(&w->vq, s->xv, s->v, s->vq);
    /* Step 3: decay */
    /* the activations run over the whole max-rank scratch (model.rs:830, 845), so its 8-aligned
     * body decides where the lane functions stop; entries past a LoRA's rank are never read */
    f32_mat_vec(w->w1, m->lw, D, s->xw, s->lora_tmp);
    rw_tanh_inplace(s->lora_tmp, m->lmax);
    f32_mat_vec(w->w2, D, m->lw, s->lora_tmp, s->lora_d);
    rw_decay_sigmoid_into(s->w, w->w0, s->lora_d, D);
    /* Step 4: a gate */
    f32_mat_vec(w->a1, m->la, D, s->xa, s->lora_tmp);
    f32_mat_vec(w->a2, D, m->la, s->lora_tmp, s->lora_d);
    rw_sigmoid_add_into(s->a, w->a0, s->lora_d, D);
    /* Step 5: output gate */
    f32_mat_vec(w->g1, m->lg, D, s->xg, s->lora_tmp);
    rw_sigmoid_inplace(s->lora_tmp, m->lmax);
    f32_mat_vec(w->g2, D, m->lg, s->lora_tmp, s->g);
    /* Step 6: key normalisation */
    for (size_t i = 0; i < D; i++) s->kk[i] = s->k[i] * w->k_k[i];
    l2_normalize_per_head(s->kk, H, N);
    /* Step 7: key modification */
    for (size_t i = 0; i < D; i++) s->k_mod[i] = s->k[i] * (1.0f + (s->a[i] - 1.0f) * w->k_a[i]);
    /* Step 8: value mixing */
    memcpy(s->v_out, s->v, D * sizeof(float));
    if (layer != 0) {
        f32_mat_vec(w->v1, m->lv, D, s->xv, s->lora_tmp);
        f32_mat_vec(w->v2, D, m->lv, s->lora_tmp, s->lora_d);
        rw_sigmoid_mix_inplace(s->v_out, v_first, w->v0, s->lora_d, D);
    }
    /* Step 9: WKV-7 state update per head */
    for (size_t h = 0; h < H; h++) {
        float* S = state + h * N * N;
        size_t hd = h * N;
        for (size_t j = 0; j < N; j++) s->kk_a[j] = s->kk[hd + j] * s->a[hd + j];
        for (size_t j = 0; j < N; j++) s->neg_kk[j] = -s->kk[hd + j];
        for (size_t i = 0; i < N; i++) {
            float sum = 0.0f;
            for (size_t j = 0; j < N; j++) sum += S[i * N + j] * s->neg_kk[j];
            s->out_h[i] = sum;
        }
        for (size_t i = 0; i < N; i++)
            for (size_t j = 0; j < N; j++) s->s_ab[i * N + j] = s->out_h[i] * s->kk_a[j];
        for (size_t i = 0; i < N; i++)
            for (size_t j = 0; j < N; j++) {
                size_t idx = i * N + j;
                S[idx] = S[idx] * s->w[hd + j] + s->s_ab[idx] + s->v_out[hd + i] * s->k_mod[hd + j];
            }
        for (size_t i = 0; i < N; i++) {
            float sum = 0.0f;
            for (size_t j = 0; j < N; j++) sum += S[i * N + j] * s->r[hd + j];
            s->out_vec[hd + i] = sum;
        }
    }
    /* Step 10: GroupNorm */
    group_norm_into(s->out_norm, s->out_vec, H, D, w->ln_x_w, w->ln_x_b, 64e-5f);
    /* Step 11: bonus */
    const float* k_src = m->g1k ? s->k_mod : s->k;
    for (size_t h = 0; h < H; h++) {
        size_t hd = h * N;
        float bonus = 0.0f;
        for (size_t j = 0; j < N; j++) bonus += s->r[hd + j] * k_src[hd + j] * w->r_k[hd + j];
        for (size_t j = 0; j < N; j++) s->out_norm[hd + j] += bonus * s->v_out[hd + j];
    }
    /* Step 12: gate and output projection */
    for (size_t i = 0; i < D; i++) s->gated[i] = s->out_norm[i] * s->g[i];
    q8_mat_vec(&w->oq, s->gated, s->tm_out, s->vq);
}

static void channel_mixing(const RwModel* m, RwScratch* s, uint32_t layer, const float* x_prev) {
    const RwLayer* w = &m->layers[layer];
    size_t D = m->D;
    for (size_t i = 0; i < D; i++) s->xx[i] = x_prev[i] - s->ln[i];
    for (size_t i = 0; i < D; i++) s->xr[i] = s->ln[i] + s->xx[i] * w->ffn_x_k[i];
    q8_mat_vec(&w->fk, s->xr, s->ffn, s->vq);
    for (size_t i = 0; i < m->F; i++) { float r = fmaxf(s->ffn[i], 0.0f); s->ffn[i] = r * r; }
    q8_mat_vec(&w->fv, s->ffn, s->cm_out, s->vq);
}

static void forward_one(const RwModel* m, RwScratch* s, uint32_t token, RwState* st, float* logits) {
    size_t D = m->D, NN = (size_t)m->H * m->N * m->N;
    if (st->every > 0 && st->since >= st->every) rw_state_reset(m, st);
    st->since++;
    memcpy(s->x, m->emb + (size_t)token * D, D * sizeof(float));
    for (uint32_t l = 0; l < m->L; l++) {
        const RwLayer* w = &m->layers[l];
        layer_norm_into(s->ln, s->x, w->ln1_w, w->ln1_b, D, 1e-5f);
        time_mixing(m, s, l, st->x_att + l * D, st->v_first, st->wkv + l * NN);
        memcpy(st->x_att + l * D, s->ln, D * sizeof(float));
        if (l == 0) memcpy(st->v_first, s->v, D * sizeof(float));
        for (size_t i = 0; i < D; i++) s->x[i] += s->tm_out[i];
        layer_norm_into(s->ln, s->x, w->ln2_w, w->ln2_b, D, 1e-5f);
        channel_mixing(m, s, l, st->x_ffn + l * D);
        memcpy(st->x_ffn + l * D, s->ln, D * sizeof(float));
        for (size_t i = 0; i < D; i++) s->x[i] += s->cm_out[i];
    }
    layer_norm_into(s->ln, s->x, m->ln_out_w, m->ln_out_b, D, 1e-5f);
    q8_mat_vec(&m->head, s->ln, logits, s->vq);
}

ORC_API void rw_forward(const RwModel* m, uint32_t token, RwState* st, float* logits) {
    RwScratch s;
    scratch_init(&s, m);
    forward_one(m, &s, token, st, logits);
    scratch_free(&s);
}

typedef struct {
    const RwModel* m;
    const uint32_t* tokens;
    RwState* const* states;
    float* logits;
    uint32_t steps;      /* tokens per stream, stream-major: tokens[b * steps + t] */
    float* last_only;    /* when non-NULL, logits of the last step only */
} MultiCtx;

static void multi_worker(void* ctx, long b0, long b1) {
    MultiCtx* c = (MultiCtx*)ctx;
    RwScratch s;
    scratch_init(&s, c->m);
    size_t V = c->m->V;
    float* tmp = c->last_only ? (float*)malloc(V * sizeof(float)) : NULL;
    for (long b = b0; b < b1; b++)
        for (uint32_t t = 0; t < c->steps; t++) {
            float* out = c->last_only ? (t + 1 == c->steps ? c->last_only + (size_t)b * V : tmp)
                                      : c->logits + ((size_t)b * c->steps + t) * V;
            forward_one(c->m, &s, c->tokens[(size_t)b * c->steps + t], c->states[b], out);
        }
    free(tmp);
    scratch_free(&s);
}

/* n streams advanced by one token each; streams run on the pool's threads, each stream
 * in the reference's single-stream order (RWKV has no lockstep path: model_loader.rs:218-223). */
ORC_API void rw_forward_multi(const RwModel* m, uint32_t n, const uint32_t* tokens, RwState* const* states, float* logits) {
    MultiCtx c = {m, tokens, states, logits, 1, NULL};
    par_for(n, (long)n * 1000000, multi_worker, &c);
}

/* n streams advanced by `steps` tokens each (tokens stream-major); only the last step's logits
 * are written when last_only != 0.  Used by the timed CPU baseline. */
ORC_API void rw_run_streams(const RwModel* m, uint32_t n, uint32_t steps, const uint32_t* tokens,
                            RwState* const* states, float* logits, int last_only) {
    MultiCtx c = {m, tokens, states, last_only ? NULL : logits, steps, last_only ? logits : NULL};
    par_for(n, (long)n * 1000000, multi_worker, &c);
}
