// RWKV-7 decode-step kernels (sm_100a), n streams per step.
//
// The reference's RWKV-7 step (src/infrastructure/rwkv7/model.rs:643-925) is single-stream
// CPU code with W8A8 projections.  Its int8 x int8 dots are exact, and everything else is a
// fixed sequence of IEEE operations, so these kernels reproduce the reference's bits: every
// element-wise step is written with explicitly rounded operations in the reference's order,
// every reduction the reference runs sequentially (LayerNorm, GroupNorm, L2 norm, the bonus
// and the 64-wide state mat-vecs) runs sequentially in one thread, the F32 LoRA mat-vecs keep
// the reference's 8-lane order (tensor.rs:1663-1705), and the W8A8 dots are int32 sums
// (dp4a or tcgen05 kind::i8), whose order does not matter.
//
// One step, per layer:
//   k_rw_ln_mix    LayerNorm + token shift + mixes; quantises xr/xk/xv (W8A8 activations)
//   k_rw_w8a8_*    r, k, v projections (one launch, three jobs)
//   k_rw_lora1     F32 LoRA down-projections (decay, a, v, gate) with tanh / sigmoid
//   k_rw_wkv       per (head, streams): LoRA up-projections, decay, a, v mix, gate, key
//                  normalisation, the WKV-7 64x64 state update, GroupNorm, bonus, gate
//   k_rw_quant     quantises the gated vector
//   k_rw_w8a8_*    output projection + residual
//   k_rw_ln_mix    LayerNorm + channel-mix shift; quantises xk
//   k_rw_w8a8_*    FFN key with squared ReLU
//   k_rw_quant     quantises the FFN activation
//   k_rw_w8a8_*    FFN value + residual
// then k_rw_ln_mix (final LayerNorm, quantised) and the W8A8 head.
#pragma once
#include "rk_kernels.cuh"
#include "rk_tc.cuh"

namespace rk {
namespace rw {

constexpr int kHS = 64;  // head size of every RWKV-7 configuration (rwkv7/model.rs:24-38)

// Tiled int8 activations: [K/64][16-stream block][16][64 B] in the 64-byte swizzle, the B-operand
// layout of the tensor-core projection (one plane of the Mamba digit layout).
__host__ __device__ __forceinline__ size_t aq_off(int cap_pad, int b, int k) {
    return (((size_t)(k >> 6) * (cap_pad >> 4) + (b >> 4)) * 16 + (b & 15)) * 64 + swz64((uint32_t)b, (uint32_t)(k & 63));
}

// ---- Element-wise functions of tensor.rs ---------------------------------------------------

// portable_sigmoidf (tensor.rs:841-843)
__device__ __forceinline__ float portable_sigmoid(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, portable_expf(-x)));
}

// The AVX2 kernels use the lane functions on the first len/8*8 elements and the portable ones on
// the rest (tensor.rs:1016-1020, 1050-1057, 1092-1101, 1136-1143).
__device__ __forceinline__ float sigmoid_at(float x, bool lane) { return lane ? lane_sigmoid(x) : portable_sigmoid(x); }

// lane_tanhf / portable_tanhf (tensor.rs:889-891, 847-849)
__device__ __forceinline__ float tanh_at(float x, bool lane) {
    if (lane) return __fsub_rn(__fmul_rn(lane_sigmoid(__fmul_rn(x, 2.0f)), 2.0f), 1.0f);
    return __fsub_rn(__fmul_rn(2.0f, portable_sigmoid(__fmul_rn(2.0f, x))), 1.0f);
}

// decay_sigmoid_into (tensor.rs:1082-1101): exp(-0.606531 * sigmoid(base + offset))
__device__ __forceinline__ float decay_at(float s, bool lane) {
    if (lane) return lane_expf(__fmul_rn(-0.606531f, lane_sigmoid(s)));
    return portable_expf(__fmul_rn(-0.606531f, portable_sigmoid(s)));
}

// Sequential sum from +0 (Rust's f32 `Sum`, a left fold).
__device__ __forceinline__ float seq_sum(const float* p, int n) {
    float s = 0.0f;
#pragma unroll 8
    for (int i = 0; i < n; i++) s = __fadd_rn(s, p[i]);
    return s;
}

// dot_avx2_order (tensor.rs:1680-1693): 8 lanes over the 8-aligned body, lane l accumulating
// columns c = l (mod 8) from +0 with one multiply and one add each, the hsum tree
// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)), then the tail added sequentially.
__device__ __forceinline__ float dot8(const float* w, const float* v, int len) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = 0.0f;
    const int body = len & ~7;
    for (int c = 0; c < body; c += 8) {
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = __fadd_rn(acc[l], __fmul_rn(w[c + l], v[c + l]));
    }
    float s = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[4]), __fadd_rn(acc[2], acc[6])),
                        __fadd_rn(__fadd_rn(acc[1], acc[5]), __fadd_rn(acc[3], acc[7])));
    for (int c = body; c < len; c++) s = __fadd_rn(s, __fmul_rn(w[c], v[c]));
    return s;
}

// ---- Step arguments -------------------------------------------------------------------------

struct RwStep {
    int n, cap, cap_pad, vocab;
    const uint32_t* slots;
    const uint32_t* tokens;
    uint32_t* rflag;        // [n] 1 = this stream's state is reset before this step
    uint32_t* since;        // [cap] tokens since the last reset
    uint32_t reset_every;   // 0 = off
    uint32_t* err;          // bit 0: bad slot/token on the device path, bit 1: pipeline timeout
};

// ---- Load-time embedding normalisation (Rwkv7Model::load, model.rs:266-275) -----------------

// One warp per row; lane 0 runs the two sequential sums of layer_norm (tensor.rs:721-732).
__global__ void k_rw_emb_norm(float* __restrict__ emb, int V, int D, const float* __restrict__ w,
                              const float* __restrict__ bias) {
    extern __shared__ float sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t row = (size_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= (size_t)V) return;
    float* xs = sm + (size_t)warp * D;
    float* er = emb + row * D;
    for (int i = lane; i < D; i += 32) xs[i] = er[i];
    __syncwarp();
    float mean = 0.0f, inv = 0.0f;
    if (lane == 0) {
        mean = __fdiv_rn(seq_sum(xs, D), (float)D);
        float var = 0.0f;
        for (int i = 0; i < D; i++) {
            float d = __fsub_rn(xs[i], mean);
            var = __fadd_rn(var, __fmul_rn(d, d));
        }
        var = __fdiv_rn(var, (float)D);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int i = lane; i < D; i += 32)
        er[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), w[i]), bias[i]);
}

// dst[j][off + k] = src[j][k]: one LoRA up-projection [D][len] into the concatenated [D][R].
__global__ void k_rw_put_cols(const float* __restrict__ src, int D, int len, int R, int off, float* __restrict__ dst) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)D * len) return;
    size_t j = i / len, k = i - j * len;
    dst[j * R + off + k] = src[i];
}

// ---- Block helpers ----------------------------------------------------------------------------

// layer_norm_into (tensor.rs:1390-1398) of xs[D] into ln[D]; tmp[D] is scratch.
__device__ __forceinline__ void block_layer_norm(const float* xs, float* tmp, float* ln, const float* __restrict__ w,
                                                 const float* __restrict__ b, int D, float* s_stat) {
    if (threadIdx.x == 0) s_stat[0] = __fdiv_rn(seq_sum(xs, D), (float)D);
    __syncthreads();
    const float mean = s_stat[0];
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float d = __fsub_rn(xs[i], mean);
        tmp[i] = __fmul_rn(d, d);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float var = __fdiv_rn(seq_sum(tmp, D), (float)D);
        s_stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    }
    __syncthreads();
    const float inv = s_stat[1];
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        ln[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), w[i]), b[i]);
    __syncthreads();
}

// quantize_vec_i8_into (tensor.rs:1791-1800) of v[K] (shared or global) for stream b: scale
// abs_max / 127 (1 for a zero vector), q = clamp(round_half_away(v / scale)), written to the
// tiled layout.  The max is exact, so the reduction order does not matter.
__device__ __forceinline__ void block_quantize(const float* v, int K, int b, int cap_pad, int8_t* __restrict__ aq,
                                               float* __restrict__ as_out, float* s_red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(v[i]));
    m = warp_allmax(m);
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float M = 0.0f;
        for (int i = 0; i < nw; i++) M = fmaxf(M, s_red[i]);
        float scale = M > 0.0f ? __fdiv_rn(M, 127.0f) : 1.0f;
        s_red[32] = __fdiv_rn(1.0f, scale);
        as_out[b] = scale;
    }
    __syncthreads();
    const float inv = s_red[32];
    for (int k = threadIdx.x * 4; k < K; k += blockDim.x * 4) {
        int q[4];
#pragma unroll
        for (int t = 0; t < 4; t++) {
            float r = roundf(__fmul_rn(v[k + t], inv));
            r = (r != r) ? 0.0f : fminf(fmaxf(r, -127.0f), 127.0f);  // Rust's `as i8` maps NaN to 0
            q[t] = (int)r;
        }
        *reinterpret_cast<int*>(aq + aq_off(cap_pad, b, k)) = pack4(q[0], q[1], q[2], q[3]);
    }
    __syncthreads();
}

// ---- LayerNorm + token shift + activation quantisation ---------------------------------------

enum LnMode { kLnTime = 0, kLnChannel = 1, kLnFinal = 2 };

struct LnMixArgs {
    int D, mode;
    const float* emb;        // layer 0 of time mixing: x = emb[token] (the step's first kernel)
    float* x;                // [cap][D] residual stream, by batch position
    const float* ln_w;
    const float* ln_b;
    float* x_prev;           // this layer's [cap][D] shift state (time: x_prev_att, channel: x_prev_ffn)
    const float* mix;        // time: [6][D] x_r, x_w, x_k, x_v, x_a, x_g; channel: [D] x_k
    int8_t* aq0;             // quantised activations, tiled: time xr / channel xk / final ln
    int8_t* aq1;             // time: xk
    int8_t* aq2;             // time: xv
    float* as;               // [3][cap] activation scales
    float* lora_in;          // time: [4][cap][D] xw, xa, xv, xg (F32 LoRA inputs)
};

// One CTA per stream.  time_mixing_scratch steps 1-2 inputs (model.rs:814-826),
// channel_mixing_scratch (:919-923), and the final LayerNorm (:690-692).
__global__ void __launch_bounds__(256) k_rw_ln_mix(RwStep sa, LnMixArgs a) {
    extern __shared__ float sm[];
    __shared__ float s_red[40];
    __shared__ uint32_t s_rf;
    const int b = blockIdx.x, D = a.D;
    float* xs = sm;
    float* ln = sm + D;
    float* tmp = sm + 2 * D;
    float* qv = sm + 3 * D;  // up to three vectors to quantise
    pdl_wait();
    pdl_trigger();
    const uint32_t slot = sa.slots[b];
    float* xb = a.x + (size_t)b * D;
    if (a.emb) {
        const uint32_t tok = sa.tokens[b];
        const bool bad = tok >= (uint32_t)sa.vocab || slot >= (uint32_t)sa.cap;
        if (threadIdx.x == 0) {
            uint32_t rf = 1u;
            if (bad) {
                atomicOr(sa.err, 1u);
            } else {
                // maybe_periodic_reset semantics: reset before the embedding once `since` reached
                // the period, then count this token
                uint32_t s = sa.since[slot];
                rf = (sa.reset_every > 0 && s >= sa.reset_every) ? 1u : 0u;
                sa.since[slot] = rf ? 1u : (s == 0xffffffffu ? s : s + 1u);
            }
            sa.rflag[b] = rf;
            s_rf = rf;
        }
        const float* er = a.emb + (size_t)(bad ? 0u : tok) * D;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            float v = bad ? 0.0f : er[i];
            xs[i] = v;
            xb[i] = v;
        }
    } else {
        if (threadIdx.x == 0) s_rf = sa.rflag[b];
        for (int i = threadIdx.x; i < D; i += blockDim.x) xs[i] = xb[i];
    }
    __syncthreads();
    const bool slot_ok = slot < (uint32_t)sa.cap;
    const bool rf = s_rf != 0u;
    block_layer_norm(xs, tmp, ln, a.ln_w, a.ln_b, D, s_red);
    int nq = 1;
    if (a.mode == kLnFinal) {
        for (int i = threadIdx.x; i < D; i += blockDim.x) qv[i] = ln[i];
    } else {
        float* xp = a.x_prev + (size_t)(slot_ok ? slot : 0u) * D;
        for (int i = threadIdx.x; i < D; i += blockDim.x) {
            const float l = ln[i];
            const float prev = (rf || !slot_ok) ? 0.0f : xp[i];
            if (slot_ok) xp[i] = l;                       // state.x_prev_* = ln_buf (model.rs:668, 681)
            const float xx = __fsub_rn(prev, l);          // sub_into(xx, x_prev, ln)
            if (a.mode == kLnChannel) {
                qv[i] = __fadd_rn(l, __fmul_rn(xx, a.mix[i]));
            } else {
                const float* m = a.mix;
                const size_t cd = (size_t)sa.cap * D;
                float* li = a.lora_in + (size_t)b * D + i;
                qv[i] = __fadd_rn(l, __fmul_rn(xx, m[i]));                        // xr
                li[0] = __fadd_rn(l, __fmul_rn(xx, m[D + i]));                    // xw
                qv[D + i] = __fadd_rn(l, __fmul_rn(xx, m[2 * D + i]));            // xk
                const float xv = __fadd_rn(l, __fmul_rn(xx, m[3 * D + i]));
                qv[2 * D + i] = xv;                                               // xv
                li[2 * cd] = xv;
                li[cd] = __fadd_rn(l, __fmul_rn(xx, m[4 * D + i]));               // xa
                li[3 * cd] = __fadd_rn(l, __fmul_rn(xx, m[5 * D + i]));           // xg
            }
        }
        if (a.mode == kLnTime) nq = 3;
    }
    __syncthreads();
    block_quantize(qv, D, b, sa.cap_pad, a.aq0, a.as, s_red);
    if (nq == 3) {
        block_quantize(qv + D, D, b, sa.cap_pad, a.aq1, a.as + sa.cap, s_red);
        block_quantize(qv + 2 * D, D, b, sa.cap_pad, a.aq2, a.as + 2 * sa.cap, s_red);
    }
}

// quantize_vec_i8_into of a global [n][K] f32 vector set (the gated time-mix output and the
// FFN activation), one CTA per stream.
__global__ void __launch_bounds__(256) k_rw_quant(RwStep sa, const float* __restrict__ v, int K, int8_t* __restrict__ aq,
                                                  float* __restrict__ as_out) {
    __shared__ float s_red[40];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x;
    block_quantize(v + (size_t)b * K, K, b, sa.cap_pad, aq, as_out, s_red);
}

// ---- W8A8 projections -------------------------------------------------------------------------

enum W8Epi { kW8Store = 0, kW8Add = 1, kW8ReluSq = 2 };

struct W8Job {
    const int8_t* w;     // tiled int8 weights [K/64][rows_pad][64]
    const float* ws;     // [M] per-row scales
    int M, rows_pad;
    const int8_t* aq;    // tiled int8 activations
    const float* as;     // [n] activation scales
    float* out;          // out[b * ldo + row]
    int ldo, epi;
};

struct W8Args {
    W8Job job[3];
    int K, n, cap_pad;
};

// out = sum as f32 * (scale_r * v_scale) (tensor.rs:1859-1866), then the caller's epilogue:
// add_inplace for the residuals (model.rs:672, 684), squared_relu_into (tensor.rs:1386-1388).
__device__ __forceinline__ void w8_epilogue(const W8Job& J, int row, int b, int acc, float ws) {
    const float v = __fmul_rn(__int2float_rn(acc), __fmul_rn(ws, J.as[b]));
    float* p = J.out + (size_t)b * J.ldo + row;
    if (J.epi == kW8Add) *p = __fadd_rn(*p, v);
    else if (J.epi == kW8ReluSq) {
        const float r = fmaxf(v, 0.0f);
        *p = __fmul_rn(r, r);
    } else *p = v;
}

// CUDA-core W8A8 (dp4a) for a few streams.  CTA = 16 rows x NS streams; warp w takes 8 rows and a
// quarter of K (exact int32 partial sums, added in shared memory).
template <int NS>
__global__ void __launch_bounds__(256) k_rw_w8a8_dp4a(W8Args a) {
    extern __shared__ int8_t s_act[];  // [NS][K]
    __shared__ int s_part[4][16][NS];
    const W8Job& J = a.job[blockIdx.z];
    const int m0 = blockIdx.x * 16, n0 = blockIdx.y * NS;
    if (m0 >= J.M) return;
    const int K = a.K, G = K >> 6;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rl = (warp & 1) * 8 + (lane >> 2), c = lane & 3, kq = warp >> 1;
    const int r = m0 + rl;
    const int g0 = (G * kq) >> 2, g1 = (G * (kq + 1)) >> 2;
    pdl_wait();
    pdl_trigger();
    const int chunks = K >> 4;
    for (int i = threadIdx.x; i < NS * chunks; i += blockDim.x) {
        const int s = i / chunks, k = (i - s * chunks) << 4, bb = n0 + s;
        int4 v = make_int4(0, 0, 0, 0);
        if (bb < a.n) v = *reinterpret_cast<const int4*>(J.aq + aq_off(a.cap_pad, bb, k));
        *reinterpret_cast<int4*>(s_act + (size_t)s * K + k) = v;
    }
    __syncthreads();
    int acc[NS];
#pragma unroll
    for (int s = 0; s < NS; s++) acc[s] = 0;
    const int8_t* wrow = J.w + (size_t)r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    for (int g = g0; g < g1; g++) {
        const int4 w = __ldg(reinterpret_cast<const int4*>(wrow + (size_t)g * J.rows_pad * 64));
#pragma unroll
        for (int s = 0; s < NS; s++) {
            const int4 x = *reinterpret_cast<const int4*>(s_act + (size_t)s * K + g * 64 + c * 16);
            acc[s] = __dp4a(w.x, x.x, acc[s]);
            acc[s] = __dp4a(w.y, x.y, acc[s]);
            acc[s] = __dp4a(w.z, x.z, acc[s]);
            acc[s] = __dp4a(w.w, x.w, acc[s]);
        }
    }
#pragma unroll
    for (int s = 0; s < NS; s++) {
        acc[s] += __shfl_xor_sync(0xffffffffu, acc[s], 1);
        acc[s] += __shfl_xor_sync(0xffffffffu, acc[s], 2);
        if (c == 0) s_part[kq][rl][s] = acc[s];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 16 * NS; i += blockDim.x) {
        const int rr = i & 15, s = i >> 4, row = m0 + rr, bb = n0 + s;
        if (row < J.M && bb < a.n) {
            const int tot = s_part[0][rr][s] + s_part[1][rr][s] + s_part[2][rr][s] + s_part[3][rr][s];
            w8_epilogue(J, row, bb, tot, J.ws[row]);
        }
    }
}

// Tensor-core W8A8: one (128-row, BN-stream) tile accumulated over all of K in one int32 TMEM
// accumulator (tcgen05.mma kind::i8, M = 128, N = BN, K = 32 per instruction).  Each pipeline stage
// is one 64-byte K slice: 8 KB of weights + BN x 64 B of activations, each one bulk copy of the
// pre-tiled operands.  Warp 0 copies, warp 1 owns TMEM and issues the MMAs, warps 2-5 read the
// accumulator (thread = row = TMEM lane) and run the epilogue.  Waits are bounded as in the Q8
// projection kernel.
template <int BN>
struct alignas(1024) W8Smem {
    static constexpr int kStages = 8;
    int8_t a[kStages][tc::kBM * 64];
    int8_t b[kStages][BN * 64];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t tfull;
    uint32_t tmem_base;
    int abort;
};

template <int BN>
__host__ __device__ constexpr uint32_t w8_cols() {
    return BN < 32 ? 32u : (uint32_t)BN;
}

template <int BN>
constexpr size_t w8_smem() {
    return sizeof(W8Smem<BN>) + 1024;
}

template <int BN>
__global__ void __launch_bounds__(192, 1) k_rw_w8a8_tc(W8Args a, uint32_t* err) {
    using namespace tc;
    extern __shared__ uint8_t smem_raw[];
    W8Smem<BN>& S = *reinterpret_cast<W8Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int kStages = W8Smem<BN>::kStages;
    constexpr uint32_t kCols = w8_cols<BN>();
    constexpr uint32_t kStageBytes = kBM * 64 + BN * 64;
    const W8Job& J = a.job[blockIdx.z];
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kBM;
    if (m0 >= J.M) return;
    const int G = a.K >> 6;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npre = G < kStages ? G : kStages;
    const int8_t* wtile = J.w + (size_t)m0 * 64;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(&S.tfull, 1);
        S.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int g = 0; g < npre; g++) {  // weights are constant: stream them before the dependency wait
            mbar_expect_tx(&S.full[g], kStageBytes);
            bulk_load(S.a[g], wtile + (size_t)g * J.rows_pad * 64, kBM * 64, &S.full[g]);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort = &S.abort;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();
            pdl_trigger();
            int issued = 0;
            const int8_t* act = J.aq + (size_t)(n0 >> 4) * 16 * 64;
            const size_t gstride = (size_t)(a.cap_pad >> 4) * 16 * 64;
            for (int g = 0; g < G; g++) {
                const int s = g % kStages;
                const uint32_t ph = (g / kStages) & 1;
                if (g >= npre) {
                    if (!mbar_wait(&S.empty[s], ph ^ 1, abort)) break;
                    mbar_expect_tx(&S.full[s], kStageBytes);
                    bulk_load(S.a[s], wtile + (size_t)g * J.rows_pad * 64, kBM * 64, &S.full[s]);
                }
                bulk_load(S.b[s], act + (size_t)g * gstride, BN * 64, &S.full[s]);
                issued = g + 1;
            }
            if (*abort) {
                int from = issued > kStages ? issued - kStages : 0;
                int to = issued > npre ? issued : npre;
                for (int g = from; g < to; g++) mbar_drain(&S.full[g % kStages], (g / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<BN>();
            int last = -1;
            for (int g = 0; g < G; g++) {
                const int s = g % kStages;
                const uint32_t ph = (g / kStages) & 1;
                if (!mbar_wait(&S.full[s], ph, abort)) break;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    mma_i8(tmem, sw64_desc(S.a[s] + ks * 32), sw64_desc(S.b[s] + ks * 32), idesc, (uint32_t)(g | ks));
                mma_commit(&S.empty[s]);
                last = g;
            }
            if (last == G - 1) mma_commit(&S.tfull);
            else if (last >= 0) mbar_drain(&S.empty[last % kStages], (last / kStages) & 1);
        }
        __syncwarp();
    } else {
        const int quad = warp & 3;
        const int row = m0 + quad * 32 + lane;
        const bool row_ok = row < J.M;
        const float ws = row_ok ? __ldg(J.ws + row) : 0.0f;
        pdl_wait();
        pdl_trigger();
        const bool ok = __all_sync(0xffffffffu, mbar_wait(&S.tfull, 0, abort));
        if (ok) {
            tc_fence_after();
            const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                int v[16];
                tmem_ld16(base + (uint32_t)c0, v);
                tmem_wait_ld();
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < 16; q++) {
                        const int bb = n0 + c0 + q;
                        if (bb < a.n) w8_epilogue(J, row, bb, v[q], ws);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (*abort && threadIdx.x == 0) atomicOr(err, 2u);
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols));
    }
}

// ---- F32 LoRA down-projections -----------------------------------------------------------------

struct Lora1Args {
    int D, R, layer0;
    int act_body;                 // 8-aligned part of the largest rank: lane functions below it
    int seg_off[4], seg_len[4];   // decay w, a, v, gate: rows of the concatenated [R][D] matrix
    int tiles_before[5];          // 32-row tiles before each segment
    const float* xin;             // [4][cap][D] xw, xa, xv, xg
    const float* w1cat;           // [R][D]
    float* h1;                    // [cap][R]: tanh(w1 xw), a1 xa, v1 xv, sigmoid(g1 xg)
};

// CTA = 32 rows of one segment x 16 streams; thread = one of the 8 dot lanes for 4 rows x 4 streams.
// Lane l sums columns l, l+8, ... in order; the hsum tree runs over the 8 lane threads with
// shuffles (xor 4, 2, 1 pair exactly (l0+l4), (l2+l6), ... as in hsum_f32).  D is a multiple of
// 64, so there is no tail.
__global__ void __launch_bounds__(256) k_rw_lora1(RwStep sa, Lora1Args a) {
    __shared__ float Ws[32][66];
    __shared__ float Xs[16][66];
    const int bt = blockIdx.x;
    int seg = 0;
    while (seg < 3 && bt >= a.tiles_before[seg + 1]) seg++;
    if (a.layer0 && seg == 2) return;  // v_lora is not used by layer 0 (model.rs:858)
    const int len = a.seg_len[seg];
    const int r0 = (bt - a.tiles_before[seg]) * 32;
    const int rows = min(32, len - r0);
    const int n0 = blockIdx.y * 16, D = a.D;
    const float* X = a.xin + (size_t)seg * sa.cap * D;
    const float* Wm = a.w1cat + (size_t)(a.seg_off[seg] + r0) * D;
    const int l8 = threadIdx.x & 7, mt = threadIdx.x >> 3, rg = mt & 7, sg = mt >> 3;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    pdl_wait();
    pdl_trigger();
    for (int k0 = 0; k0 < D; k0 += 64) {
        for (int e = threadIdx.x; e < 32 * 64; e += 256) {
            const int rr = e >> 6, cc = e & 63;
            Ws[rr][cc] = rr < rows ? Wm[(size_t)rr * D + k0 + cc] : 0.0f;
        }
        for (int e = threadIdx.x; e < 16 * 64; e += 256) {
            const int ss = e >> 6, cc = e & 63;
            Xs[ss][cc] = n0 + ss < sa.n ? X[(size_t)(n0 + ss) * D + k0 + cc] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int c = l8 + 8 * i;
            float w[4], x[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                w[t] = Ws[rg * 4 + t][c];
                x[t] = Xs[sg * 4 + t][c];
            }
#pragma unroll
            for (int p = 0; p < 4; p++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[p][q] = __fadd_rn(acc[p][q], __fmul_rn(w[p], x[q]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int p = 0; p < 4; p++)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            float v = acc[p][q];
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
            v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
            acc[p][q] = v;
        }
    if (l8 == 0) {
        // the reference applies tanh / sigmoid to its whole max-rank scratch (model.rs:830, 845),
        // so the lane/portable split is at the largest rank's 8-aligned length
        const int body = a.act_body;
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int row = r0 + rg * 4 + p;
            if (row >= len) continue;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int bb = n0 + sg * 4 + q;
                if (bb >= sa.n) continue;
                float v = acc[p][q];
                if (seg == 0) v = tanh_at(v, row < body);          // tanh_inplace (model.rs:830)
                else if (seg == 3) v = sigmoid_at(v, row < body);  // sigmoid_inplace (model.rs:845)
                a.h1[(size_t)bb * a.R + a.seg_off[seg] + row] = v;
            }
        }
    }
}

// ---- WKV-7 head update ---------------------------------------------------------------------------

struct WkvArgs {
    int D, H, R, layer0, g1k;
    int seg_off[4], seg_len[4];
    const float* rkv;      // [3][cap][D] r, k, v projections
    const float* h1;       // [cap][R]
    const float* w2cat;    // [D][R] decay / a / v / gate up-projections, row = channel
    const float* w0;
    const float* a0;
    const float* v0;
    const float* k_k;
    const float* k_a;
    const float* r_k;
    const float* lnx_w;
    const float* lnx_b;
    float* wkv;            // this layer's state [cap][H][16][64][4]: row i's 16-byte chunk q at (q * 64 + i)
    float* v_first;        // [cap][D]
    float* gated;          // [cap][D]
};

constexpr int kWkvSB = 4;  // streams per CTA (64 threads each)

__host__ __device__ constexpr int wkv_rp(int R) { return R | 1; }  // odd row stride: no bank conflicts

inline size_t wkv_smem(int R) {
    return ((size_t)kHS * wkv_rp(R) + (size_t)kWkvSB * R + (size_t)kWkvSB * 8 * kHS) * sizeof(float);
}

// CTA = one head x kWkvSB streams; thread (s, j) owns channel j of the head for stream s and row j
// of that stream's 64x64 state.  time_mixing_scratch steps 3-12 (model.rs:828-913) for one head.
__global__ void __launch_bounds__(kHS * kWkvSB) k_rw_wkv(RwStep sa, WkvArgs a) {
    extern __shared__ float sm[];
    __shared__ float s_st[kWkvSB][4];
    const int R = a.R, Rp = wkv_rp(R), D = a.D;
    float* W = sm;                                  // [64][Rp]
    float* hs = W + kHS * Rp;                       // [SB][R]
    float* vec = hs + kWkvSB * R;                   // [SB][8][64]
    const int h = blockIdx.x, n0 = blockIdx.y * kWkvSB;
    const int s = threadIdx.x >> 6, j = threadIdx.x & 63;
    const int b = n0 + s, c = h * kHS + j;
    // the up-projection rows of this head: constant, loaded before the dependency wait
    for (int i = threadIdx.x; i < kHS * R; i += blockDim.x) {
        const int jj = i / R, k = i - jj * R;
        W[jj * Rp + k] = a.w2cat[(size_t)(h * kHS + jj) * R + k];
    }
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < kWkvSB * R; i += blockDim.x) {
        const int ss = i / R, k = i - ss * R;
        hs[i] = n0 + ss < sa.n ? a.h1[(size_t)(n0 + ss) * R + k] : 0.0f;
    }
    __syncthreads();
    uint32_t slot = 0;
    bool act = b < sa.n;
    if (act) {
        slot = sa.slots[b];
        act = slot < (uint32_t)sa.cap;
    }
    const bool rf = act && sa.rflag[b] != 0u;
    float* V = vec + s * 8 * kHS;  // 0 w, 1 kk*a, 2 k_mod, 3 r, 4 -kk, 5 v_out, 6 scratch, 7 bonus terms
    float g = 0.0f, vout = 0.0f, kk = 0.0f, aa = 0.0f;
    if (act) {
        const float* hb = hs + s * R;
        const float* wr = W + j * Rp;
        const float lw = dot8(wr + a.seg_off[0], hb + a.seg_off[0], a.seg_len[0]);
        const float la = dot8(wr + a.seg_off[1], hb + a.seg_off[1], a.seg_len[1]);
        g = dot8(wr + a.seg_off[3], hb + a.seg_off[3], a.seg_len[3]);
        const size_t cd = (size_t)sa.cap * D;
        const float rr = a.rkv[(size_t)b * D + c];
        const float kv = a.rkv[cd + (size_t)b * D + c];
        const float vv = a.rkv[2 * cd + (size_t)b * D + c];
        const bool lane = c < (D & ~7);
        V[j] = decay_at(__fadd_rn(a.w0[c], lw), lane);            // step 3
        aa = sigmoid_at(__fadd_rn(a.a0[c], la), lane);            // step 4
        kk = __fmul_rn(kv, a.k_k[c]);                             // step 6
        const float kmod = __fmul_rn(kv, __fadd_rn(1.0f, __fmul_rn(__fsub_rn(aa, 1.0f), a.k_a[c])));  // step 7
        if (a.layer0) {                                           // step 8
            vout = vv;
            a.v_first[(size_t)slot * D + c] = vv;                 // state.v_first = v (model.rs:669-671)
        } else {
            const float lv = dot8(wr + a.seg_off[2], hb + a.seg_off[2], a.seg_len[2]);
            const float mix = sigmoid_at(__fadd_rn(a.v0[c], lv), lane);
            const float vf = a.v_first[(size_t)slot * D + c];
            vout = __fadd_rn(vv, __fmul_rn(__fsub_rn(vf, vv), mix));
        }
        V[2 * kHS + j] = kmod;
        V[3 * kHS + j] = rr;
        V[5 * kHS + j] = vout;
        V[6 * kHS + j] = __fmul_rn(kk, kk);
        V[7 * kHS + j] = __fmul_rn(__fmul_rn(rr, a.g1k ? kmod : kv), a.r_k[c]);  // step 11 terms
    }
    __syncthreads();
    if (j == 0 && act) {  // l2_normalize_per_head_inplace (tensor.rs:1416-1424)
        const float norm = __fsqrt_rn(seq_sum(V + 6 * kHS, kHS));
        s_st[s][0] = norm > 1e-12f ? __fdiv_rn(1.0f, norm) : 0.0f;
        s_st[s][3] = seq_sum(V + 7 * kHS, kHS);  // bonus
    }
    __syncthreads();
    if (act) {
        kk = __fmul_rn(kk, s_st[s][0]);
        V[kHS + j] = __fmul_rn(kk, aa);
        V[4 * kHS + j] = -kk;
    }
    __syncthreads();
    float o = 0.0f;
    if (act) {  // step 9, row i = j of this head's state
        float4* st = reinterpret_cast<float4*>(a.wkv + ((size_t)slot * a.H + h) * (kHS * kHS));
        float S[kHS];
#pragma unroll
        for (int q = 0; q < kHS / 4; q++) {
            float4 t = rf ? make_float4(0.f, 0.f, 0.f, 0.f) : st[q * kHS + j];
            S[4 * q] = t.x;
            S[4 * q + 1] = t.y;
            S[4 * q + 2] = t.z;
            S[4 * q + 3] = t.w;
        }
        float temp = 0.0f;  // (state @ -kk)[i]
#pragma unroll
        for (int q = 0; q < kHS; q++) temp = __fadd_rn(temp, __fmul_rn(S[q], V[4 * kHS + q]));
        const float vi = V[5 * kHS + j];
#pragma unroll
        for (int q = 0; q < kHS; q++) {
            const float sab = __fmul_rn(temp, V[kHS + q]);
            const float nv = __fadd_rn(__fadd_rn(__fmul_rn(S[q], V[q]), sab), __fmul_rn(vi, V[2 * kHS + q]));
            S[q] = nv;
            o = __fadd_rn(o, __fmul_rn(nv, V[3 * kHS + q]));  // (state @ r)[i]
        }
#pragma unroll
        for (int q = 0; q < kHS / 4; q++) st[q * kHS + j] = make_float4(S[4 * q], S[4 * q + 1], S[4 * q + 2], S[4 * q + 3]);
    }
    __syncthreads();  // slot 6 is free again
    if (act) V[6 * kHS + j] = o;
    __syncthreads();
    if (j == 0 && act) {  // group_norm_into (tensor.rs:1400-1414), one group per head
        const float mean = __fdiv_rn(seq_sum(V + 6 * kHS, kHS), (float)kHS);
        float var = 0.0f;
        for (int q = 0; q < kHS; q++) {
            const float d = __fsub_rn(V[6 * kHS + q], mean);
            var = __fadd_rn(var, __fmul_rn(d, d));
        }
        var = __fdiv_rn(var, (float)kHS);
        s_st[s][1] = mean;
        s_st[s][2] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 64e-5f)));
    }
    __syncthreads();
    if (act) {
        float on = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(o, s_st[s][1]), s_st[s][2]), a.lnx_w[c]), a.lnx_b[c]);
        on = __fadd_rn(on, __fmul_rn(s_st[s][3], vout));          // step 11
        a.gated[(size_t)b * D + c] = __fmul_rn(on, g);            // step 12
    }
}

}  // namespace rw
}  // namespace rk
