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

// Sequential sum from +0 (Rust's f32 `Sum`, a left fold), run by one thread.  The values are read
// 32 at a time into registers ahead of the dependent adds, so the chain costs one add latency per
// element instead of one shared-memory round trip.
__device__ __forceinline__ float seq_sum(const float* p, int n) {
    float s = 0.0f;
    int i = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
#pragma unroll 2
        for (; i + 32 <= n; i += 32) {
            float4 v[8];
#pragma unroll
            for (int q = 0; q < 8; q++) v[q] = reinterpret_cast<const float4*>(p + i)[q];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                s = __fadd_rn(s, v[q].x);
                s = __fadd_rn(s, v[q].y);
                s = __fadd_rn(s, v[q].z);
                s = __fadd_rn(s, v[q].w);
            }
        }
    }
    for (; i < n; i++) s = __fadd_rn(s, p[i]);
    return s;
}

// Sequential sum of (p[i] - mean)^2 from +0: the variance pass of layer_norm / group_norm.
__device__ __forceinline__ float seq_sq_dev(const float* p, int n, float mean) {
    float s = 0.0f;
    int i = 0;
    if ((reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
#pragma unroll 2
        for (; i + 32 <= n; i += 32) {
            float d[32];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const float4 v = reinterpret_cast<const float4*>(p + i)[q];
                d[4 * q] = __fsub_rn(v.x, mean);
                d[4 * q + 1] = __fsub_rn(v.y, mean);
                d[4 * q + 2] = __fsub_rn(v.z, mean);
                d[4 * q + 3] = __fsub_rn(v.w, mean);
            }
#pragma unroll
            for (int q = 0; q < 32; q++) s = __fadd_rn(s, __fmul_rn(d[q], d[q]));
        }
    }
    for (; i < n; i++) {
        const float d = __fsub_rn(p[i], mean);
        s = __fadd_rn(s, __fmul_rn(d, d));
    }
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

// dot_avx2_order with the matrix row read at a stride (the head-major up-projection layout).
__device__ __forceinline__ float dot8s(const float* w, int stride, const float* v, int len) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; l++) acc[l] = 0.0f;
    const int body = len & ~7;
    for (int c = 0; c < body; c += 8) {
#pragma unroll
        for (int l = 0; l < 8; l++) acc[l] = __fadd_rn(acc[l], __fmul_rn(w[(c + l) * stride], v[c + l]));
    }
    float s = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[4]), __fadd_rn(acc[2], acc[6])),
                        __fadd_rn(__fadd_rn(acc[1], acc[5]), __fadd_rn(acc[3], acc[7])));
    for (int c = body; c < len; c++) s = __fadd_rn(s, __fmul_rn(w[c * stride], v[c]));
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
    uint32_t* vslot;        // [n] validated slots, written by the step's first kernel (kRejected = bad
                            // slot or token); every later kernel gets them as `slots`
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
        const float var = __fdiv_rn(seq_sq_dev(xs, D, mean), (float)D);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int i = lane; i < D; i += 32)
        er[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xs[i], mean), inv), w[i]), bias[i]);
}

// One LoRA up-projection [D][len] (row = channel) into the layer's head-major [H][R][64] matrix:
// channel c = 64 h + j, column k lands at (h R + off + k) * 64 + j.  A head's up-projections are
// then one contiguous block that k_rw_wkv copies in with a single bulk copy, and thread j reads
// column k at stride 64 (no bank conflicts).
__global__ void k_rw_put_up(const float* __restrict__ src, int D, int len, int R, int off, float* __restrict__ dst) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)D * len) return;
    const size_t c = i / len, k = i - c * len;
    dst[((c / kHS) * R + off + k) * kHS + (c % kHS)] = src[i];
}

// ---- Activation quantisation helpers ----------------------------------------------------------

// quantize_vec_i8_into (tensor.rs:1791-1800): scale = abs_max / 127 (1 for a zero vector),
// q = clamp(round_half_away(v / scale)).  The max is exact, so its reduction order does not matter.
__device__ __forceinline__ float q8_scale(float amax) { return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f; }

__device__ __forceinline__ int q8_one(float v, float inv) {
    float r = roundf(__fmul_rn(v, inv));
    r = (r != r) ? 0.0f : fminf(fmaxf(r, -127.0f), 127.0f);  // Rust's `as i8` maps NaN to 0
    return (int)r;
}

__device__ __forceinline__ int q8_pack(float4 v, float inv) {
    return pack4(q8_one(v.x, inv), q8_one(v.y, inv), q8_one(v.z, inv), q8_one(v.w, inv));
}

__device__ __forceinline__ float amax4(float4 v) {
    return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// a + b * c element-wise (add_scaled_into, tensor.rs:747-751)
__device__ __forceinline__ float4 add_scaled4(float4 a, float4 b, float4 c) {
    return make_float4(__fadd_rn(a.x, __fmul_rn(b.x, c.x)), __fadd_rn(a.y, __fmul_rn(b.y, c.y)),
                       __fadd_rn(a.z, __fmul_rn(b.z, c.z)), __fadd_rn(a.w, __fmul_rn(b.w, c.w)));
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

// One CTA of D/4 threads per stream, thread t owning elements 4t..4t+3.  time_mixing_scratch
// steps 1-2 inputs (model.rs:814-826), channel_mixing_scratch (:919-923), and the final LayerNorm
// (:690-692).  Every global load is issued before the LayerNorm's two sequential sums (thread 0,
// layer_norm_into tensor.rs:1390-1398), which are the kernel's critical path.
__global__ void __launch_bounds__(1024) k_rw_ln_mix(RwStep sa, LnMixArgs a) {
    extern __shared__ float xs[];  // [D]
    __shared__ float s_red[3][32];
    __shared__ float s_stat[8];
    __shared__ uint32_t s_rf;
    const int b = blockIdx.x, D = a.D, t = threadIdx.x, i0 = 4 * t;
    const int lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    const int nmix = a.mode == kLnTime ? 6 : (a.mode == kLnChannel ? 1 : 0);
    // constant vectors: before the dependency wait
    const float4 lw = ldg4(a.ln_w + i0), lb = ldg4(a.ln_b + i0);
    float4 m[6];
#pragma unroll
    for (int q = 0; q < 6; q++) m[q] = q < nmix ? ldg4(a.mix + (size_t)q * D + i0) : make_float4(0.f, 0.f, 0.f, 0.f);
    pdl_wait();
    pdl_trigger();
    const uint32_t slot = sa.slots[b];
    bool slot_ok = slot < (uint32_t)sa.cap;
    float* xb = a.x + (size_t)b * D;
    float4 x;
    if (a.emb) {
        // the step's first kernel: a bad slot or token rejects the stream for the whole step (no
        // state read or written, no counter change, zero logits)
        const uint32_t tok = sa.tokens[b];
        const bool bad = tok >= (uint32_t)sa.vocab || !slot_ok;
        slot_ok = !bad;
        if (t == 0) {
            sa.vslot[b] = bad ? kRejected : slot;
            uint32_t rf = 0u;
            if (bad) {
                atomicOr(sa.err, 1u);
            } else {
                // maybe_periodic_reset semantics: reset before the embedding once `since` reached
                // the period, then count this token
                const uint32_t sn = sa.since[slot];
                rf = (sa.reset_every > 0 && sn >= sa.reset_every) ? 1u : 0u;
                sa.since[slot] = rf ? 1u : (sn == 0xffffffffu ? sn : sn + 1u);
            }
            sa.rflag[b] = rf;
            s_rf = rf;
        }
        x = bad ? make_float4(0.f, 0.f, 0.f, 0.f) : ldg4(a.emb + (size_t)tok * D + i0);
        st4(xb + i0, x);
    } else {
        if (t == 0) s_rf = sa.rflag[b];
        x = ld4(xb + i0);
    }
    float* xp_row = a.x_prev + (size_t)(slot_ok ? slot : 0u) * D;
    float4 xp = make_float4(0.f, 0.f, 0.f, 0.f);
    if (a.mode != kLnFinal && slot_ok) xp = ld4(xp_row + i0);
    st4(xs + i0, x);
    __syncthreads();
    if (t == 0) {
        const float mean = __fdiv_rn(seq_sum(xs, D), (float)D);
        const float var = __fdiv_rn(seq_sq_dev(xs, D, mean), (float)D);
        s_stat[0] = mean;
        s_stat[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
    }
    __syncthreads();
    const float mean = s_stat[0], inv = s_stat[1];
    float4 ln;
    ln.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.x, mean), inv), lw.x), lb.x);
    ln.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.y, mean), inv), lw.y), lb.y);
    ln.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.z, mean), inv), lw.z), lb.z);
    ln.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.w, mean), inv), lw.w), lb.w);
    float4 q[3];
    int nq = 1;
    if (a.mode == kLnFinal) {
        q[0] = slot_ok ? ln : make_float4(0.f, 0.f, 0.f, 0.f);  // a rejected stream's logits are zeros
    } else {
        if (s_rf || !slot_ok) xp = make_float4(0.f, 0.f, 0.f, 0.f);
        if (slot_ok) st4(xp_row + i0, ln);  // state.x_prev_* = ln_buf (model.rs:668, 681)
        const float4 xx = make_float4(__fsub_rn(xp.x, ln.x), __fsub_rn(xp.y, ln.y), __fsub_rn(xp.z, ln.z),
                                      __fsub_rn(xp.w, ln.w));  // sub_into(xx, x_prev, ln)
        if (a.mode == kLnChannel) {
            q[0] = add_scaled4(ln, xx, m[0]);
        } else {
            const size_t cd = (size_t)sa.cap * D;
            float* li = a.lora_in + (size_t)b * D + i0;
            q[0] = add_scaled4(ln, xx, m[0]);                // xr
            st4(li, add_scaled4(ln, xx, m[1]));              // xw
            q[1] = add_scaled4(ln, xx, m[2]);                // xk
            q[2] = add_scaled4(ln, xx, m[3]);                // xv
            st4(li + 2 * cd, q[2]);
            st4(li + cd, add_scaled4(ln, xx, m[4]));         // xa
            st4(li + 3 * cd, add_scaled4(ln, xx, m[5]));     // xg
            nq = 3;
        }
    }
    // one reduction round for the up to three vectors to quantise
#pragma unroll
    for (int v = 0; v < 3; v++) {
        if (v < nq) {
            const float mv = warp_allmax(amax4(q[v]));
            if (lane == 0) s_red[v][warp] = mv;
        }
    }
    __syncthreads();
    if (t < nq) {
        float M = 0.0f;
        for (int w = 0; w < nw; w++) M = fmaxf(M, s_red[t][w]);
        const float scale = q8_scale(M);
        s_stat[2 + t] = __fdiv_rn(1.0f, scale);
        a.as[(size_t)t * sa.cap + b] = scale;
    }
    __syncthreads();
    int8_t* aqs[3] = {a.aq0, a.aq1, a.aq2};
#pragma unroll
    for (int v = 0; v < 3; v++)
        if (v < nq) *reinterpret_cast<int*>(aqs[v] + aq_off(sa.cap_pad, b, i0)) = q8_pack(q[v], s_stat[2 + v]);
}

// quantize_vec_i8_into of a global [n][K] f32 vector set (the gated time-mix output and the
// FFN activation): one CTA per stream; each thread keeps its up to kQuantPer float4 in registers
// across the max reduction, so the vector is read once.
constexpr int kQuantPer = 4;  // K <= 256 threads x 4 x 4 = 4096 in one pass

__global__ void __launch_bounds__(256) k_rw_quant(RwStep sa, const float* __restrict__ v, int K, int8_t* __restrict__ aq,
                                                  float* __restrict__ as_out) {
    __shared__ float s_red[8];
    pdl_wait();
    pdl_trigger();
    const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float* vb = v + (size_t)b * K;
    float4 x[kQuantPer];
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < kQuantPer; i++) {
        const int k = (i * 256 + t) * 4;
        x[i] = k < K ? ld4(vb + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        m = fmaxf(m, amax4(x[i]));
    }
    for (int k = (kQuantPer * 256 + t) * 4; k < K; k += 1024) m = fmaxf(m, amax4(ld4(vb + k)));
    m = warp_allmax(m);
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    float M = s_red[0];
#pragma unroll
    for (int w = 1; w < 8; w++) M = fmaxf(M, s_red[w]);
    const float scale = q8_scale(M);
    const float inv = __fdiv_rn(1.0f, scale);
    if (t == 0) as_out[b] = scale;
#pragma unroll
    for (int i = 0; i < kQuantPer; i++) {
        const int k = (i * 256 + t) * 4;
        if (k < K) *reinterpret_cast<int*>(aq + aq_off(sa.cap_pad, b, k)) = q8_pack(x[i], inv);
    }
    for (int k = (kQuantPer * 256 + t) * 4; k < K; k += 1024)
        *reinterpret_cast<int*>(aq + aq_off(sa.cap_pad, b, k)) = q8_pack(ld4(vb + k), inv);
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

// The epilogue for 16 consecutive streams of one row (b0 .. b0+15, the first nb valid): the
// residual operands are loaded as one batch before any store, so a residual add costs one memory
// round trip per 16 streams instead of one per stream.
__device__ __forceinline__ void w8_epilogue16(const W8Job& J, int row, int b0, int nb, const int (&acc)[16], float ws) {
    float v[16];
#pragma unroll
    for (int q = 0; q < 16; q++) v[q] = q < nb ? __fmul_rn(__int2float_rn(acc[q]), __fmul_rn(ws, J.as[b0 + q])) : 0.0f;
    float* p = J.out + (size_t)b0 * J.ldo + row;
    if (J.epi == kW8Add) {
        float old[16];
#pragma unroll
        for (int q = 0; q < 16; q++) old[q] = q < nb ? p[(size_t)q * J.ldo] : 0.0f;
#pragma unroll
        for (int q = 0; q < 16; q++)
            if (q < nb) p[(size_t)q * J.ldo] = __fadd_rn(old[q], v[q]);
    } else if (J.epi == kW8ReluSq) {
#pragma unroll
        for (int q = 0; q < 16; q++) {
            const float r = fmaxf(v[q], 0.0f);
            if (q < nb) p[(size_t)q * J.ldo] = __fmul_rn(r, r);
        }
    } else {
#pragma unroll
        for (int q = 0; q < 16; q++)
            if (q < nb) p[(size_t)q * J.ldo] = v[q];
    }
}

// CUDA-core W8A8 (dp4a) for a few streams.  CTA = 16 rows x NS streams; warp w takes 8 rows and a
// quarter of K (exact int32 partial sums, added in shared memory).  The first kDp4aPre weight
// chunks of each lane are loaded before the dependency wait, so at small batch the weight stream
// overlaps the tail of the preceding kernel.
constexpr int kDp4aPre = 12;

__device__ __forceinline__ void dp4a_acc(int& acc, int4 w, int4 x) {
    acc = __dp4a(w.x, x.x, acc);
    acc = __dp4a(w.y, x.y, acc);
    acc = __dp4a(w.z, x.z, acc);
    acc = __dp4a(w.w, x.w, acc);
}

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
    const int g0 = (G * kq) >> 2, g1 = (G * (kq + 1)) >> 2, ng = g1 - g0;
    const int8_t* wrow = J.w + (size_t)r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
    const size_t gstride = (size_t)J.rows_pad * 64;
    int4 wpre[kDp4aPre];
#pragma unroll
    for (int i = 0; i < kDp4aPre; i++)
        if (i < ng) wpre[i] = __ldg(reinterpret_cast<const int4*>(wrow + (size_t)(g0 + i) * gstride));
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
#pragma unroll
    for (int i = 0; i < kDp4aPre; i++) {
        if (i < ng) {
            const int g = g0 + i;
#pragma unroll
            for (int s = 0; s < NS; s++)
                dp4a_acc(acc[s], wpre[i], *reinterpret_cast<const int4*>(s_act + (size_t)s * K + g * 64 + c * 16));
        }
    }
    for (int g = g0 + kDp4aPre; g < g1; g++) {
        const int4 w = __ldg(reinterpret_cast<const int4*>(wrow + (size_t)g * gstride));
#pragma unroll
        for (int s = 0; s < NS; s++)
            dp4a_acc(acc[s], w, *reinterpret_cast<const int4*>(s_act + (size_t)s * K + g * 64 + c * 16));
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
                const int b0 = n0 + c0;
                if (row_ok && b0 < a.n) w8_epilogue16(J, row, b0, min(16, a.n - b0), v, ws);
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
    int tiles_before[5];          // kLoraRows-row tiles before each segment
    const float* xin;             // [4][cap][D] xw, xa, xv, xg
    const float* w1cat;           // [R][D]
    float* h1;                    // [cap][R]: tanh(w1 xw), a1 xa, v1 xv, sigmoid(g1 xg)
};

// CTA = 16 rows of one segment x 16 streams; thread = one of the 8 dot lanes for 2 rows x 4
// streams.  Lane l sums columns l, l+8, ... in order; the hsum tree runs over the 8 lane threads
// with shuffles (xor 4, 2, 1 pair exactly (l0+l4), (l2+l6), ... as in hsum_f32).  K is staged in
// chunks of up to kLoraKC columns, so a 768-wide model needs one global round trip per CTA.
// D is a multiple of 64, so there is no tail.
constexpr int kLoraRows = 16;
constexpr int kLoraStreams = 16;
constexpr int kLoraKC = 768;
constexpr int kLoraStride = kLoraKC + 4;  // row stride = 4 (mod 32) words: conflict-free lane reads

inline size_t lora1_smem() { return (size_t)(kLoraRows + kLoraStreams) * kLoraStride * sizeof(float); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(tc::smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(256) k_rw_lora1(RwStep sa, Lora1Args a) {
    extern __shared__ float sm[];
    float* Ws = sm;                              // [16][kLoraStride]
    float* Xs = sm + kLoraRows * kLoraStride;    // [16][kLoraStride]
    const int bt = blockIdx.x;
    int seg = 0;
    while (seg < 3 && bt >= a.tiles_before[seg + 1]) seg++;
    if (a.layer0 && seg == 2) return;  // v_lora is not used by layer 0 (model.rs:858)
    const int len = a.seg_len[seg];
    const int r0 = (bt - a.tiles_before[seg]) * kLoraRows;
    const int rows = min(kLoraRows, len - r0);
    const int n0 = blockIdx.y * kLoraStreams, D = a.D;
    const int nst = min(kLoraStreams, sa.n - n0);
    const float* X = a.xin + (size_t)seg * sa.cap * D;
    const float* Wm = a.w1cat + (size_t)(a.seg_off[seg] + r0) * D;
    const int l8 = threadIdx.x & 7, mt = threadIdx.x >> 3, rg = mt & 7, sg = mt >> 3;
    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    // asynchronous 16-byte copies straight into shared memory; the weight chunk (constant) is
    // requested before the dependency wait, the activations after it
    auto stage_w = [&](int k0, int kc4) {
        for (int e = threadIdx.x; e < kLoraRows * kc4; e += 256) {
            const int rr = e / kc4, c4 = e - rr * kc4;
            float4* dst = reinterpret_cast<float4*>(Ws + rr * kLoraStride) + c4;
            if (rr < rows) cp_async16(dst, reinterpret_cast<const float4*>(Wm + (size_t)rr * D + k0) + c4);
            else *dst = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    stage_w(0, min(kLoraKC, D) >> 2);
    pdl_wait();
    pdl_trigger();
    for (int k0 = 0; k0 < D; k0 += kLoraKC) {
        const int kc = min(kLoraKC, D - k0), kc4 = kc >> 2;
        if (k0 > 0) stage_w(k0, kc4);
        for (int e = threadIdx.x; e < kLoraStreams * kc4; e += 256) {
            const int ss = e / kc4, c4 = e - ss * kc4;
            float4* dst = reinterpret_cast<float4*>(Xs + ss * kLoraStride) + c4;
            if (ss < nst) cp_async16(dst, reinterpret_cast<const float4*>(X + (size_t)(n0 + ss) * D + k0) + c4);
            else *dst = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        cp_async_wait_all();
        __syncthreads();
        const float* w0p = Ws + (rg * 2) * kLoraStride + l8;
        const float* x0p = Xs + (sg * 4) * kLoraStride + l8;
#pragma unroll 4
        for (int c = 0; c < kc; c += 8) {
            float w[2], x[4];
#pragma unroll
            for (int t = 0; t < 2; t++) w[t] = w0p[t * kLoraStride + c];
#pragma unroll
            for (int t = 0; t < 4; t++) x[t] = x0p[t * kLoraStride + c];
#pragma unroll
            for (int p = 0; p < 2; p++)
#pragma unroll
                for (int q = 0; q < 4; q++) acc[p][q] = __fadd_rn(acc[p][q], __fmul_rn(w[p], x[q]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int p = 0; p < 2; p++)
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
        for (int p = 0; p < 2; p++) {
            const int row = r0 + rg * 2 + p;
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
    const float* w2cat;    // [H][R][64] decay / a / v / gate up-projections, head-major (k_rw_put_up)
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

inline size_t wkv_smem(int R) {
    return ((size_t)kHS * R + (size_t)kWkvSB * R + (size_t)kWkvSB * 8 * kHS) * sizeof(float);
}

// CTA = one head x kWkvSB streams; thread (s, j) owns channel j of the head for stream s and row j
// of that stream's 64x64 state.  time_mixing_scratch steps 3-12 (model.rs:828-913) for one head.
__global__ void __launch_bounds__(kHS * kWkvSB) k_rw_wkv(RwStep sa, WkvArgs a) {
    extern __shared__ float sm[];
    __shared__ float s_st[kWkvSB][4];
    __shared__ uint64_t s_bar;
    __shared__ int s_abort;
    const int R = a.R, D = a.D;
    float* W = sm;                                  // [R][64] this head's up-projections
    float* hs = W + kHS * R;                        // [SB][R]
    float* vec = hs + kWkvSB * R;                   // [SB][8][64]
    const int h = blockIdx.x, n0 = blockIdx.y * kWkvSB;
    const int s = threadIdx.x >> 6, j = threadIdx.x & 63;
    const int b = n0 + s, c = h * kHS + j;
    const uint32_t wbytes = (uint32_t)(kHS * R * sizeof(float));
    if (threadIdx.x == 0) {  // the up-projections are constant: one bulk copy before the dependency wait
        tc::mbar_init(&s_bar, 1);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tc::mbar_expect_tx(&s_bar, wbytes);
        tc::bulk_load(W, a.w2cat + (size_t)h * R * kHS, wbytes, &s_bar);
    }
    // Everything except the LoRA hidden vectors is read before the dependency wait: the
    // projections r/k/v come from two kernels back, the state, v_first and the reset flags from
    // earlier still, and every kernel of the step waits for its predecessor before it lets the next
    // one start, so all of them are complete once this kernel runs.
    uint32_t slot = 0;
    bool act = b < sa.n;
    if (act) {
        slot = sa.slots[b];
        act = slot < (uint32_t)sa.cap;
    }
    const bool rf = act && sa.rflag[b] != 0u;
    const size_t cd = (size_t)sa.cap * D;
    float rr = 0.f, kv = 0.f, vv = 0.f, vf = 0.f;
    float S[kHS];
    float4* st = reinterpret_cast<float4*>(a.wkv + ((size_t)slot * a.H + h) * (kHS * kHS));
    if (act) {
        rr = a.rkv[(size_t)b * D + c];
        kv = a.rkv[cd + (size_t)b * D + c];
        vv = a.rkv[2 * cd + (size_t)b * D + c];
        if (!a.layer0) vf = a.v_first[(size_t)slot * D + c];
#pragma unroll
        for (int q = 0; q < kHS / 4; q++) {
            const float4 t = rf ? make_float4(0.f, 0.f, 0.f, 0.f) : st[q * kHS + j];
            S[4 * q] = t.x;
            S[4 * q + 1] = t.y;
            S[4 * q + 2] = t.z;
            S[4 * q + 3] = t.w;
        }
    }
    const float w0 = a.w0[c], a0 = a.a0[c], v0 = a.v0[c], k_k = a.k_k[c], k_a = a.k_a[c], r_k = a.r_k[c];
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < kWkvSB * R; i += blockDim.x) {
        const int ss = i / R, k = i - ss * R;
        hs[i] = n0 + ss < sa.n ? a.h1[(size_t)(n0 + ss) * R + k] : 0.0f;
    }
    if (threadIdx.x == 0 && !tc::mbar_wait(&s_bar, 0, &s_abort)) {
        tc::mbar_drain(&s_bar, 0);
        atomicOr(sa.err, 2u);
    }
    __syncthreads();
    if (s_abort) return;
    float* V = vec + s * 8 * kHS;  // 0 w, 1 kk*a, 2 k_mod, 3 r, 4 -kk, 5 v_out, 6 scratch, 7 bonus terms
    float g = 0.0f, vout = 0.0f, kk = 0.0f, aa = 0.0f;
    if (act) {
        const float* hb = hs + s * R;
        const float* wr = W + j;
        const float lw = dot8s(wr + a.seg_off[0] * kHS, kHS, hb + a.seg_off[0], a.seg_len[0]);
        const float la = dot8s(wr + a.seg_off[1] * kHS, kHS, hb + a.seg_off[1], a.seg_len[1]);
        g = dot8s(wr + a.seg_off[3] * kHS, kHS, hb + a.seg_off[3], a.seg_len[3]);
        const bool lane = c < (D & ~7);
        V[j] = decay_at(__fadd_rn(w0, lw), lane);                 // step 3
        aa = sigmoid_at(__fadd_rn(a0, la), lane);                 // step 4
        kk = __fmul_rn(kv, k_k);                                  // step 6
        const float kmod = __fmul_rn(kv, __fadd_rn(1.0f, __fmul_rn(__fsub_rn(aa, 1.0f), k_a)));  // step 7
        if (a.layer0) {                                           // step 8
            vout = vv;
            a.v_first[(size_t)slot * D + c] = vv;                 // state.v_first = v (model.rs:669-671)
        } else {
            const float lv = dot8s(wr + a.seg_off[2] * kHS, kHS, hb + a.seg_off[2], a.seg_len[2]);
            const float mix = sigmoid_at(__fadd_rn(v0, lv), lane);
            vout = __fadd_rn(vv, __fmul_rn(__fsub_rn(vf, vv), mix));
        }
        V[2 * kHS + j] = kmod;
        V[3 * kHS + j] = rr;
        V[5 * kHS + j] = vout;
        V[6 * kHS + j] = __fmul_rn(kk, kk);
        V[7 * kHS + j] = __fmul_rn(__fmul_rn(rr, a.g1k ? kmod : kv), r_k);  // step 11 terms
    }
    __syncthreads();
    if (j == 0 && act) {  // l2_normalize_per_head_inplace (tensor.rs:1416-1424)
        const float norm = __fsqrt_rn(seq_sum(V + 6 * kHS, kHS));
        s_st[s][0] = norm > 1e-12f ? __fdiv_rn(1.0f, norm) : 0.0f;
    }
    if (j == 32 && act) s_st[s][3] = seq_sum(V + 7 * kHS, kHS);  // bonus, in the other warp
    __syncthreads();
    if (act) {
        kk = __fmul_rn(kk, s_st[s][0]);
        V[kHS + j] = __fmul_rn(kk, aa);
        V[4 * kHS + j] = -kk;
    }
    __syncthreads();
    float o = 0.0f;
    if (act) {  // step 9, row i = j of this head's state
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
        const float var = __fdiv_rn(seq_sq_dev(V + 6 * kHS, kHS, mean), (float)kHS);
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
