// CUDA-core kernels of the Mamba-1 decode step (sm_100a).
//
// Step for n lockstep streams (reference: MambaModel::forward_multi,
// src/infrastructure/mamba/model.rs:773-935; plugin pool_forward, mamba_cuda.cu:604-635):
//   k_embed      token -> x (Q8: dequantised row), periodic-reset flag per stream
//   per layer:
//     k_norm       RMSNorm/LayerNorm of x -> f32 activation or Q8 digit planes
//     in_proj      GEMV (f32 or Q8) whose epilogue runs the causal conv1d + SiLU on the
//                  x-branch rows (updating the conv state) and stores the z-branch
//     x_proj       f32 GEMV -> (dt_raw, B, C)
//     k_scan       dt_proj + softplus + selective state update + D skip + z gate, emitting the
//                  next projection's activation (f32 or digit planes)
//     out_proj     GEMV whose epilogue adds the residual
//   k_norm (final) + head GEMV -> logits
//
// Layouts in HBM (all row-major):
//   weights      f32 [rows][K] or int8 [rows][K] + f32 scales [rows][K/64]
//   conv state   f32 [layer][slot][dc-1][d_inner]          (channel fastest: coalesced per tap)
//   ssm state    f32 [layer][slot][d_inner/64][d_state][64]  (64-channel blocks, channel fastest:
//                coalesced per state index, and one (slot, channel block) is 4 KiB contiguous)
//   activations  f32 [stream][K], or int8 digit planes [3][stream][K] + f32 2^e [stream][K/64]
#pragma once
#include "rk_math.cuh"

namespace rk {

constexpr int kDState = 16;
constexpr int kDConv = 4;
constexpr int kGroup = 64;

// Offsets of state element (tap or state index k, channel j) of a (layer, slot) in the layouts
// above; the SSM state pads d_inner to whole 64-channel blocks.  (A channel-blocked conv state was
// measured: the F32 path's per-(row, stream) epilogue ran 2.3x slower on it.)
__host__ __device__ __forceinline__ int state_blocks(int di) { return (di + 63) >> 6; }
__host__ __device__ __forceinline__ size_t conv_off(int layer, int cap, uint32_t slot, int di, int k, int j) {
    return (((size_t)layer * cap + slot) * (kDConv - 1) + k) * di + j;
}
__host__ __device__ __forceinline__ size_t ssm_off(int layer, int cap, uint32_t slot, int di, int k, int j) {
    return ((((size_t)layer * cap + slot) * state_blocks(di) + (j >> 6)) * kDState + k) * 64 + (j & 63);
}

// ------------------------------------------------------------------------------------------
// Load-time kernels
// ------------------------------------------------------------------------------------------

// Q8wMatrix::quantize (src/domain/gemv.rs:256-273): one warp per group of `group` consecutive
// floats; scale = max|w| / 127 (1 for an all-zero group), q = clamp(round(w * (1/scale))).
// roundf rounds half away from zero like Rust's f32::round.
__global__ void k_quantize_q8(const float* __restrict__ w, size_t n_groups, int group, int8_t* __restrict__ q,
                              float* __restrict__ scales) {
    size_t gi = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    int lane = threadIdx.x & 31;
    if (gi >= n_groups) return;
    const float* wg = w + gi * group;
    float amax = 0.0f;
    for (int i = lane; i < group; i += 32) amax = fmaxf(amax, fabsf(wg[i]));
    amax = warp_allmax(amax);
    float scale = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    float inv = __fdiv_rn(1.0f, scale);
    for (int i = lane; i < group; i += 32) {
        float r = roundf(__fmul_rn(wg[i], inv));
        r = fminf(fmaxf(r, -127.0f), 127.0f);
        q[gi * group + i] = (int8_t)(int)r;
    }
    if (lane == 0) scales[gi] = scale;
}

// Per-row scales broadcast to every 64-column group, so one kernel serves both Q8 variants.
__global__ void k_broadcast_scales(const float* __restrict__ row_scale, int rows, int groups,
                                   float* __restrict__ out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < (size_t)rows * groups) out[i] = row_scale[i / groups];
}

// Row-major int8 [rows][cols] -> tiled [cols/64][rows_pad][64] (rows >= rows are left as they are:
// the destination is zeroed first).
__global__ void k_tile_q8(const int8_t* __restrict__ src, int rows, int cols, int rows_pad, int8_t* __restrict__ dst) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 16-byte chunk
    size_t per_row = (size_t)cols / 16;
    if (i >= (size_t)rows * per_row) return;
    int r = (int)(i / per_row), k = (int)(i - (size_t)r * per_row) * 16;
    *reinterpret_cast<int4*>(dst + wq_off(rows_pad, r, k)) = *reinterpret_cast<const int4*>(src + (size_t)r * cols + k);
}

// A = exp(A_log) as the reference's lane_expf computes it (tensor.rs:1314), stored [16][di];
// conv weights transposed to [dc][di]; dt_proj weights transposed to [dr][di].
__global__ void k_prep_layer(const float* __restrict__ a_log, const float* __restrict__ conv_w,
                             const float* __restrict__ dt_w, int di, int dr, float* __restrict__ a_t,
                             float* __restrict__ conv_t, float* __restrict__ dt_wt) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= di) return;
#pragma unroll
    for (int n = 0; n < kDState; n++) a_t[n * di + j] = lane_expf(a_log[j * kDState + n]);
#pragma unroll
    for (int k = 0; k < kDConv; k++) conv_t[k * di + j] = conv_w[j * kDConv + k];
    for (int c = 0; c < dr; c++) dt_wt[(size_t)c * di + j] = dt_w[(size_t)j * dr + c];
}

// ------------------------------------------------------------------------------------------
// Per-step kernels
// ------------------------------------------------------------------------------------------

struct StepArgs {
    int n;                        // streams in this step
    int cap;                      // pool capacity (slots)
    const uint32_t* slots;        // [n] device
    const uint32_t* tokens;       // [n] device
    uint32_t* rflag;              // [n] 1 = this stream's state restarts from zero this step
    uint32_t* since;              // [cap] forwards since the slot's last reset
    uint32_t reset_every;         // 0 = never (host-driven resets only)
    uint32_t* err;                // device error word (bad slot/token seen on device)
    uint32_t* vslot;              // [n] out: the stream's slot, or kRejected for a bad slot/token
    uint32_t* bar = nullptr;      // grid-barrier counter of the fused step, zeroed here
};

// Embedding row + the periodic reset decision (MambaState::maybe_periodic_reset,
// src/infrastructure/mamba/model.rs:315-320): reset when since >= every, then since += 1.
// The state itself is never written here: every conv/scan read of a flagged stream uses zeros.
// A stream with a bad slot or token is rejected: its validated slot becomes kRejected, which every
// later kernel of the step treats as "no slot" (no state read or written, no counter change), and
// the final norm emits zeros for it, so its output row is all zeros.
__global__ void k_embed(StepArgs a, const float* __restrict__ emb_f, const int8_t* __restrict__ emb_q,
                        const float* __restrict__ emb_s, int d, int vocab, float* __restrict__ x) {
    pdl_wait();
    pdl_trigger();
    int b = blockIdx.x;
    if (a.bar && b == 0 && threadIdx.x == 0) *a.bar = 0u;
    if (b >= a.n) return;
    uint32_t tok = a.tokens[b], slot = a.slots[b];
    bool bad = tok >= (uint32_t)vocab || slot >= (uint32_t)a.cap;
    if (threadIdx.x == 0) {
        a.vslot[b] = bad ? kRejected : slot;
        if (bad) {
            atomicOr(a.err, 1u);
            a.rflag[b] = 0u;
        } else {
            uint32_t s = a.since[slot];
            uint32_t rf = (a.reset_every > 0 && s >= a.reset_every) ? 1u : 0u;
            a.since[slot] = rf ? 1u : (s == 0xffffffffu ? s : s + 1u);
            a.rflag[b] = rf;
        }
    }
    float* xb = x + (size_t)b * d;
    if (bad) {
        for (int j = threadIdx.x; j < d; j += blockDim.x) xb[j] = 0.0f;
        return;
    }
    if (emb_q) {  // dequant_row_into (src/domain/gemv.rs:284-295): q * scale (tiled int8 rows)
        const int vpad = round_up(vocab, 128);
        const float* sr = emb_s + (size_t)tok * (d / kGroup);
        for (int j = threadIdx.x; j < d; j += blockDim.x)
            xb[j] = __fmul_rn((float)emb_q[wq_off(vpad, (int)tok, j)], sr[j / kGroup]);
    } else {
        const float* er = emb_f + (size_t)tok * d;
        for (int j = threadIdx.x; j < d; j += blockDim.x) xb[j] = er[j];
    }
}

// Activation sink of a norm / scan: f32 vector or the three Q8 digit planes.
struct ActOut {
    float* f;       // [cap][K] f32, or nullptr
    int8_t* q;      // tiled digit planes [K/64][3][cap_pad][64], or nullptr
    float* e;       // [cap][kEStride] group scales 2^e
    int cap_pad;    // streams per plane, rounded up to 64
    int K;
};

// Norm of one stream by one warp (layer_norm_step, src/infrastructure/mamba/model.rs:193-200).
// Lane l owns columns 128c + 4l .. 128c + 4l + 3; sums are sequential per lane, then a butterfly.
// RMSNorm: x * (1 / sqrt(sum(x^2)/d + eps)) * w; LayerNorm: (x - mean) * inv_std * w + b.
// The norm's weight and bias columns of one lane (constant: loaded before the dependency wait).
template <int NC>
struct NormWeights {
    float4 w[NC], b[NC];
    __device__ __forceinline__ void load(const float* __restrict__ wp, const float* __restrict__ bp, int d, int lane) {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int k = c * 128 + lane * 4;
            w[c] = k < d ? __ldg(reinterpret_cast<const float4*>(wp + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
            b[c] = (bp && k < d) ? __ldg(reinterpret_cast<const float4*>(bp + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

// The stream's row, lane l holding columns 128c + 4l .. 128c + 4l + 3 (zeros past d).
template <int NC>
__device__ __forceinline__ void norm_load(const float* xb, int d, int lane, float4 (&v)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
        int k = c * 128 + lane * 4;
        v[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < d) v[c] = *reinterpret_cast<const float4*>(xb + k);
    }
}

// Normalises the loaded row in place (columns past d become zero).
template <int NC>  // NC = d / 128 rounded up; d <= 128 * NC
__device__ __forceinline__ void norm_apply(float4 (&v)[NC], int d, const NormWeights<NC>& nw, bool has_bias,
                                           int lane) {
    float mean = 0.0f, inv;
    if (has_bias) {
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            s = __fadd_rn(s, v[c].x); s = __fadd_rn(s, v[c].y); s = __fadd_rn(s, v[c].z); s = __fadd_rn(s, v[c].w);
        }
        s = warp_allsum(s);
        mean = __fdiv_rn(s, (float)d);
        float q = 0.0f;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int k = c * 128 + lane * 4;
            if (k < d) {
                float t;
                t = __fsub_rn(v[c].x, mean); q = __fmaf_rn(t, t, q);
                t = __fsub_rn(v[c].y, mean); q = __fmaf_rn(t, t, q);
                t = __fsub_rn(v[c].z, mean); q = __fmaf_rn(t, t, q);
                t = __fsub_rn(v[c].w, mean); q = __fmaf_rn(t, t, q);
            }
        }
        q = warp_allsum(q);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)d), 1e-5f)));
    } else {
        float q = 0.0f;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            q = __fmaf_rn(v[c].x, v[c].x, q); q = __fmaf_rn(v[c].y, v[c].y, q);
            q = __fmaf_rn(v[c].z, v[c].z, q); q = __fmaf_rn(v[c].w, v[c].w, q);
        }
        q = warp_allsum(q);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(q, (float)d), 1e-5f)));
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        int k = c * 128 + lane * 4;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k < d) {
            const float4 wv = nw.w[c];
            if (has_bias) {
                const float4 bv = nw.b[c];
                o.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].x, mean), inv), wv.x), bv.x);
                o.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].y, mean), inv), wv.y), bv.y);
                o.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].z, mean), inv), wv.z), bv.z);
                o.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].w, mean), inv), wv.w), bv.w);
            } else {
                o.x = __fmul_rn(__fmul_rn(v[c].x, inv), wv.x);
                o.y = __fmul_rn(__fmul_rn(v[c].y, inv), wv.y);
                o.z = __fmul_rn(__fmul_rn(v[c].z, inv), wv.z);
                o.w = __fmul_rn(__fmul_rn(v[c].w, inv), wv.w);
            }
        }
        v[c] = o;
    }
}

// Digit planes of a normalised row over 64-column groups: lanes 0-15 hold group 2c, lanes 16-31
// group 2c+1.  sink(k, d1x4, d2x4, d3x4, gs, lead) receives lane-packed digits of columns
// k .. k+3 (k < d only); `lead` marks the group's first lane, which also passes the exponent.
// (cmod, crem): emit only the chunks c with c % cmod == crem (several warps sharing one stream).
template <int NC, class Sink>
__device__ __forceinline__ void norm_emit_q(const float4 (&o)[NC], int d, int lane, Sink sink, int cmod = 1,
                                            int crem = 0) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c % cmod != crem) continue;
        int k = c * 128 + lane * 4;
        float m = fmaxf(fmaxf(fabsf(o[c].x), fabsf(o[c].y)), fmaxf(fabsf(o[c].z), fabsf(o[c].w)));
        m = warp_allmax(m, 16);
        float ginv, gs = group_scale(m, &ginv);
        if (k < d) {
            Digits3 a0 = split_digits(o[c].x, ginv), a1 = split_digits(o[c].y, ginv);
            Digits3 a2 = split_digits(o[c].z, ginv), a3 = split_digits(o[c].w, ginv);
            sink(k, pack4(a0.d1, a1.d1, a2.d1, a3.d1), pack4(a0.d2, a1.d2, a2.d2, a3.d2),
                 pack4(a0.d3, a1.d3, a2.d3, a3.d3), gs, (lane & 15) == 0);
        }
    }
}

// Norm of one stream by one warp into an activation sink (f32 row or tiled digit planes).
template <int NC>
__device__ __forceinline__ void norm_emit(int b, const float4 (&o)[NC], int d, const ActOut& out, int lane) {
    if (out.f) {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            int k = c * 128 + lane * 4;
            if (k < d) *reinterpret_cast<float4*>(out.f + (size_t)b * out.K + k) = o[c];
        }
        return;
    }
    // four consecutive columns stay inside one 16-byte chunk of the swizzled row
    norm_emit_q<NC>(o, d, lane, [&](int k, int p1, int p2, int p3, float gs, bool lead) {
        *reinterpret_cast<int*>(out.q + dq_off(out.cap_pad, 0, b, k)) = p1;
        *reinterpret_cast<int*>(out.q + dq_off(out.cap_pad, 1, b, k)) = p2;
        *reinterpret_cast<int*>(out.q + dq_off(out.cap_pad, 2, b, k)) = p3;
        if (lead) out.e[(size_t)b * kEStride + (k / kGroup)] = gs;
    });
}

// A rejected stream's normalised row is replaced by zeros (the final norm: zero logits).
template <int NC>
__device__ __forceinline__ void zero_if_rejected(float4 (&v)[NC], bool rejected) {
    if (!rejected) return;
#pragma unroll
    for (int c = 0; c < NC; c++) v[c] = make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int NC>
__device__ __forceinline__ void norm_row_warp(int b, const float* x, int d, const NormWeights<NC>& nw,
                                              bool has_bias, const ActOut& out, int lane, bool rejected) {
    float4 v[NC];
    norm_load<NC>(x + (size_t)b * d, d, lane, v);
    norm_apply<NC>(v, d, nw, has_bias, lane);
    zero_if_rejected<NC>(v, rejected);
    norm_emit<NC>(b, v, d, out, lane);
}

// One stream per warp.  vslot (the step's validated slots, or nullptr for a layer norm): rows of
// rejected streams come out as zeros.
template <int NC>
__global__ void k_norm(int n, const float* __restrict__ x, int d, const float* __restrict__ w,
                       const float* __restrict__ bias, ActOut out, const uint32_t* __restrict__ vslot) {
    NormWeights<NC> nw;
    nw.load(w, bias, d, threadIdx.x & 31);
    pdl_wait();
    pdl_trigger();
    int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= n) return;
    const bool rejected = vslot && vslot[b] == kRejected;
    norm_row_warp<NC>(b, x, d, nw, bias != nullptr, out, threadIdx.x & 31, rejected);
}

// ------------------------------------------------------------------------------------------
// GEMV epilogues: called once per (row, stream) with the finished dot product.
// ------------------------------------------------------------------------------------------

// Each epilogue also has a chunked form, apply<CH>(row, b0, nb, v): the CH streams b0..b0+nb-1
// of one row at once, with every load issued before any dependent arithmetic, so a thread that
// owns a row keeps CH memory operations in flight instead of walking the streams one by one.

// Stream metadata of a tile (slot and reset flag per stream), staged once per CTA; only the
// in_proj epilogue reads it.
struct TileMeta {
    const uint32_t* slot;   // [BN] tile-relative
    const uint32_t* fresh;  // [BN]
};

struct EpiStore {  // out[b][row] = v
    float* out;
    int ld;
    __device__ __forceinline__ void stage(int, int, uint32_t*, uint32_t*, int, int) const {}
    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH], TileMeta, int) const {
        apply<CH>(row, b0, nb, v);
    }
    __device__ __forceinline__ void operator()(int row, int b, float v) const { out[(size_t)b * ld + row] = v; }
    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH]) const {
#pragma unroll
        for (int i = 0; i < CH; i++)
            if (i < nb) out[(size_t)(b0 + i) * ld + row] = v[i];
    }
};

// The LM head's store when probabilities follow: the logits are stored as EpiStore does, and the
// tensor-core tile kernel also writes, for each of its streams, the (max, sum of exp(l - max)) of
// its 128 rows to red[stream][tile] (k_proj_q8_tc), so one normalising pass finishes the softmax
// without reading the logits twice.
struct EpiStoreSoftmax : EpiStore {
    float* red;  // [stream][parts][2]
    int parts;   // row tiles of the head
};
template <class E>
struct TileSoftmax {
    static constexpr bool value = false;
};
template <>
struct TileSoftmax<EpiStoreSoftmax> {
    static constexpr bool value = true;
};

struct EpiResidual {  // x[b][row] += v (src/infrastructure/mamba/model.rs:716-719)
    float* x;
    int ld;
    __device__ __forceinline__ void stage(int, int, uint32_t*, uint32_t*, int, int) const {}
    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH], TileMeta, int) const {
        apply<CH>(row, b0, nb, v);
    }
    __device__ __forceinline__ void operator()(int row, int b, float v) const {
        float* p = x + (size_t)b * ld + row;
        *p = __fadd_rn(*p, v);
    }
    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH]) const {
        float old[CH];
#pragma unroll
        for (int i = 0; i < CH; i++) old[i] = i < nb ? x[(size_t)(b0 + i) * ld + row] : 0.0f;
#pragma unroll
        for (int i = 0; i < CH; i++)
            if (i < nb) x[(size_t)(b0 + i) * ld + row] = __fadd_rn(old[i], v[i]);
    }
};

// One channel of the causal conv1d step + SiLU: taps t0..t3 over (s0, s1, s2, v), then the bias.
__device__ __forceinline__ float conv_silu_taps(float s0, float s1, float s2, float v, float t0, float t1, float t2,
                                                float t3, float bias) {
    float val = __fadd_rn(0.0f, __fmul_rn(s0, t0));
    val = __fadd_rn(val, __fmul_rn(s1, t1));
    val = __fadd_rn(val, __fmul_rn(s2, t2));
    val = __fadd_rn(val, __fmul_rn(v, t3));
    val = __fadd_rn(val, bias);
    return __fmul_rn(val, lane_sigmoid(val));
}

// in_proj epilogue: rows [0, di) are the x-branch, fed straight into the causal conv1d + SiLU
// (conv_silu_block, src/infrastructure/mamba/model.rs:134-153: val = sum_k st[k]*w[k] + x*w[3]
// + b, shift, SiLU); rows [di, 2di) are the gate z.
struct EpiInProj {
    int di, cap, layer;
    const uint32_t* slots;
    const uint32_t* rflag;
    float* conv_state;        // [layer][slot][3][di]
    const float* conv_t;      // [4][di]
    const float* conv_b;      // [di]
    float* conv_out;          // [stream][di]
    float* z;                 // [stream][di]
    bool defer = false;       // store the x-branch before the conv; k_xproj_part runs conv + SiLU

    __device__ __forceinline__ float conv_silu(int j, float s0, float s1, float s2, float v) const {
        return conv_silu_taps(s0, s1, s2, v, conv_t[j], conv_t[di + j], conv_t[2 * di + j], conv_t[3 * di + j],
                              conv_b[j]);
    }

    __device__ __forceinline__ void operator()(int row, int b, float v) const {
        if (row >= di) {
            z[(size_t)b * di + (row - di)] = v;
            return;
        }
        if (defer) {
            conv_out[(size_t)b * di + row] = v;
            return;
        }
        int j = row;
        uint32_t slot = slots[b];
        if (slot >= (uint32_t)cap) return;  // rejected stream (device-side check in k_embed)
        float* st = conv_state + conv_off(layer, cap, slot, di, 0, j);
        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
        if (!rflag[b]) {
            s0 = st[0];
            s1 = st[di];
            s2 = st[2 * di];
        }
        st[0] = s1;
        st[di] = s2;
        st[2 * di] = v;
        conv_out[(size_t)b * di + j] = conv_silu(j, s0, s1, s2, v);
    }

    // stage the slots and reset flags of streams b0..b0+nb-1 into tile-local arrays
    // (thread `tid` of `nthreads` cooperating threads)
    __device__ __forceinline__ void stage(int b0, int nb, uint32_t* slot_s, uint32_t* fresh_s, int tid,
                                          int nthreads) const {
        for (int i = tid; i < nb; i += nthreads) {
            uint32_t sl = slots[b0 + i];
            uint32_t rf = rflag[b0 + i];
            slot_s[i] = sl;
            fresh_s[i] = rf;
        }
    }

    // chunk of CH streams, tile-relative index t0 = b0 - tile start, metadata from the staged arrays
    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH], TileMeta meta,
                                          int t0) const {
        if (row >= di || defer) {
            float* dst = row >= di ? z + (row - di) : conv_out + row;
#pragma unroll
            for (int i = 0; i < CH; i++)
                if (i < nb) dst[(size_t)(b0 + i) * di] = v[i];
            return;
        }
        const int j = row;
        float* st[CH];
        bool live[CH], rd[CH];
#pragma unroll
        for (int i = 0; i < CH; i++) {
            uint32_t slot = i < nb ? meta.slot[t0 + i] : 0xffffffffu;
            live[i] = slot < (uint32_t)cap;
            rd[i] = live[i] && meta.fresh[t0 + i] == 0;
            st[i] = conv_state + conv_off(layer, cap, live[i] ? slot : 0u, di, 0, j);
        }
        float s0[CH], s1[CH], s2[CH];
#pragma unroll
        for (int i = 0; i < CH; i++) {
            s0[i] = rd[i] ? st[i][0] : 0.0f;
            s1[i] = rd[i] ? st[i][di] : 0.0f;
            s2[i] = rd[i] ? st[i][2 * di] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < CH; i++) {
            if (!live[i]) continue;
            st[i][0] = s1[i];
            st[i][di] = s2[i];
            st[i][2 * di] = v[i];
            conv_out[(size_t)(b0 + i) * di + j] = conv_silu(j, s0[i], s1[i], s2[i], v[i]);
        }
    }

    template <int CH>
    __device__ __forceinline__ void apply(int row, int b0, int nb, const float (&v)[CH]) const {
        if (row >= di || defer) {
            float* dst = row >= di ? z + (row - di) : conv_out + row;
#pragma unroll
            for (int i = 0; i < CH; i++)
                if (i < nb) dst[(size_t)(b0 + i) * di] = v[i];
            return;
        }
        const int j = row;
        float* st[CH];
        bool live[CH], fresh[CH];
#pragma unroll
        for (int i = 0; i < CH; i++) {
            uint32_t slot = i < nb ? slots[b0 + i] : 0xffffffffu;
            live[i] = slot < (uint32_t)cap;
            fresh[i] = live[i] && rflag[b0 + i] != 0;
            st[i] = conv_state + conv_off(layer, cap, live[i] ? slot : 0u, di, 0, j);
        }
        float s0[CH], s1[CH], s2[CH];
#pragma unroll
        for (int i = 0; i < CH; i++) {
            bool rd = live[i] && !fresh[i];
            s0[i] = rd ? st[i][0] : 0.0f;
            s1[i] = rd ? st[i][di] : 0.0f;
            s2[i] = rd ? st[i][2 * di] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < CH; i++) {
            if (!live[i]) continue;
            st[i][0] = s1[i];
            st[i][di] = s2[i];
            st[i][2 * di] = v[i];
            conv_out[(size_t)(b0 + i) * di + j] = conv_silu(j, s0[i], s1[i], s2[i], v[i]);
        }
    }
};

// ------------------------------------------------------------------------------------------
// F32 GEMV: y[b][r] = W[r] . act[b].  Per (row, stream) the recipe is fixed: lane l accumulates
// columns 128c + 4l + i (c ascending, i = 0..3) with FMA from zero, then a butterfly sum.
// The CTA tiles (streams x rows); rows within a warp share nothing in their arithmetic.
// Grid: x = stream tiles (fastest, so CTAs reading the same weight rows run together and the
// rows come from L2 after the first tile), y = row blocks of 8 * RW rows.
// ------------------------------------------------------------------------------------------
template <int RW, int NS, int NCH, class Epi>
__global__ void __launch_bounds__(256) k_gemv_f32(int M, int K, const float* __restrict__ W,
                                                  const float* __restrict__ act, int ld_act, int n, Epi epi) {
    extern __shared__ float4 smem_f4[];
    float* xs = reinterpret_cast<float*>(smem_f4);  // [NS][K]
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int r0 = blockIdx.y * (8 * RW) + warp * RW;
    // the weights are constant: with unrolled chunks, every weight load of the row(s) is issued
    // before the dependency wait (NCH x RW independent 16-byte loads per lane)
    constexpr int kNW = NCH > 0 ? NCH : 1;
    float4 wv[kNW][RW];
    if constexpr (NCH > 0) {
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            int k = c * 128 + lane * 4;
#pragma unroll
            for (int r = 0; r < RW; r++)
                wv[c][r] = (k < K && r0 + r < M)
                               ? __ldg(reinterpret_cast<const float4*>(W + (size_t)(r0 + r) * K + k))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    pdl_wait();
    pdl_trigger();
    int b0 = blockIdx.x * NS;
    int ns = min(NS, n - b0);
    int K4 = K >> 2;
    for (int i = threadIdx.x; i < ns * K4; i += blockDim.x) {
        int s = i / K4, k4 = i - s * K4;
        reinterpret_cast<float4*>(xs)[s * K4 + k4] =
            reinterpret_cast<const float4*>(act + (size_t)(b0 + s) * ld_act)[k4];
    }
    __syncthreads();
    if (r0 >= M) return;
    float acc[RW][NS];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int s = 0; s < NS; s++) acc[r][s] = 0.0f;
    if constexpr (NCH > 0) {
#pragma unroll
        for (int c = 0; c < NCH; c++) {
            int k = c * 128 + lane * 4;
            if (k < K) {
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    if (s < ns) {
                        float4 xv = *reinterpret_cast<const float4*>(xs + s * K + k);
#pragma unroll
                        for (int r = 0; r < RW; r++) {
                            acc[r][s] = __fmaf_rn(wv[c][r].x, xv.x, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[c][r].y, xv.y, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[c][r].z, xv.z, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[c][r].w, xv.w, acc[r][s]);
                        }
                    }
                }
            }
        }
    } else {
        // rolled chunk loop: the same per-element order, fewer registers
        int nch = (K + 127) >> 7;
        for (int c = 0; c < nch; c++) {
            int k = c * 128 + lane * 4;
            if (k < K) {
                float4 wv[RW];
#pragma unroll
                for (int r = 0; r < RW; r++)
                    wv[r] = (r0 + r < M) ? __ldg(reinterpret_cast<const float4*>(W + (size_t)(r0 + r) * K + k))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int s = 0; s < NS; s++) {
                    if (s < ns) {
                        float4 xv = *reinterpret_cast<const float4*>(xs + s * K + k);
#pragma unroll
                        for (int r = 0; r < RW; r++) {
                            acc[r][s] = __fmaf_rn(wv[r].x, xv.x, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[r].y, xv.y, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[r].z, xv.z, acc[r][s]);
                            acc[r][s] = __fmaf_rn(wv[r].w, xv.w, acc[r][s]);
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int s = 0; s < NS; s++) acc[r][s] = warp_allsum(acc[r][s]);
    // spread the epilogue over lanes: lane (r * NS + s) % 32 writes output (r, s)
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int s = 0; s < NS; s++)
            if (((r * NS + s) & 31) == lane && s < ns && r0 + r < M) epi(r0 + r, b0 + s, acc[r][s]);
}

// The same GEMV for 4 rows x 8 streams per warp (the large-batch shape), with the same bits and
// about half the instructions:
//  * the activations are staged as stream pairs interleaved by column, in lane order within each
//    128-column chunk ([pair][chunk][column half][lane][2 columns][2 streams]), so one
//    conflict-free 16-byte shared load gives a lane two columns of a stream pair, and each
//    (row, stream pair) runs its two
//    sequential FMA chains as one packed fma.rn.f32x2 (a fused multiply-add is the same operation
//    on the packed pipe; nothing is left to contract);
//  * the 32 lane sums of the warp's 32 outputs are reduced by a reduce-scatter over the same xor
//    butterfly (offsets 16, 8, 4, 2, 1): at each level a lane keeps the half of its outputs whose
//    index bit matches its own lane bit and adds its partner's copy, so every output gets exactly
//    warp_allsum's tree (IEEE addition is commutative) and lane l ends holding output l
//    (row l / 8, stream l % 8), with 62 shuffles instead of 160.
template <class Epi>
__global__ void __launch_bounds__(256) k_gemv_f32_p(int M, int K, const float* __restrict__ W,
                                                    const float* __restrict__ act, int ld_act, int n, Epi epi) {
    constexpr int RW = 4, NS = 8;
    extern __shared__ float4 smem_f4[];
    float* xs = reinterpret_cast<float*>(smem_f4);  // [NS / 2][nch][2][32][4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.y * (8 * RW) + warp * RW;
    pdl_wait();
    pdl_trigger();
    const int b0 = blockIdx.x * NS, ns = min(NS, n - b0);
    const int K4 = K >> 2, nch = (K + 127) >> 7;
    for (int i = threadIdx.x; i < NS * K4; i += blockDim.x) {
        const int s = i / K4, k4 = i - s * K4;  // columns 4 k4 .. 4 k4 + 3 = chunk c, lane k4 % 32
        const float4 v = s < ns ? reinterpret_cast<const float4*>(act + (size_t)(b0 + s) * ld_act)[k4]
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        float* d = xs + ((size_t)((s >> 1) * nch + (k4 >> 5)) * 2) * 128 + (k4 & 31) * 4 + (s & 1);
        d[0] = v.x;
        d[2] = v.y;
        d[128] = v.z;
        d[130] = v.w;
    }
    __syncthreads();
    if (r0 >= M) return;
    f2 acc[RW][NS / 2];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int q = 0; q < NS / 2; q++) acc[r][q] = f2_splat(0.0f);
    for (int c = 0; c < nch; c++) {
        const int k = c * 128 + lane * 4;
        if (k < K) {
            f2 w2[RW][4];
#pragma unroll
            for (int r = 0; r < RW; r++) {
                const float4 wv = (r0 + r < M) ? __ldg(reinterpret_cast<const float4*>(W + (size_t)(r0 + r) * K + k))
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
                w2[r][0] = f2_splat(wv.x);
                w2[r][1] = f2_splat(wv.y);
                w2[r][2] = f2_splat(wv.z);
                w2[r][3] = f2_splat(wv.w);
            }
#pragma unroll
            for (int q = 0; q < NS / 2; q++) {
                const float* xq = xs + ((size_t)(q * nch + c) * 2) * 128 + lane * 4;
                const float4 xa = *reinterpret_cast<const float4*>(xq);        // columns k, k + 1
                const float4 xb = *reinterpret_cast<const float4*>(xq + 128);  // columns k + 2, k + 3
                const f2 x0 = f2_pack(xa.x, xa.y), x1 = f2_pack(xa.z, xa.w);
                const f2 x2 = f2_pack(xb.x, xb.y), x3 = f2_pack(xb.z, xb.w);
#pragma unroll
                for (int r = 0; r < RW; r++) {
                    acc[r][q] = f2_fma(w2[r][0], x0, acc[r][q]);
                    acc[r][q] = f2_fma(w2[r][1], x1, acc[r][q]);
                    acc[r][q] = f2_fma(w2[r][2], x2, acc[r][q]);
                    acc[r][q] = f2_fma(w2[r][3], x3, acc[r][q]);
                }
            }
        }
    }
    // reduce-scatter: output j = r * 8 + s
    float v[32];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int q = 0; q < NS / 2; q++) f2_unpack(acc[r][q], v[r * 8 + 2 * q], v[r * 8 + 2 * q + 1]);
#pragma unroll
    for (int d = 16, L = 32; d >= 1; d >>= 1, L >>= 1) {
        const bool up = (lane & d) != 0;
#pragma unroll
        for (int i = 0; i < L / 2; i++) {
            const float keep = up ? v[L / 2 + i] : v[i];
            const float give = up ? v[i] : v[L / 2 + i];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, give, d));
        }
    }
    const int r = lane >> 3, sidx = lane & 7;
    if (sidx < ns && r0 + r < M) epi(r0 + r, b0 + sidx, v[0]);
}

// ------------------------------------------------------------------------------------------
// x_proj: (dt_raw, B, C)[b][r] = W_x[r] . conv_out[b] in a fixed two-level order.  Each 64-channel
// group g gives a sequential FMA chain over its channels from zero (xproj_chain); the group sums
// are then added in group order.  The fused step kernel evaluates the group chains in the CTAs
// that produce those channels and adds them in the same order, so both give the same bits.
// ------------------------------------------------------------------------------------------
constexpr int kXGroup = 64;

__device__ __forceinline__ float xproj_chain(const float* w, const float* x, int len) {
    float acc = 0.0f;
#pragma unroll 16
    for (int c = 0; c < len; c++) acc = __fmaf_rn(w[c], x[c], acc);
    return acc;
}

// The same chain with the weights read as 16-byte vectors (len == 64, w 16-byte aligned).
__device__ __forceinline__ float xproj_chain64_v(const float* __restrict__ w, const float* x) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float4 wv[16];
#pragma unroll
    for (int i = 0; i < 16; i++) wv[i] = __ldg(w4 + i);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        acc = __fmaf_rn(wv[i].x, x[4 * i], acc);
        acc = __fmaf_rn(wv[i].y, x[4 * i + 1], acc);
        acc = __fmaf_rn(wv[i].z, x[4 * i + 2], acc);
        acc = __fmaf_rn(wv[i].w, x[4 * i + 3], acc);
    }
    return acc;
}

// (dt_raw, B, C) of stream b: its x_proj group chains [G][M] added in group order.
__device__ __forceinline__ void xproj_sum_groups(const float* pb, int G, int M, float* out) {
    for (int r = threadIdx.x; r < M; r += blockDim.x) {
        float v[32];
        float tot = 0.0f;
        for (int g0 = 0; g0 < G; g0 += 32) {
#pragma unroll
            for (int q = 0; q < 32; q++) v[q] = g0 + q < G ? __ldcg(pb + (size_t)(g0 + q) * M + r) : 0.0f;
#pragma unroll
            for (int q = 0; q < 32; q++)
                if (g0 + q < G) tot = (g0 + q == 0) ? v[q] : __fadd_rn(tot, v[q]);
        }
        out[r] = tot;
    }
}

// Group chains of x_proj for one 64-channel group and a tile of SPB streams: part[b][g][r].  Grid
// (groups, stream tiles).  The group's weights [M][64] and activations [SPB][64] are staged in
// shared memory (rows padded to 68 floats), and each thread runs an RB-row x SK-stream block of
// chains with 16-byte shared loads (each weight and activation load feeds several chains); large
// batches use 64-stream tiles with 4 x 8 blocks, so the weights are staged once per 64 streams.
// The last of a stream tile's G CTAs (a per-tile arrival counter, reset by that CTA) adds each
// (stream, row)'s chains in group order into zp[b][r].
//
// With cv.on the activations are the in_proj x-branch before the conv (EpiInProj::defer): the
// staging pass runs the causal conv1d + SiLU of its (stream, channel) block exactly as the in_proj
// epilogue would (state shift, conv_silu_taps, rejected streams untouched), writes conv_out and the
// state, and stages the result.  Every (stream, channel) belongs to exactly one CTA, so converting
// conv_out in place is safe; many CTAs per SM keep far more state loads in flight than the
// tensor-core epilogue's eight warps.
struct XConv {
    bool on;
    int cap, layer;
    const uint32_t* slots;    // validated slots (kRejected: leave the stream alone)
    const uint32_t* rflag;    // per stream: read zeros instead of the stored state
    float* state;             // [layer][slot][3][di]
    const float* taps;        // [4][di]
    const float* bias;        // [di]
    float* out;               // conv_out, the same buffer as act
};

template <int SPB, int RB, int SK>
__global__ void __launch_bounds__(256) k_xproj_part(int M, int K, const float* __restrict__ W, const float* act,
                                                    int n, float* part, float* zp, uint32_t* tile_count, XConv cv) {
    static_assert(SPB % SK == 0, "stream blocks tile the stream tile");
    extern __shared__ float4 smem_f4[];
    float* xw = reinterpret_cast<float*>(smem_f4);  // [M][68]
    float* xc = xw + M * 68;                         // [SPB][68]
    const int g = blockIdx.x, G = gridDim.x, b0 = blockIdx.y * SPB, ns = min(SPB, n - b0);
    const int c0 = g * kXGroup, len = min(kXGroup, K - c0);
    const int tid = threadIdx.x;
    __shared__ float s_tap[5][kXGroup];  // conv taps 0..3 and bias of the group's channels
    __shared__ uint32_t s_slot[SPB], s_rd[SPB];
    if (cv.on && tid < kXGroup) {
#pragma unroll
        for (int k = 0; k < 4; k++) s_tap[k][tid] = tid < len ? __ldg(cv.taps + (size_t)k * K + c0 + tid) : 0.0f;
        s_tap[4][tid] = tid < len ? __ldg(cv.bias + c0 + tid) : 0.0f;
    }
    // the weights are constant: staged before the dependency wait, eight loads in flight per
    // thread before their stores
    for (int base = 0; base < M * 64; base += 8 * 256) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = base + u * 256 + tid, r = i >> 6, c = i & 63;
            v[u] = (i < M * 64 && c < len) ? __ldg(W + (size_t)r * K + c0 + c) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int i = base + u * 256 + tid;
            if (i < M * 64) xw[(i >> 6) * 68 + (i & 63)] = v[u];
        }
    }
    pdl_wait();
    pdl_trigger();
    if (!cv.on) {
        for (int base = 0; base < SPB * 64; base += 4 * 256) {
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * 256 + tid, sidx = i >> 6, c = i & 63;
                v[u] = (i < SPB * 64 && sidx < ns && c < len) ? act[(size_t)(b0 + sidx) * K + c0 + c] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = base + u * 256 + tid;
                if (i < SPB * 64) xc[(i >> 6) * 68 + (i & 63)] = v[u];
            }
        }
    } else {
        for (int i = tid; i < SPB; i += 256) {
            const uint32_t sl = i < ns ? cv.slots[b0 + i] : kRejected;
            s_slot[i] = sl;
            s_rd[i] = sl < (uint32_t)cv.cap && cv.rflag[b0 + i] == 0;
        }
        __syncthreads();
        // kU (stream, channel) elements per thread and pass: every load is issued before the
        // stores that could alias it
        constexpr int kU = SPB >= 64 ? 8 : 4;
        for (int base = 0; base < SPB * 64; base += kU * 256) {
            float x[kU], s0[kU], s1[kU], s2[kU];
            float* st[kU];
#pragma unroll
            for (int u = 0; u < kU; u++) {
                const int i = base + u * 256 + tid, sidx = i >> 6, c = i & 63;
                const bool in = i < SPB * 64 && sidx < ns && c < len;
                const uint32_t sl = in ? s_slot[sidx] : kRejected;
                const bool live = sl < (uint32_t)cv.cap, rd = live && s_rd[sidx];
                st[u] = live ? cv.state + conv_off(cv.layer, cv.cap, sl, K, 0, c0 + c) : nullptr;
                x[u] = live ? act[(size_t)(b0 + sidx) * K + c0 + c] : 0.0f;
                s0[u] = rd ? st[u][0] : 0.0f;
                s1[u] = rd ? st[u][K] : 0.0f;
                s2[u] = rd ? st[u][2 * K] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < kU; u++) {
                const int i = base + u * 256 + tid, sidx = i >> 6, c = i & 63;
                float y = 0.0f;
                if (st[u]) {
                    st[u][0] = s1[u];
                    st[u][K] = s2[u];
                    st[u][2 * K] = x[u];
                    y = conv_silu_taps(s0[u], s1[u], s2[u], x[u], s_tap[0][c], s_tap[1][c], s_tap[2][c], s_tap[3][c],
                                       s_tap[4][c]);
                    cv.out[(size_t)(b0 + sidx) * K + c0 + c] = y;
                }
                if (i < SPB * 64) xc[sidx * 68 + c] = y;
            }
        }
    }
    __syncthreads();
    // thread (row set rq, stream lane sl) runs rows rq + RQ i and streams sl + SQ j: consecutive
    // lanes read consecutive 68-float rows, so a warp's 16-byte shared loads hit distinct banks
    constexpr int SQ = SPB / SK;
    const int RQ = (M + RB - 1) / RB, nblk = RQ * SQ;
    for (int t = tid; t < nblk; t += 256) {
        const int rq = t / SQ, sl = t - rq * SQ;
        const float* wr[RB];
#pragma unroll
        for (int i = 0; i < RB; i++) wr[i] = xw + min(rq + RQ * i, M - 1) * 68;
        float acc[RB][SK];
#pragma unroll
        for (int i = 0; i < RB; i++)
#pragma unroll
            for (int j = 0; j < SK; j++) acc[i][j] = 0.0f;
        if (len == kXGroup) {
#pragma unroll 2
            for (int c = 0; c < 64; c += 4) {
                float4 w4[RB];
#pragma unroll
                for (int i = 0; i < RB; i++) w4[i] = *reinterpret_cast<const float4*>(wr[i] + c);
#pragma unroll
                for (int j = 0; j < SK; j++) {
                    const float4 xv = *reinterpret_cast<const float4*>(xc + (sl + SQ * j) * 68 + c);
#pragma unroll
                    for (int i = 0; i < RB; i++) {
                        acc[i][j] = __fmaf_rn(w4[i].x, xv.x, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w4[i].y, xv.y, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w4[i].z, xv.z, acc[i][j]);
                        acc[i][j] = __fmaf_rn(w4[i].w, xv.w, acc[i][j]);
                    }
                }
            }
        } else {  // a last, shorter group (F32 shapes only)
            for (int c = 0; c < len; c++)
#pragma unroll
                for (int j = 0; j < SK; j++)
#pragma unroll
                    for (int i = 0; i < RB; i++) acc[i][j] = __fmaf_rn(wr[i][c], xc[(sl + SQ * j) * 68 + c], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < RB; i++)
#pragma unroll
            for (int j = 0; j < SK; j++) {
                const int r = rq + RQ * i, sidx = sl + SQ * j;
                if (r < M && sidx < ns) part[((size_t)(b0 + sidx) * G + g) * M + r] = acc[i][j];
            }
    }
    __shared__ int s_last;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        s_last = atomicAdd(&tile_count[blockIdx.y], 1u) == (uint32_t)(G - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if ((M & 3) == 0 && G <= 32) {
        // thread = (stream, 4 consecutive rows): every group's 16 bytes requested at once
        const int nq = M >> 2;
        for (int o = tid; o < ns * nq; o += 256) {
            const int sidx = o / nq, r4 = (o - sidx * nq) * 4;
            const float4* pp = reinterpret_cast<const float4*>(part + (size_t)(b0 + sidx) * G * M + r4);
            float4 v[32];
#pragma unroll
            for (int q = 0; q < 32; q++) v[q] = q < G ? __ldcg(pp + (size_t)q * nq) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 t = v[0];
#pragma unroll
            for (int q = 1; q < 32; q++) {
                if (q < G) {
                    t.x = __fadd_rn(t.x, v[q].x);
                    t.y = __fadd_rn(t.y, v[q].y);
                    t.z = __fadd_rn(t.z, v[q].z);
                    t.w = __fadd_rn(t.w, v[q].w);
                }
            }
            *reinterpret_cast<float4*>(zp + (size_t)(b0 + sidx) * M + r4) = t;
        }
    } else {
        for (int sidx = 0; sidx < ns; sidx++)
            xproj_sum_groups(part + (size_t)(b0 + sidx) * G * M, G, M, zp + (size_t)(b0 + sidx) * M);
    }
    if (tid == 0) tile_count[blockIdx.y] = 0u;
}

// ------------------------------------------------------------------------------------------
// Q8 GEMV on CUDA cores (dp4a).  Lane l covers 16 bytes (quarter q = l & 3) of group slot
// gs = l >> 2; a warp covers 8 groups (512 weight bytes) per load.  The three digit sums of a
// group are exact int32, reduced across the 4 quarter lanes with integer shuffles; the row then
// accumulates its groups sequentially, g = 0..G-1, with group_accumulate().  The tensor-core
// kernel produces the same integers and runs the same combine, hence the same bits.
// Smem: digit planes of the NSB-stream tile [NSB][3][K] and group scales [NSB][G].
// ------------------------------------------------------------------------------------------
template <int RW, int NSB, int GI, class Epi>
__global__ void __launch_bounds__(256) k_gemv_q8(int M, int K, const int8_t* __restrict__ Wq,
                                                 const float* __restrict__ Ws, const int8_t* __restrict__ actq,
                                                 const float* __restrict__ acte, int cap_pad, int n, Epi epi) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float4 smem_f4[];
    int8_t* dq = reinterpret_cast<int8_t*>(smem_f4);                  // [NSB][3][K]
    float* de = reinterpret_cast<float*>(dq + (size_t)NSB * 3 * K);   // [NSB][G]
    const int G = K / kGroup;
    const int NS = q8_splits(G);
    int b0 = blockIdx.x * NSB;
    int ns = min(NSB, n - b0);
    int K16 = K >> 4;
    for (int i = threadIdx.x; i < ns * 3 * K16; i += blockDim.x) {
        int s = i / (3 * K16), rem = i - s * 3 * K16, p = rem / K16, k16 = rem - p * K16;
        reinterpret_cast<int4*>(dq)[(s * 3 + p) * K16 + k16] =
            *reinterpret_cast<const int4*>(actq + dq_off(cap_pad, p, b0 + s, k16 * 16));
    }
    for (int i = threadIdx.x; i < ns * G; i += blockDim.x) {
        int s = i / G, g = i - s * G;
        de[s * G + g] = acte[(size_t)(b0 + s) * kEStride + g];
    }
    __syncthreads();
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int gs = lane >> 2, qt = lane & 3;
    int r0 = blockIdx.y * (8 * RW) + warp * RW;
    const int mpad = round_up(M, 128);
#pragma unroll 1
    for (int r = r0; r < min(r0 + RW, M); r++) {
        int4 wv[GI];
#pragma unroll
        for (int gi = 0; gi < GI; gi++) {
            int g = gi * 8 + gs;
            wv[gi] = g < G ? __ldg(reinterpret_cast<const int4*>(Wq + wq_off(mpad, r, g * kGroup + qt * 16)))
                           : make_int4(0, 0, 0, 0);
        }
#pragma unroll 1
        for (int s = 0; s < ns; s++) {
            float val[GI];
#pragma unroll
            for (int gi = 0; gi < GI; gi++) {
                int g = gi * 8 + gs;
                int a1 = 0, a2 = 0, a3 = 0;
                if (g < G) {
                    const int8_t* base = dq + (size_t)s * 3 * K + g * kGroup + qt * 16;
                    int4 x1 = *reinterpret_cast<const int4*>(base);
                    int4 x2 = *reinterpret_cast<const int4*>(base + K);
                    int4 x3 = *reinterpret_cast<const int4*>(base + 2 * K);
                    a1 = __dp4a(wv[gi].x, x1.x, a1); a1 = __dp4a(wv[gi].y, x1.y, a1);
                    a1 = __dp4a(wv[gi].z, x1.z, a1); a1 = __dp4a(wv[gi].w, x1.w, a1);
                    a2 = __dp4a(wv[gi].x, x2.x, a2); a2 = __dp4a(wv[gi].y, x2.y, a2);
                    a2 = __dp4a(wv[gi].z, x2.z, a2); a2 = __dp4a(wv[gi].w, x2.w, a2);
                    a3 = __dp4a(wv[gi].x, x3.x, a3); a3 = __dp4a(wv[gi].y, x3.y, a3);
                    a3 = __dp4a(wv[gi].z, x3.z, a3); a3 = __dp4a(wv[gi].w, x3.w, a3);
                }
                a1 += __shfl_xor_sync(0xffffffffu, a1, 1); a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
                a2 += __shfl_xor_sync(0xffffffffu, a2, 1); a2 += __shfl_xor_sync(0xffffffffu, a2, 2);
                a3 += __shfl_xor_sync(0xffffffffu, a3, 1); a3 += __shfl_xor_sync(0xffffffffu, a3, 2);
                val[gi] = digit_value(a1, a2, a3);
            }
            // the split order of every Q8 projection path (q8_splits): groups accumulated in order
            // within each split, split sums added in split order
            float acc = 0.0f, tot = 0.0f;
            int sp = 0, send = (G * 1) / NS;
#pragma unroll
            for (int gi = 0; gi < GI; gi++) {
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    int g = gi * 8 + t;
                    float v = __shfl_sync(0xffffffffu, val[gi], t * 4);
                    if (g < G) {
                        acc = group_accumulate(acc, v, __ldg(Ws + (size_t)r * G + g), de[s * G + g]);
                        if (g + 1 == send) {
                            tot = sp == 0 ? acc : __fadd_rn(tot, acc);
                            acc = 0.0f;
                            sp++;
                            send = (G * (sp + 1)) / NS;
                        }
                    }
                }
            }
            if (lane == (s & 31)) epi(r, b0 + s, tot);
        }
    }
}

// ------------------------------------------------------------------------------------------
// Selective scan (scan_block + ssm_recurrence_d16_scalar, src/infrastructure/mamba/model.rs:174-190,
// src/domain/tensor.rs:1301-1325), per (stream, channel):
//   dt = softplus(dt_proj[j] . dt_raw + dt_bias[j])     (8-lane dot order of f32_rows)
//   if |dt| >= 1e-6: s[n] = exp(0 - dt*A[n]) * s[n] + (dt*x) * B[n]   (A = exp(A_log))
//   y = hsum_ssm(s[l]*C[l] + s[l+8]*C[l+8]) + D[j]*x;  gated = y * (z * sigmoid(z))
// Four threads share a channel: thread t owns the dot lanes {t, t+4} and the states
// {t, t+4, t+8, t+12}.  The reference's fixed trees map onto two shuffle levels:
//   hsum8     ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)):  pair sums, xor 2, then xor 1
//   hsum_ssm  ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)):  pair sums, xor 1, then xor 2
// so all four threads hold the reference's values.  A block is one 64-channel group of one
// stream (grid (d_inner/64, n), 256 threads), which is also the quantisation group of the
// out_proj activation digits.
// ------------------------------------------------------------------------------------------
struct ScanArgs {
    int di, dr, xr, cap, layer;
    const uint32_t* slots;
    const uint32_t* rflag;
    const float* zp;       // [stream][xr] = (dt_raw, B, C)
    const float* conv_out; // [stream][di]
    const float* z;        // [stream][di]
    const float* dt_wt;    // [dr][di] (transposed dt_proj weights)
    const float* dt_b;     // [di]
    const float* a_t;      // [16][di]
    const float* dvec;     // [di]
    float* ssm;            // [layer][slot][16][di]
    bool x_late = false;   // conv_out comes from the kernel just before (k_xproj_part with the conv):
                           //   read it after the dependency wait, not before
};

// One thread per channel (large batches: no repeated work) or four (small batches: shorter
// dependency chains per thread).  Both evaluate the same trees in the same order.
// One thread's pieces of the scan (the one-thread-per-channel form):
//   dt_dot8_body  dt_proj over the 8-aligned body of dt_rank, lane l accumulating columns c + l,
//                 then hsum8 ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)); w(c) is column c's weight
//   ssm_out16     hsum_ssm of s[l]*C[l] + s[l+8]*C[l+8]: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
template <class W>
__device__ __forceinline__ float dt_dot8_body(const float* zs, int body, W w) {
    float l[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < body; c += 8) {
#pragma unroll
        for (int q = 0; q < 8; q++) l[q] = __fadd_rn(l[q], __fmul_rn(w(c + q), zs[c + q]));
    }
    return __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[2], l[6])),
                     __fadd_rn(__fadd_rn(l[1], l[5]), __fadd_rn(l[3], l[7])));
}

// Row stride (words) of the stream-blocked scan's channel-major dt_proj copy: dt_rank rounded up
// to 8, plus 4, so 16-byte loads of eight consecutive channels hit distinct banks.
__host__ __device__ __forceinline__ int scan_blk_wstride(int dr) { return ((dr + 7) & ~7) + 4; }
constexpr int kScanAStride = 18;  // A's 16 states: 2 mod 4 words, so 8-byte loads are conflict-free

// dt_dot8_body with the channel's dt_proj row w (16-byte aligned, body a multiple of 8) and zs
// (16-byte aligned): lanes (l, l+1) as packed pairs, two 16-byte loads of each per 8 columns, the
// same partial sums and the same hsum8 tree ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).
__device__ __forceinline__ float dt_dot8_body_v(const float* zs, const float* w, int body, f2 z) {
    f2 l01 = f2_splat(0.0f), l23 = l01, l45 = l01, l67 = l01;
    for (int c = 0; c < body; c += 8) {
        const float4 w0 = *reinterpret_cast<const float4*>(w + c), w1 = *reinterpret_cast<const float4*>(w + c + 4);
        const float4 z0 = *reinterpret_cast<const float4*>(zs + c), z1 = *reinterpret_cast<const float4*>(zs + c + 4);
        l01 = f2_add(l01, f2_mulz(f2_pack(w0.x, w0.y), f2_pack(z0.x, z0.y), z));
        l23 = f2_add(l23, f2_mulz(f2_pack(w0.z, w0.w), f2_pack(z0.z, z0.w), z));
        l45 = f2_add(l45, f2_mulz(f2_pack(w1.x, w1.y), f2_pack(z1.x, z1.y), z));
        l67 = f2_add(l67, f2_mulz(f2_pack(w1.z, w1.w), f2_pack(z1.z, z1.w), z));
    }
    float r0, r1;  // ((l0+l4)+(l2+l6), (l1+l5)+(l3+l7))
    f2_unpack(f2_add(f2_add(l01, l45), f2_add(l23, l67)), r0, r1);
    return __fadd_rn(r0, r1);
}

// ssm_out16 with C 8-byte aligned: lanes (q, q+1) as packed pairs, the same tree.
__device__ __forceinline__ float ssm_out16_v(const float (&s)[kDState], const float* C, f2 z) {
    f2 ln[4];
#pragma unroll
    for (int q = 0; q < 8; q += 2)
        ln[q >> 1] = f2_add(f2_mulz(f2_pack(s[q], s[q + 1]), *reinterpret_cast<const f2*>(C + q), z),
                            f2_mulz(f2_pack(s[q + 8], s[q + 9]), *reinterpret_cast<const f2*>(C + q + 8), z));
    float p0, p1, q0, q1;  // (l0+l4, l1+l5), (l2+l6, l3+l7)
    f2_unpack(f2_add(ln[0], ln[2]), p0, p1);
    f2_unpack(f2_add(ln[1], ln[3]), q0, q1);
    return __fadd_rn(__fadd_rn(p0, p1), __fadd_rn(q0, q1));
}

__device__ __forceinline__ float ssm_out16(const float (&s)[kDState], const float* C) {
    float ln[8];
#pragma unroll
    for (int q = 0; q < 8; q++) ln[q] = __fadd_rn(__fmul_rn(s[q], C[q]), __fmul_rn(s[q + 8], C[q + 8]));
    return __fadd_rn(__fadd_rn(__fadd_rn(ln[0], ln[4]), __fadd_rn(ln[1], ln[5])),
                     __fadd_rn(__fadd_rn(ln[2], ln[6]), __fadd_rn(ln[3], ln[7])));
}

// The work of one CTA (256 threads): stream b, channel block blk.  `fill(zs)` puts the stream's
// x_proj output (dt_raw, B, C) into shared memory and synchronises the CTA; every operand that
// does not depend on it is loaded first.
template <int TPC, class Fill>
__device__ __forceinline__ void scan_block(const ScanArgs& a, const ActOut& out, int b, int blk, float* zs,
                                           float* s_max, Fill fill) {
    constexpr int kCh = 256 / TPC;           // channels per block
    constexpr int kSt = kDState / TPC;       // states per thread
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = TPC == 1 ? 0 : (lane & 3);
    const int jl = TPC == 1 ? threadIdx.x : warp * 8 + (lane >> 2);
    const int j = blk * kCh + jl;
    const uint32_t slot = a.slots[b];
    const bool ok = j < a.di && slot < (uint32_t)a.cap;
    const bool fresh = a.rflag[b] != 0;
    float* st = a.ssm + ssm_off(a.layer, a.cap, ok ? slot : 0u, a.di, 0, ok ? j : 0);
    // Everything except x_proj's (dt_raw, B, C) is read before the dependency wait: the state and
    // the reset flag come from earlier steps and kernels, conv_out and z from the in_proj two
    // launches back (complete, since every kernel waits for its predecessor before it lets the
    // next one start), the weights are constant.  With x_late conv_out is written by x_proj itself
    // and is read after the wait.
    float s[kSt];
#pragma unroll
    for (int k = 0; k < kSt; k++) s[k] = (ok && !fresh) ? st[(t + TPC * k) * 64] : 0.0f;
    const int jj = ok ? j : 0;
    float xv = a.x_late ? 0.0f : a.conv_out[(size_t)b * a.di + jj];
    const float zv = a.z[(size_t)b * a.di + jj];
    // dt_proj row, 8-lane dot order: lane l accumulates columns c + l of the 8-aligned body
    const float* wt = a.dt_wt + jj;
    const int body = a.dr & ~7;
    constexpr int kPre = 8;  // dt_proj columns c + t, c + t + 4 prefetched for dt_rank <= 64 (TPC = 4)
    float wa[kPre], wb[kPre];
    if constexpr (TPC != 1) {
#pragma unroll
        for (int i = 0; i < kPre; i++) {
            const int c = 8 * i;
            wa[i] = c < body ? __ldg(wt + (size_t)(c + t) * a.di) : 0.0f;
            wb[i] = c < body ? __ldg(wt + (size_t)(c + t + 4) * a.di) : 0.0f;
        }
    }
    float at[kSt];
#pragma unroll
    for (int k = 0; k < kSt; k++) at[k] = __ldg(a.a_t + (size_t)(t + TPC * k) * a.di + jj);
    const float dtb = __ldg(a.dt_b + jj), dv = __ldg(a.dvec + jj);
    fill(zs);
    if (a.x_late) xv = a.conv_out[(size_t)b * a.di + jj];
    float dt;
    if constexpr (TPC == 1) {
        dt = dt_dot8_body(zs, body, [&](int c) { return wt[(size_t)c * a.di]; });
    } else {
        // this thread holds lanes t and t+4; the quad finishes hsum8 with xor 2 then xor 1
        float la = 0.0f, lb = 0.0f;
#pragma unroll
        for (int i = 0; i < kPre; i++) {
            const int c = 8 * i;
            if (c < body) {
                la = __fadd_rn(la, __fmul_rn(wa[i], zs[c + t]));
                lb = __fadd_rn(lb, __fmul_rn(wb[i], zs[c + t + 4]));
            }
        }
        for (int c = 8 * kPre; c < body; c += 8) {
            la = __fadd_rn(la, __fmul_rn(wt[(size_t)(c + t) * a.di], zs[c + t]));
            lb = __fadd_rn(lb, __fmul_rn(wt[(size_t)(c + t + 4) * a.di], zs[c + t + 4]));
        }
        float pr = __fadd_rn(la, lb);
        pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
        dt = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 1));
    }
    for (int c = body; c < a.dr; c++) dt = __fadd_rn(dt, __fmul_rn(wt[(size_t)c * a.di], zs[c]));
    dt = softplus(__fadd_rn(dt, dtb));

    const float* B = zs + a.dr;
    const float* C = zs + a.dr + kDState;
    const bool update = !(fabsf(dt) < 1e-6f);
    if (update) {  // state pairs on the packed pipe (same bits)
        const f2 z2 = f2_zero(), dt2 = f2_splat(dt), dtx2 = f2_splat(__fmul_rn(dt, xv));
#pragma unroll
        for (int k = 0; k < kSt; k += 2) {
            const int n2 = t + TPC * k;
            const f2 arg = f2_sub(f2_splat(0.0f), f2_mulz(dt2, f2_pack(at[k], at[k + 1]), z2));
            const f2 sn = f2_add(f2_mulz(lane_expf2(arg, z2), f2_pack(s[k], s[k + 1]), z2),
                                 f2_mulz(dtx2, f2_pack(B[n2], B[n2 + TPC]), z2));
            f2_unpack(sn, s[k], s[k + 1]);
        }
    }
    if (ok && (update || fresh)) {
#pragma unroll
        for (int k = 0; k < kSt; k++) st[(t + TPC * k) * 64] = s[k];
    }
    // y = hsum_ssm(lanes) + D x, lanes[l] = s[l] C[l] + s[l+8] C[l+8],
    // hsum_ssm = ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
    float h;
    if constexpr (TPC == 1) {
        h = ssm_out16(s, C);
    } else {
        // states t, t+4, t+8, t+12 here: lanes t and t+4, then xor 1 and xor 2 across the quad
        const float l0 = __fadd_rn(__fmul_rn(s[0], C[t]), __fmul_rn(s[2], C[t + 8]));
        const float l4 = __fadd_rn(__fmul_rn(s[1], C[t + 4]), __fmul_rn(s[3], C[t + 12]));
        h = __fadd_rn(l0, l4);
        h = __fadd_rn(h, __shfl_xor_sync(0xffffffffu, h, 1));
        h = __fadd_rn(h, __shfl_xor_sync(0xffffffffu, h, 2));
    }
    const float y = __fadd_rn(h, __fmul_rn(dv, xv));
    const float gated = ok ? __fmul_rn(y, __fmul_rn(zv, lane_sigmoid(zv))) : 0.0f;
    if (out.f) {
        if (ok && t == 0) out.f[(size_t)b * out.K + j] = gated;
        return;
    }
    // digit planes over 64-channel groups: 64 / (32 / TPC) warps per group
    constexpr int kWarpsPerGroup = 64 * TPC / 32;
    float m = warp_allmax(fabsf(gated));
    if (lane == 0) s_max[warp] = m;
    __syncthreads();
    const int w0 = (warp / kWarpsPerGroup) * kWarpsPerGroup;
    m = s_max[w0];
#pragma unroll
    for (int w = 1; w < kWarpsPerGroup; w++) m = fmaxf(m, s_max[w0 + w]);
    if (!ok || t != 0) return;
    float ginv, gs = group_scale(m, &ginv);
    Digits3 dg = split_digits(gated, ginv);
    out.q[dq_off(out.cap_pad, 0, b, j)] = (int8_t)dg.d1;
    out.q[dq_off(out.cap_pad, 1, b, j)] = (int8_t)dg.d2;
    out.q[dq_off(out.cap_pad, 2, b, j)] = (int8_t)dg.d3;
    if ((j & (kGroup - 1)) == 0) out.e[(size_t)b * kEStride + j / kGroup] = gs;
}

template <int TPC>
__global__ void __launch_bounds__(256) k_scan(ScanArgs a, ActOut out) {
    extern __shared__ float4 smem_f4[];
    float* zs = reinterpret_cast<float*>(smem_f4);  // [xr]
    __shared__ float s_max[8];
    const int b = blockIdx.y;
    scan_block<TPC>(a, out, b, blockIdx.x, zs, s_max, [&](float* z) {
        pdl_wait();
        pdl_trigger();
        const float* zpb = a.zp + (size_t)b * a.xr;
        for (int i = threadIdx.x; i < a.xr; i += blockDim.x) z[i] = zpb[i];
        __syncthreads();
    });
}

// Large-batch scan: one CTA per (64-channel group, block of SB streams), thread = (channel, stream
// lane of 4), SB / 4 passes.  The group's dt_proj columns, A, dt bias and D are staged in shared
// memory once per CTA instead of being re-read from L2 for every stream (the one-stream CTAs of
// k_scan), and the next pass's state, conv output and z are loaded while the current pass
// computes.  The arithmetic is scan_block<1>'s (same bits); d_inner must be a multiple of 64.
// 32-stream blocks (1,024 streams: 79 vs 90 us) run three CTAs per SM, 16-stream blocks two.
template <int SB>
__global__ void __launch_bounds__(256, SB >= 32 ? 3 : 2) k_scan_blk(ScanArgs a, ActOut out, int n) {
    extern __shared__ float4 smem_f4[];
    // channel-major copies of the group's operands, so a thread's columns are wide shared loads
    // without bank conflicts: dt_proj [64][ws] (16-byte loads, row stride 4 mod 8 words) and A
    // [64][18] (8-byte loads, 2 mod 4), then the dt bias and D [64] each, then (dt_raw, B, C) of
    // the block's streams [SB][xr] (xr and dt_rank multiples of 4)
    const int ws = scan_blk_wstride(a.dr);
    float* wt = reinterpret_cast<float*>(smem_f4);
    float* atc = wt + 64 * ws;
    float* w = atc + 64 * kScanAStride;              // [64] dt bias, [64] D
    float* zs = w + 2 * 64;
    __shared__ float s_max[2][8];
    const int g = blockIdx.x, b0 = blockIdx.y * SB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ch = tid & 63, sl = tid >> 6, j = g * 64 + ch;
    // constant operands (before the dependency wait): the group's columns, coalesced reads
    for (int i = tid; i < a.dr * 64; i += 256)
        wt[(i & 63) * ws + (i >> 6)] = __ldg(a.dt_wt + (size_t)(i >> 6) * a.di + g * 64 + (i & 63));
    for (int i = tid; i < kDState * 64; i += 256)
        atc[(i & 63) * kScanAStride + (i >> 6)] = __ldg(a.a_t + (size_t)(i >> 6) * a.di + g * 64 + (i & 63));
    if (tid < 64) {
        w[tid] = __ldg(a.dt_b + j);
        w[64 + tid] = __ldg(a.dvec + j);
    }
    // one pass's per-thread operands: state, conv output, z (written by earlier kernels)
    struct Op {
        float s[kDState];
        float xv, zv;
        bool ok, fresh;
        uint32_t slot;
    };
    auto load = [&](int pass, Op& o, bool with_x) {
        const int b = b0 + pass * 4 + sl;
        o.ok = false;
        o.fresh = false;
        o.slot = 0;
        o.xv = o.zv = 0.0f;
        if (b < n) {
            o.slot = a.slots[b];
            o.ok = o.slot < (uint32_t)a.cap;
            o.fresh = a.rflag[b] != 0;
            if (with_x) o.xv = a.conv_out[(size_t)b * a.di + j];
            o.zv = a.z[(size_t)b * a.di + j];
        }
        const float* st = a.ssm + ssm_off(a.layer, a.cap, o.ok ? o.slot : 0u, a.di, 0, j);
#pragma unroll
        for (int k = 0; k < kDState; k++) o.s[k] = (o.ok && !o.fresh) ? st[k * 64] : 0.0f;
    };
    const f2 z2 = f2_zero();
    Op cur;
    load(0, cur, !a.x_late);
    pdl_wait();
    pdl_trigger();
    if (a.x_late && b0 + sl < n) cur.xv = a.conv_out[(size_t)(b0 + sl) * a.di + j];
    for (int i = tid; i < SB * a.xr; i += 256) {
        const int s = i / a.xr, b = b0 + s;
        zs[i] = b < n ? a.zp[(size_t)b * a.xr + (i - s * a.xr)] : 0.0f;
    }
    __syncthreads();
    const float* wrow = wt + ch * ws;
    const float* arow = atc + ch * kScanAStride;
    const float dtb = w[ch], dv = w[64 + ch];
    const int body = a.dr & ~7;
    for (int pass = 0; pass < SB / 4; pass++) {
        Op nxt;
        if (pass + 1 < SB / 4) load(pass + 1, nxt, true);
        const int s = pass * 4 + sl, b = b0 + s;
        const float* zb = zs + s * a.xr;
        float dt = dt_dot8_body_v(zb, wrow, body, z2);
        for (int c = body; c < a.dr; c++) dt = __fadd_rn(dt, __fmul_rn(wrow[c], zb[c]));
        dt = softplus(__fadd_rn(dt, dtb));
        const float* B = zb + a.dr;
        const float* C = zb + a.dr + kDState;
        const bool update = !(fabsf(dt) < 1e-6f);
        if (update) {
            // states in pairs on the packed f32x2 pipe: the same per-state operations and bits
            const f2 dt2 = f2_splat(dt), dtx2 = f2_splat(__fmul_rn(dt, cur.xv));
#pragma unroll
            for (int k = 0; k < kDState; k += 2) {
                const f2 arg = f2_sub(f2_splat(0.0f), f2_mulz(dt2, *reinterpret_cast<const f2*>(arow + k), z2));
                const f2 da = lane_expf2(arg, z2);
                const f2 sn = f2_add(f2_mulz(da, f2_pack(cur.s[k], cur.s[k + 1]), z2),
                                     f2_mulz(dtx2, *reinterpret_cast<const f2*>(B + k), z2));
                f2_unpack(sn, cur.s[k], cur.s[k + 1]);
            }
        }
        if (cur.ok && (update || cur.fresh)) {
            float* st = a.ssm + ssm_off(a.layer, a.cap, cur.slot, a.di, 0, j);
#pragma unroll
            for (int k = 0; k < kDState; k++) st[k * 64] = cur.s[k];
        }
        const float y = __fadd_rn(ssm_out16_v(cur.s, C, z2), __fmul_rn(dv, cur.xv));
        const float gated = cur.ok ? __fmul_rn(y, __fmul_rn(cur.zv, lane_sigmoid(cur.zv))) : 0.0f;
        if (out.f) {
            if (cur.ok) out.f[(size_t)b * out.K + j] = gated;
        } else {
            // digit planes over the stream's 64 channels (warps 2 sl, 2 sl + 1)
            float m = warp_allmax(fabsf(gated));
            if (lane == 0) s_max[pass & 1][warp] = m;
            __syncthreads();
            m = fmaxf(s_max[pass & 1][warp & ~1], s_max[pass & 1][warp | 1]);
            if (cur.ok) {
                float ginv, gs = group_scale(m, &ginv);
                const Digits3 dg = split_digits(gated, ginv);
                out.q[dq_off(out.cap_pad, 0, b, j)] = (int8_t)dg.d1;
                out.q[dq_off(out.cap_pad, 1, b, j)] = (int8_t)dg.d2;
                out.q[dq_off(out.cap_pad, 2, b, j)] = (int8_t)dg.d3;
                if (ch == 0) out.e[(size_t)b * kEStride + g] = gs;
            }
        }
        if (pass + 1 < SB / 4) cur = nxt;
    }
}

// Zero the conv and SSM state of the listed slots in every layer, and their reset counters.
__global__ void k_zero_slots(const uint32_t* __restrict__ slots, int n_slots, int cap, int layers, int di,
                             float* __restrict__ conv, float* __restrict__ ssm, uint32_t* __restrict__ since) {
    const int cb = (kDConv - 1) * di, sb = state_blocks(di) * 64 * kDState;
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    int k = blockIdx.y;
    int layer = blockIdx.z;
    if (k >= n_slots) return;
    uint32_t slot = slots[k];
    if (slot >= (uint32_t)cap) return;
    if (i < cb + sb) {  // a (layer, slot)'s conv and ssm state are each one contiguous block
        if (i < cb) conv[conv_off(layer, cap, slot, di, 0, 0) + i] = 0.0f;
        else ssm[ssm_off(layer, cap, slot, di, 0, 0) + (i - cb)] = 0.0f;
    }
    if (i == 0 && layer == 0) since[slot] = 0u;
}

}  // namespace rk
