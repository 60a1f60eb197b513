// Device arithmetic shared by every kernel of the decode step.
//
// Two rules hold throughout:
//  * Element-wise math (exp, ln, softplus, sigmoid, the conv tap sum, the SSM update) is the
//    reference CPU path's own operation sequence written with explicitly rounded IEEE
//    operations (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn), so nvcc cannot contract or
//    reorder it.  Given the same inputs these produce the reference's bits
//    (src/domain/tensor.rs:765-861 Cephes exp / musl ln / softplus, :877-891 lane sigmoid).
//  * Reductions use fixed trees that depend only on the element's own data, never on the
//    batch size, the batch position or the slot, and no float atomics anywhere.  That is what
//    makes a stream's logits bit-identical for every n (the determinism contract of
//    docs/api/PLUGIN-FFI-V2.md section 4).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace rk {

// ---- Cephes exp (tensor.rs:765-794) -------------------------------------------------------
constexpr float kExpLo = -87.3365447505531f;
constexpr float kExpHi = 88.3762626647949f;

__device__ __forceinline__ float cephes_exp_core(float x) {
    const float LOG2E = 1.44269504088896341f;
    const float LN2_HI = 6.93145751953125E-1f;
    const float LN2_LO = 1.42860682030941723212E-6f;
    const float P0 = 1.9875691500E-4f, P1 = 1.3981999507E-3f, P2 = 8.3334519073E-3f;
    const float P3 = 4.1665795894E-2f, P4 = 1.6666665459E-1f, P5 = 5.0000001201E-1f;
    float fx = __fmul_rn(x, LOG2E);
    // round half to even with the reference's 2^23 magic-constant trick (|fx| < 2^22 here); the
    // integer comes from the same sum's bits, so no float-to-int conversion unit is involved
    const float big = __fadd_rn(fx, 12582912.0f);
    float nf = __fsub_rn(big, 12582912.0f);
    int n = __float_as_int(big) - 0x4B400000;
    float r = __fsub_rn(__fsub_rn(x, __fmul_rn(nf, LN2_HI)), __fmul_rn(nf, LN2_LO));
    float r2 = __fmul_rn(r, r);
    float y = P0;
    y = __fadd_rn(__fmul_rn(y, r), P1);
    y = __fadd_rn(__fmul_rn(y, r), P2);
    y = __fadd_rn(__fmul_rn(y, r), P3);
    y = __fadd_rn(__fmul_rn(y, r), P4);
    y = __fadd_rn(__fmul_rn(y, r), P5);
    y = __fadd_rn(__fadd_rn(__fmul_rn(y, r2), r), 1.0f);
    float pow2n = __int_as_float((int)(((unsigned)(n + 127)) << 23));
    return __fmul_rn(y, pow2n);
}

// portable_expf: clamp keeps NaN as NaN.
__device__ __forceinline__ float portable_expf(float x) {
    x = x < kExpLo ? kExpLo : (x > kExpHi ? kExpHi : x);
    return cephes_exp_core(x);
}

// lane_expf (tensor.rs:877-879): one lane of the SIMD exp, a NaN lane becomes exp(kExpLo).
__device__ __forceinline__ float lane_expf(float x) {
    x = (x != x) ? kExpLo : x;
    x = x < kExpLo ? kExpLo : (x > kExpHi ? kExpHi : x);
    return cephes_exp_core(x);
}

// ---- Two lanes per instruction (sm_100 packed f32x2) -------------------------------------
// add/sub/mul/fma.rn.f32x2 round each 32-bit half exactly as the scalar .rn instruction does (no
// flush to zero), so a pair of element-wise chains can run with half the instructions.  One trap:
// the assembler contracts a packed multiply that feeds a packed add into one fused multiply-add
// even with .rn (measured: about 1 % of Cephes exps one ulp off), which the scalar __fmul_rn /
// __fadd_rn never allow.  So every product that feeds an add or subtract is written as
// fma(a, b, z) with z = -0.0 held in memory the compiler cannot see into (g_f2_zero): that is the
// correctly rounded product (x + -0 = x for every x, including +0 and -0), and nothing is left to
// contract.  f2 holds (lo, hi) in one 64-bit register pair.
typedef unsigned long long f2;

__device__ float g_f2_zero = -0.0f;  // never written

__device__ __forceinline__ f2 f2_pack(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(f2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 f2_splat(float v) { return f2_pack(v, v); }
// (-0.0, -0.0) as a run-time value: read once per thread, passed to f2_mulz
__device__ __forceinline__ f2 f2_zero() { return f2_splat(*(volatile const float*)&g_f2_zero); }
__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {  // only where the product feeds no add
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_mulz(f2 a, f2 b, f2 z) {  // a * b rounded once, never contracted
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(z));
    return r;
}
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {  // a * b + c rounded once
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ f2 f2_add(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 f2_sub(f2 a, f2 b) {
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// lane_expf of both halves (z from f2_zero): the clamp per half (a NaN half becomes kExpLo, as
// fmaxf returns the non-NaN operand), cephes_exp_core's operations as packed pairs, and the 2^n
// scale from the magic-sum bits of both halves at once: bits - (0x4B400000 - 127) is n + 127 in
// [1, 255] per half (no borrow across halves), and shifting the 64-bit pair left by 23 moves each
// half's 8-bit value into its own exponent field.
__device__ __forceinline__ f2 lane_expf2(f2 x, f2 z) {
    float x0, x1;
    f2_unpack(x, x0, x1);
    const f2 xc = f2_pack(fminf(fmaxf(x0, kExpLo), kExpHi), fminf(fmaxf(x1, kExpLo), kExpHi));
    const f2 fx = f2_mulz(xc, f2_splat(1.44269504088896341f), z);
    const f2 big = f2_add(fx, f2_splat(12582912.0f));
    const f2 nf = f2_sub(big, f2_splat(12582912.0f));
    const f2 r = f2_sub(f2_sub(xc, f2_mulz(nf, f2_splat(6.93145751953125E-1f), z)),
                        f2_mulz(nf, f2_splat(1.42860682030941723212E-6f), z));
    const f2 r2 = f2_mul(r, r);
    f2 y = f2_add(f2_mulz(f2_splat(1.9875691500E-4f), r, z), f2_splat(1.3981999507E-3f));
    y = f2_add(f2_mulz(y, r, z), f2_splat(8.3334519073E-3f));
    y = f2_add(f2_mulz(y, r, z), f2_splat(4.1665795894E-2f));
    y = f2_add(f2_mulz(y, r, z), f2_splat(1.6666665459E-1f));
    y = f2_add(f2_mulz(y, r, z), f2_splat(5.0000001201E-1f));
    y = f2_add(f2_add(f2_mulz(y, r2, z), r), f2_splat(1.0f));
    const f2 pow2n = (big - 0x4B3FFF814B3FFF81ull) << 23;
    return f2_mul(y, pow2n);
}

// ---- musl/FreeBSD logf (tensor.rs:799-837) ------------------------------------------------
__device__ __forceinline__ float portable_lnf(float x) {
    const float LN2_HI = 6.9313812256e-01f, LN2_LO = 9.0580006145e-06f;
    const float LG1 = 0.66666662693f, LG2 = 0.40000972152f, LG3 = 0.28498786688f, LG4 = 0.24279078841f;
    unsigned ix = __float_as_uint(x);
    int k = 0;
    if (ix < 0x00800000u || (ix >> 31) != 0) {
        if ((ix << 1) == 0) return __int_as_float(0xff800000);  // -inf
        if ((ix >> 31) != 0) return __int_as_float(0x7fc00000);  // NaN
        k -= 25;
        ix = __float_as_uint(__fmul_rn(x, __uint_as_float(0x4c000000u)));
    } else if (ix >= 0x7f800000u) {
        return x;
    } else if (ix == 0x3f800000u) {
        return 0.0f;
    }
    ix = ix + (0x3f800000u - 0x3f3504f3u);
    k += (int)(ix >> 23) - 0x7f;
    ix = (ix & 0x007fffffu) + 0x3f3504f3u;
    float xn = __uint_as_float(ix);
    float f = __fsub_rn(xn, 1.0f);
    float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
    float dk = (float)k;
    float z = __fmul_rn(s, s);
    float w = __fmul_rn(z, z);
    float t1 = __fmul_rn(w, __fadd_rn(LG2, __fmul_rn(w, LG4)));
    float t2 = __fmul_rn(z, __fadd_rn(LG1, __fmul_rn(w, LG3)));
    float r = __fadd_rn(t2, t1);
    float hfsq = __fmul_rn(__fmul_rn(0.5f, f), f);
    // s * (hfsq + r) + dk * LN2_LO - hfsq + f + dk * LN2_HI, evaluated left to right
    float acc = __fmul_rn(s, __fadd_rn(hfsq, r));
    acc = __fadd_rn(acc, __fmul_rn(dk, LN2_LO));
    acc = __fsub_rn(acc, hfsq);
    acc = __fadd_rn(acc, f);
    return __fadd_rn(acc, __fmul_rn(dk, LN2_HI));
}

// portable_softplus (tensor.rs:859-861): threshold 20.
__device__ __forceinline__ float softplus(float x) {
    return x > 20.0f ? x : portable_lnf(__fadd_rn(1.0f, portable_expf(x)));
}

// lane_sigmoidf (tensor.rs:881-885): 1 / (1 + exp(0 - x)).
__device__ __forceinline__ float lane_sigmoid(float x) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, lane_expf(__fsub_rn(0.0f, x))));
}

// ---- Fixed reduction trees ----------------------------------------------------------------

// Butterfly sum over the 32 lanes: every lane ends with the same value (float addition is
// commutative, and each level pairs equal partial sums), independent of any other warp.
__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ float warp_allmax(float v, int width = 32) {
    for (int off = width >> 1; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// ---- Activation digits for the Q8 projections ---------------------------------------------
//
// A Q8 projection computes y[r] = sum_g scale[r,g] * sum_{c in g} q[r,c] * x[c] over 64-column
// groups g (Q8_GROUP, src/infrastructure/mamba/model.rs:50-56).  The engine evaluates each
// group sum with exact integer arithmetic: x restricted to group g is written as
//     x ~= 2^e * (d1 + d2 * 2^-7 + d3 * 2^-14),  d1, d2, d3 integers in [-64, 64],
// where 2^e is chosen so that max|x_g| * 2^-e lies in [32, 64).  The three int8 digit planes
// multiply the int8 weights with int32 accumulation (dp4a on CUDA cores, tcgen05 kind::i8 on
// the tensor cores); |sum| <= 64*127*64 < 2^24, so every group sum is exact, in any order, on
// any unit.  The digits keep 20 significant bits relative to the group maximum.  Only the
// per-group combine below rounds, and it runs in the same order on every path, so the CUDA-core
// and tensor-core projections produce identical bits at every batch size.

constexpr float kDigitTiny = 7.888609052210118e-31f;  // 2^-100: smaller groups encode as zero

struct Digits3 {
    int d1, d2, d3;
};

// e_bits: exponent scale for a group whose max |x| is m.  Returns 2^e as a float and
// 2^-e in *inv (both exact powers of two); a zero (or below 2^-100) group gives 0 / 0.
__device__ __forceinline__ float group_scale(float m, float* inv) {
    if (!(m >= kDigitTiny)) {  // also maps NaN to a zero group
        *inv = 0.0f;
        return 0.0f;
    }
    int E = (int)((__float_as_uint(m) >> 23) & 0xff) - 127;  // floor(log2 m) for normal m
    int e = E - 5;                                             // m * 2^-e in [32, 64)
    *inv = __uint_as_float((unsigned)(127 - e) << 23);
    return __uint_as_float((unsigned)(127 + e) << 23);
}

// round(t) to nearest-even for |t| < 2^22, as a float and as an int: t + 1.5 * 2^23 lands where the
// spacing is 1, so the sum is already rounded and its low mantissa bits are the integer.
__device__ __forceinline__ float round_even_small(float t, int* i) {
    const float big = __fadd_rn(t, 12582912.0f);
    *i = __float_as_int(big) - 0x4B400000;
    return __fsub_rn(big, 12582912.0f);
}

__device__ __forceinline__ Digits3 split_digits(float x, float inv) {
    float t = __fmul_rn(x, inv);  // exact: power-of-two scaling, |t| < 64
    Digits3 r;
    float d1 = round_even_small(t, &r.d1);
    float t2 = __fmul_rn(__fsub_rn(t, d1), 128.0f);  // both exact
    float d2 = round_even_small(t2, &r.d2);
    float t3 = __fmul_rn(__fsub_rn(t2, d2), 128.0f);
    round_even_small(t3, &r.d3);
    return r;
}

// Exact int -> float for |a| < 2^22 without the conversion unit: the bits 0x4B400000 + a are
// the float 1.5 * 2^23 + a (integer spacing there is 1), and subtracting 1.5 * 2^23 is exact.
__device__ __forceinline__ float small_int_to_float(int a) {
    return __fsub_rn(__int_as_float(0x4B400000 + a), 12582912.0f);
}

// Combine the three exact digit sums of one group: ((a1 + a2 * 2^-7) + a3 * 2^-14).
// |a_i| <= 64 * 127 * 64 < 2^22, so each conversion is exact.
// a2 * 2^-7 and a3 * 2^-14 are exact, so each fused multiply-add rounds exactly once, like the
// separate add it replaces.
__device__ __forceinline__ float digit_value(int a1, int a2, int a3) {
    float v = __fmaf_rn(small_int_to_float(a2), 0.0078125f, small_int_to_float(a1));
    return __fmaf_rn(small_int_to_float(a3), 6.103515625e-05f, v);
}

// digit_value + group_accumulate of two streams of one row and group on the packed pipe: the same
// operations per lane (exact conversions, the two exact-product FMAs, rn(ws * ae), the product
// written with f2_mulz so it cannot be contracted into the add), so the same bits.
__device__ __forceinline__ void group_accumulate2(float& acc0, float& acc1, int a1_0, int a1_1, int a2_0, int a2_1,
                                                  int a3_0, int a3_1, float w_scale, f2 a_scale, f2 z) {
    const f2 big = f2_splat(12582912.0f);
    const f2 x1 = f2_sub(f2_pack(__int_as_float(0x4B400000 + a1_0), __int_as_float(0x4B400000 + a1_1)), big);
    const f2 x2 = f2_sub(f2_pack(__int_as_float(0x4B400000 + a2_0), __int_as_float(0x4B400000 + a2_1)), big);
    const f2 x3 = f2_sub(f2_pack(__int_as_float(0x4B400000 + a3_0), __int_as_float(0x4B400000 + a3_1)), big);
    f2 v = f2_fma(x2, f2_splat(0.0078125f), x1);
    v = f2_fma(x3, f2_splat(6.103515625e-05f), v);
    const f2 acc = f2_add(f2_pack(acc0, acc1), f2_mulz(v, f2_mul(f2_splat(w_scale), a_scale), z));
    f2_unpack(acc, acc0, acc1);
}

// Accumulation order of a Q8 projection row (every path): the G groups are cut into
// S = max(1, G / 3) consecutive splits (split s = groups [G s / S, G (s+1) / S)); each split's
// groups are accumulated in order from 0 (group_accumulate), and the split sums are added in split
// order.  S depends only on the matrix shape, so every kernel and batch size gives the same bits,
// and a tensor-core launch may run the splits in parallel CTAs.
__host__ __device__ __forceinline__ int q8_splits(int G) { return G >= 6 ? G / 3 : 1; }

// One step of the sequential group accumulation of a row: acc + v * (w_scale * 2^e).
__device__ __forceinline__ float group_accumulate(float acc, float v, float w_scale, float a_scale) {
    return __fadd_rn(acc, __fmul_rn(v, __fmul_rn(w_scale, a_scale)));
}

// ---- Tiled int8 layouts shared by the Q8 producers and consumers ---------------------------
//
// Rows of 64 bytes (one quantisation group) are stored in the tensor cores' 64-byte swizzle:
// 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3).  Both int8 operands are laid out in
// HBM exactly as a pipeline stage needs them in shared memory, so every stage is one contiguous
// bulk copy (no per-row TMA requests):
//   Q8 weights     [group][rows rounded up to 128][64 B]
//   digit planes   [group][16-stream block][plane][16][64 B]  (streams rounded up to 64)
// In the digit layout the three planes of any run of 16-stream blocks are contiguous, so one
// copy brings a tile's B operand and one MMA multiplies all three planes (N = 3 x streams).
__host__ __device__ __forceinline__ uint32_t swz64(uint32_t row, uint32_t byte) {
    return (((byte >> 4) ^ ((row >> 1) & 3u)) << 4) | (byte & 15u);
}

__host__ __device__ __forceinline__ size_t wq_off(int rows_pad, int r, int k) {
    return ((size_t)(k >> 6) * rows_pad + r) * 64 + swz64((uint32_t)r, (uint32_t)(k & 63));
}

__host__ __device__ __forceinline__ size_t dq_off(int cap_pad, int p, int b, int k) {
    return ((((size_t)(k >> 6) * (cap_pad >> 4) + (b >> 4)) * 3 + p) * 16 + (b & 15)) * 64 +
           swz64((uint32_t)b, (uint32_t)(k & 63));
}

__host__ __device__ __forceinline__ int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Per-stream group exponents 2^e of the digit planes: [stream][kEStride], whatever the vector
// length, so writers of different vectors (the norm: d/64 groups, the scan: d_inner/64) never touch
// another stream's entries.  Every Q8 projection has at most 32 groups.
constexpr int kEStride = 32;

// Validated slot of a stream whose slot or token failed the device-side check: no slot at all,
// at least as large as every pool capacity, so every `slot < cap` test skips the stream.
constexpr uint32_t kRejected = 0xffffffffu;

// Programmatic dependent launch: wait for the preceding kernel of the stream (and its memory)
// before touching anything it wrote, then let the next kernel start its own prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ int pack4(int a, int b, int c, int d) {
    return (a & 0xff) | ((b & 0xff) << 8) | ((c & 0xff) << 16) | ((d & 0xff) << 24);
}

}  // namespace rk
