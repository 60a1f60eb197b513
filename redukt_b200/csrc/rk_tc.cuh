// Q8 projections on the 5th-generation tensor cores (tcgen05, kind::i8, sm_100a).
//
// y[r][b] = sum_g scale[r][g] * 2^e[b][g] * (A1 + A2 * 2^-7 + A3 * 2^-14),
//   A_i = sum_{c in group g} q[r][c] * digit_i[b][c]   (exact int32)
// The int8 weights are the A operand (M = 128 rows per tile, K-major, straight from HBM by TMA);
// the three int8 digit planes of the activations are B operands (N = streams, K-major).  Each
// pipeline stage carries one 64-column quantisation group: 8 KB of weights + 3 x N x 64 B of
// digits.  The MMA warp issues, per group, 2 K-steps x 3 planes of tcgen05.mma into three int32
// TMEM accumulators (double-buffered: group g+1 multiplies while the epilogue reads group g).
// The epilogue warps read the accumulators with tcgen05.ld (thread = row = TMEM lane) and run
// the same digit_value/group_accumulate sequence as the CUDA-core kernel, so both paths give the
// same bits.  No TMA multicast (this code runs on every GPU of a multi-GPU job).
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4) .. +31).
// Every wait is bounded: on timeout the CTA records an error word, stops issuing work, drains
// the copies it started and frees its TMEM before returning.
#pragma once
#include <cuda.h>

#include "rk_kernels.cuh"

namespace rk {
namespace tc {

constexpr int kBM = 128;      // rows per tile = TMEM lanes
constexpr int kBK = 64;       // bytes of K per stage = one quantisation group
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kAutoMinStreams = 4;   // below this the CUDA-core kernel is used
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any legitimate wait

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

template <int BN>
struct alignas(1024) Smem {
    int8_t a[kStages][kBM * kBK];         // 8 KB per stage, 1024-aligned (64B-swizzle atoms)
    int8_t b[kStages][3][BN * kBK];       // digit planes
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
    int abort;
    float ae[BN * 32];                    // 2^e of the tile's streams for up to 32 groups
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; returns false (and raises the CTA abort flag) when the limit is reached or
// another role of the CTA has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            return false;
        }
    }
}

// Bounded wait that ignores the abort flag (used to drain work already in flight).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity) && globaltimer_ns() - t0 < kWaitLimitNs) {
    }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 64-byte swizzle layout:
// rows of 64 bytes, 8-row atoms of 512 bytes stacked along M/N (stride byte offset 512).
__device__ __forceinline__ uint64_t sw64_desc(const void* p) {
    uint64_t addr = smem_u32(p);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;          // start address
    d |= (uint64_t)1 << 16;                // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(512 >> 4) << 32;       // stride byte offset
    d |= (uint64_t)1 << 46;                // descriptor version (sm_100)
    d |= (uint64_t)4 << 61;                // layout: 64-byte swizzle
    return d;
}

// Instruction descriptor: D = s32, A = B = s8, both K-major, N x 128.
template <int BN>
__device__ __forceinline__ uint32_t idesc_i8() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int BN>
__host__ __device__ constexpr uint32_t tmem_cols() {
    return (2 * 3 * BN) <= 128 ? 128u : ((2 * 3 * BN) <= 256 ? 256u : 512u);
}

// Dynamic shared memory for a launch: enough for the tile, and enough that no more CTAs become
// resident on one SM than its 512 TMEM columns can serve at once.
template <int BN>
constexpr size_t launch_smem() {
    constexpr size_t need = sizeof(Smem<BN>) + 1024;
    constexpr size_t per_sm = 512 / tmem_cols<BN>();
    constexpr size_t floor_bytes = (size_t)233472 / (per_sm + 1) + 1024;
    return need > floor_bytes ? need : floor_bytes;
}

// One (128-row, BN-stream) output tile over all K groups of one Q8 projection.
template <int BN, class Epi>
__global__ void __launch_bounds__(kThreads, 1)
k_proj_q8_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_act, int M, int K,
             int cap, int n, const float* __restrict__ w_scale, const float* __restrict__ act_e, uint32_t* err,
             Epi epi) {
    extern __shared__ uint8_t smem_raw[];
    Smem<BN>& S = *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int G = K / kBK;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kBM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr uint32_t kCols = tmem_cols<BN>();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&S.tfull[i], 1);
            mbar_init(&S.tempty[i], 128);
        }
        S.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    for (int i = threadIdx.x; i < BN * G; i += blockDim.x) {
        int b = i / G, g = i - b * G;
        S.ae[b * 32 + g] = (n0 + b < n) ? act_e[(size_t)(n0 + b) * G + g] : 0.0f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort = &S.abort;

    if (warp == 0) {
        if (lane == 0) {
            constexpr uint32_t kStageBytes = kBM * kBK + 3 * BN * kBK;
            int issued = 0;
            for (int g = 0; g < G; g++) {
                int s = g % kStages;
                uint32_t ph = (g / kStages) & 1;
                if (!mbar_wait(&S.empty[s], ph ^ 1, abort)) break;
                mbar_expect_tx(&S.full[s], kStageBytes);
                tma_load_2d(S.a[s], &tm_w, g * kBK, m0, &S.full[s]);
#pragma unroll
                for (int p = 0; p < 3; p++) tma_load_2d(S.b[s][p], &tm_act, g * kBK, p * cap + n0, &S.full[s]);
                issued = g + 1;
            }
            if (*abort) {  // drain the copies this CTA started before its shared memory goes away
                for (int g = (issued > kStages ? issued - kStages : 0); g < issued; g++)
                    mbar_drain(&S.full[g % kStages], (g / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<BN>();
            int last = -1;
            for (int g = 0; g < G; g++) {
                int s = g % kStages;
                uint32_t ph = (g / kStages) & 1;
                int buf = g & 1;
                uint32_t bph = (g >> 1) & 1;
                if (!mbar_wait(&S.full[s], ph, abort)) break;
                if (!mbar_wait(&S.tempty[buf], bph ^ 1, abort)) break;
                tc_fence_after();
                uint32_t dbase = tmem + (uint32_t)(buf * 3 * BN);
#pragma unroll
                for (int p = 0; p < 3; p++) {
#pragma unroll
                    for (int ks = 0; ks < 2; ks++) {
                        uint64_t ad = sw64_desc(S.a[s] + ks * 32);
                        uint64_t bd = sw64_desc(S.b[s][p] + ks * 32);
                        mma_i8(dbase + (uint32_t)(p * BN), ad, bd, idesc, (uint32_t)ks);
                    }
                }
                mma_commit(&S.empty[s]);
                mma_commit(&S.tfull[buf]);
                last = g;
            }
            // the accumulators must be written before TMEM is released, also on abort
            if (last >= 0) mbar_drain(&S.tfull[last & 1], (last >> 1) & 1);
        }
        __syncwarp();
    } else {
        // epilogue: thread owns one output row (TMEM lane) and BN running sums
        const int quad = warp & 3;
        const int row = m0 + quad * 32 + lane;
        const bool row_ok = row < M;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        float acc[BN];
#pragma unroll
        for (int b = 0; b < BN; b++) acc[b] = 0.0f;
        for (int g = 0; g < G; g++) {
            int buf = g & 1;
            uint32_t bph = (g >> 1) & 1;
            // warp-uniform decision: tcgen05.ld below needs the whole warp converged
            bool ok = __all_sync(0xffffffffu, mbar_wait(&S.tfull[buf], bph, abort));
            if (!ok) break;
            tc_fence_after();
            float wsg = row_ok ? __ldg(w_scale + (size_t)row * G + g) : 0.0f;
            uint32_t base = tmem + lane_off + (uint32_t)(buf * 3 * BN);
#pragma unroll
            for (int c = 0; c < BN / 16; c++) {
                int a1[16], a2[16], a3[16];
                tmem_ld16(base + (uint32_t)(c * 16), a1);
                tmem_ld16(base + (uint32_t)(BN + c * 16), a2);
                tmem_ld16(base + (uint32_t)(2 * BN + c * 16), a3);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    int b = c * 16 + j;
                    acc[b] = group_accumulate(acc[b], digit_value(a1[j], a2[j], a3[j]), wsg, S.ae[b * 32 + g]);
                }
            }
            tc_fence_before();
            mbar_arrive(&S.tempty[buf]);
        }
        if (!*abort && row_ok) {
#pragma unroll
            for (int b = 0; b < BN; b++)
                if (n0 + b < n) epi(row, n0 + b, acc[b]);
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

}  // namespace tc
}  // namespace rk
