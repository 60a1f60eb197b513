// Q8 projections on the 5th-generation tensor cores (tcgen05, kind::i8, sm_100a).
//
// y[r][b] = sum_g scale[r][g] * 2^e[b][g] * (A1 + A2 * 2^-7 + A3 * 2^-14),
//   A_i = sum_{c in group g} q[r][c] * digit_i[b][c]   (exact int32)
// The int8 weights are the A operand (M = 128 rows per tile, K-major); the three int8 digit
// planes of the activations are B operands (N = streams, K-major).  Each pipeline stage carries
// one 64-column quantisation group: 8 KB of weights + 3 x N x 64 B of digits, brought in by
// bulk copies (cp.async.bulk) from operands that are stored pre-tiled and pre-swizzled in HBM.  The MMA warp issues, per group, 2 K-steps x 3 planes of tcgen05.mma into three int32
// TMEM accumulators (double-buffered: group g+1 multiplies while the epilogue reads group g).
// The epilogue warps read the accumulators with tcgen05.ld (thread = row = TMEM lane) and run
// the same digit_value/group_accumulate sequence as the CUDA-core kernel, so both paths give the
// same bits.  Every operand copy is a plain bulk copy into this CTA's own shared memory, so the
// kernel runs unchanged on every GPU of a multi-GPU job.
//
// Warp roles: warp 0 = copy producer, warp 1 = TMEM owner + MMA issuer, then one or two
// epilogue warpgroups (warp w reads TMEM lanes 32*(w%4) .. +31; with two warpgroups each owns
// half of the tile's streams).
// Every wait is bounded: on timeout the CTA records an error word, stops issuing work, drains
// the copies it started and frees its TMEM before returning.
#pragma once
#include "rk_kernels.cuh"

namespace rk {
namespace tc {

constexpr int kBM = 128;      // rows per tile = TMEM lanes
constexpr int kBK = 64;       // bytes of K per stage = one quantisation group
template <int BN>
constexpr int stages_for() { return BN == 16 ? 12 : 8; }  // deep enough to cover a ~2 us copy round trip

constexpr int kAutoMinStreams = 1;   // the tensor-core kernel serves every batch size (CUDA cores when forced)
// Wait bound in SM clock cycles (about 2 s at the B200's 1.9 GHz boost clock, longer when the
// clock is lower): far beyond any legitimate wait.  clock64 is a cheap per-SM counter.
constexpr long long kWaitLimitCycles = 4000000000ll;

// Test settings of the bounded waits (option "wait_limit_us" / "wait_test"; device globals of the
// library, read only on a wait's slow path):
//   g_wait_cycles  limit of every tensor-core mbarrier wait, in SM cycles
//   g_wait_ns      limit of every fused-step wait (grid barrier, bulk copies), in ns
//   g_wait_test    one-shot: 1 = CTA 0 of the next fused step skips its first grid-barrier arrival,
//                  2 = CTA 0 of the next tensor-core projection never issues its first activation
//                  copy.  Either makes one bounded wait run out (nothing faults or hangs: every wait
//                  gives up at its limit); the CTA that acts on it clears it.
__device__ long long g_wait_cycles = kWaitLimitCycles;
__device__ unsigned long long g_wait_ns = 200ull * 1000 * 1000;
__device__ int g_wait_test = 0;

__device__ __forceinline__ long long wait_limit_cycles() { return *(volatile long long*)&g_wait_cycles; }

// True once for the CTA that takes a pending one-shot wait test of kind `kind`.
__device__ __forceinline__ bool take_wait_test(int kind) {
    if (*(volatile int*)&g_wait_test != kind) return false;
    return atomicCAS(&g_wait_test, kind, 0) == kind;
}

template <int BN, int ST = stages_for<BN>(), int MB = 1>
struct TileCfg {
    static constexpr int kBufs = BN == 16 ? 4 : 2;          // TMEM accumulator sets in flight
    static constexpr int kColsUsed = kBufs * 3 * BN;
    static constexpr uint32_t kCols = kColsUsed <= 128 ? 128u : (kColsUsed <= 256 ? 256u : 512u);
    static constexpr int kEG = 2;                            // epilogue warpgroups (each owns BN/2 streams)
    static constexpr int kSPT = BN / kEG;                    // streams per epilogue thread
    static constexpr int kThreads = 64 + 128 * kEG;          // producer + MMA warp + epilogue
    static constexpr int kMinBlocks = MB;                    // CTAs per SM the registers must allow
};

template <int BN, int ST = stages_for<BN>()>
struct alignas(1024) Smem {
    static constexpr int kStages = ST;
    int8_t a[kStages][kBM * kBK];         // 8 KB per stage, 1024-aligned (64B-swizzle atoms)
    int8_t b[kStages][3 * BN * kBK];      // digit planes: [16-stream block][plane][16 rows][64 B]
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint32_t slot[BN];                    // stream metadata of the tile (in_proj epilogue)
    uint32_t fresh[BN];
    uint64_t tfull[TileCfg<BN, ST>::kBufs];
    uint64_t tempty[TileCfg<BN, ST>::kBufs];
    uint64_t gather;                      // split-K: the last CTA's copy of the tile's partial sums
    int last;                             // split-K: this CTA combines the tile
    uint32_t tmem_base;
    int abort;
    alignas(16) float ae[32 * BN];        // 2^e of the tile's streams for up to 32 groups, [group][stream]
    float ws[32 * kBM];                   // weight scales of the tile's rows, [group][row]
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
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > wait_limit_cycles()) {
                *abort = 1;
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag (used to drain work already in flight).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    const long long lim = wait_limit_cycles();
    while (!mbar_try_wait(bar, parity) && clock64() - t0 < lim) {
    }
}

// One contiguous bulk copy global -> shared (16-byte aligned, size a multiple of 16), completing
// on `bar` with complete_tx.  The operands are stored pre-tiled in HBM (rk_math.cuh), so a whole
// pipeline stage is one request instead of one request per 64-byte row.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
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
template <int N>
__device__ __forceinline__ uint32_t idesc_i8() {
    static_assert(N % 16 == 0 && N >= 16 && N <= 256, "M=128 needs N in 16..256, multiple of 16");
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
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

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

// kSPT (8 or 16) consecutive accumulator columns of this thread's TMEM lane
template <int N>
__device__ __forceinline__ void tmem_ld_n(uint32_t taddr, int (&r)[N]) {
    if constexpr (N == 16) tmem_ld16(taddr, r);
    else tmem_ld8(taddr, r);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <int BN>
__host__ __device__ constexpr uint32_t tmem_cols() {
    return TileCfg<BN>::kCols;  // the same for every stage count
}

// Dynamic shared memory for a launch: enough for the tile, and enough that no more CTAs become
// resident on one SM than its 512 TMEM columns can serve at once (at most 227 KB).
template <int BN, int ST = stages_for<BN>()>
constexpr size_t launch_smem() {
    constexpr size_t need = sizeof(Smem<BN, ST>) + 1024;
    constexpr size_t per_sm = 512 / tmem_cols<BN>();
    constexpr size_t floor_bytes = (size_t)233472 / (per_sm + 1) + 1024;
    constexpr size_t want = need > floor_bytes ? need : floor_bytes;
    static_assert(need <= 232448, "tile does not fit in shared memory");
    return want > 232448 ? 232448 : want;
}

constexpr int kMaxGatherSplits = 8;  // split launches gather at most this many split blocks

// Split-K launch: with splits == Z (a divisor of S), CTA z of a tile runs splits [S z / Z, S (z+1) / Z)
// and stores each one's 128 x BN sums to `part`; the tile's last CTA to finish (an atomic counter per
// tile) copies the tile's S blocks into shared memory and adds them in split order.  With splits == 1
// one CTA runs all splits.
struct SplitK {
    int splits;          // CTAs per tile: 1 or a divisor of q8_splits(G)
    float* part;         // [tiles][S][128][BN] split sums
    uint32_t* counter;   // [tiles], zero between launches (the last CTA of a tile resets its entry)
};

// One (128-row, BN-stream) output tile over all K groups (or one split) of one Q8 projection.
template <int BN, class Epi, int ST = stages_for<BN>(), int MB = 1>
__global__ void __launch_bounds__(TileCfg<BN, ST, MB>::kThreads, TileCfg<BN, ST, MB>::kMinBlocks)
k_proj_q8_tc(const int8_t* __restrict__ wq, const int8_t* __restrict__ dq, int M, int K, int cap_pad, int n,
             const float* __restrict__ w_scale, const float* __restrict__ act_e, uint32_t* err, Epi epi, SplitK sk) {
    extern __shared__ uint8_t smem_raw[];
    Smem<BN, ST>& S = *reinterpret_cast<Smem<BN, ST>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int kBufs = TileCfg<BN, ST, MB>::kBufs;
    constexpr int kEG = TileCfg<BN, ST, MB>::kEG;
    constexpr int kSPT = TileCfg<BN, ST, MB>::kSPT;
    constexpr int kThreads = TileCfg<BN, ST, MB>::kThreads;
    constexpr int kStages = Smem<BN, ST>::kStages;
    constexpr uint32_t kCols = TileCfg<BN, ST, MB>::kCols;
    constexpr uint32_t kStageBytes = kBM * kBK + 3 * BN * kBK;
    const int G = K / kBK;                          // groups of a row
    const int NS = q8_splits(G);                     // splits of the accumulation order
    const bool split = BN == 16 && sk.splits > 1;    // this launch: splits.. CTAs per tile (narrow tiles only)
    const int nz = split ? sk.splits : 1;            // CTAs per tile; divides NS
    const int zs = split ? (int)blockIdx.z : 0;
    const int s0 = (NS * zs) / nz, s1 = (NS * (zs + 1)) / nz;  // this CTA's splits [s0, s1)
    const int gb = (G * s0) / NS;                    // and groups [gb, gb + GL)
    const int GL = (G * s1) / NS - gb;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * kBM;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npre = GL < kStages ? GL : kStages;
    const int m_pad = round_up(M, kBM);
    const int8_t* wtile = wq + ((size_t)gb * m_pad + m0) * 64;  // row m0 of group gb in the tiled layout

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int i = 0; i < kBufs; i++) {
            mbar_init(&S.tfull[i], 1);
            mbar_init(&S.tempty[i], 128 * kEG);
        }
        mbar_init(&S.gather, 1);
        S.abort = 0;
        S.last = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // weights are never written by the step: stream the first stages before the preceding
        // kernel has finished
        for (int g = 0; g < npre; g++) {
            mbar_expect_tx(&S.full[g], kStageBytes);
            bulk_load(S.a[g], wtile + (size_t)g * m_pad * 64, kBM * kBK, &S.full[g]);
        }
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // Only barrier initialisation and the TMEM allocation gate the producer and MMA warps; the
    // epilogue warps stage their scales and stream metadata below while the first stages land.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort = &S.abort;

    if (warp == 0) {
        if (lane == 0) {
            pdl_wait();  // the activation digits come from the preceding kernel
            pdl_trigger();
            int issued = 0;
            // wait test: stage 0 never receives its activation bytes, so its full barrier never
            // completes and the MMA warp's bounded wait runs out
            const bool skip0 = blockIdx.x == 0 && blockIdx.y == 0 && take_wait_test(2);
            for (int g = 0; g < GL; g++) {
                int s = g % kStages;
                uint32_t ph = (g / kStages) & 1;
                if (g >= npre) {
                    if (!mbar_wait(&S.empty[s], ph ^ 1, abort)) break;
                    mbar_expect_tx(&S.full[s], kStageBytes);
                    bulk_load(S.a[s], wtile + (size_t)g * m_pad * 64, kBM * kBK, &S.full[s]);
                }
                if (!(skip0 && g == 0))
                    bulk_load(S.b[s], dq + ((size_t)(gb + g) * (cap_pad >> 4) + (n0 >> 4)) * 3 * 16 * 64,
                              3 * BN * kBK, &S.full[s]);
                issued = g + 1;
            }
            if (*abort) {  // drain the copies this CTA started before its shared memory goes away
                int from = issued > kStages ? issued - kStages : 0;
                int to = issued > npre ? issued : npre;  // the prefetched weight stages count too
                for (int g = from; g < to; g++) mbar_drain(&S.full[g % kStages], (g / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8<3 * BN>();
            int last = -1;
            for (int g = 0; g < GL; g++) {
                int s = g % kStages;
                uint32_t ph = (g / kStages) & 1;
                int buf = g % kBufs;
                uint32_t bph = (g / kBufs) & 1;
                if (!mbar_wait(&S.full[s], ph, abort)) break;
                if (!mbar_wait(&S.tempty[buf], bph ^ 1, abort)) break;
                tc_fence_after();
                // one MMA per K-step: the three digit planes are stacked along N, so accumulator
                // column (16-stream block u, plane p, stream j) = 48u + 16p + j
                uint32_t dbase = tmem + (uint32_t)(buf * 3 * BN);
#pragma unroll
                for (int ks = 0; ks < 2; ks++)
                    mma_i8(dbase, sw64_desc(S.a[s] + ks * 32), sw64_desc(S.b[s] + ks * 32), idesc, (uint32_t)ks);
                mma_commit(&S.empty[s]);
                mma_commit(&S.tfull[buf]);
                last = g;
            }
            // the accumulators must be written before TMEM is released, also on abort
            if (last >= 0) mbar_drain(&S.tfull[last % kBufs], (last / kBufs) & 1);
        }
        __syncwarp();
    } else {
        // epilogue: thread owns one output row (TMEM lane) and kSPT running sums
        const int e = warp - 2;
        const int quad = warp & 3;
        const int half = e >> 2;                  // which kSPT streams of the tile
        const int u0 = (half * kSPT) / 16;        // first 16-stream block
        const int j0 = (half * kSPT) % 16;        // first stream inside it (kSPT = 8)
        const int rl = quad * 32 + lane;
        const int row = m0 + rl;
        const bool row_ok = row < M;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        {
            // stage the tile's weight scales (never written by the step: before the dependency
            // wait), then the activation scales and stream metadata, each as one batch of loads
            const int et = threadIdx.x - 64;  // 0 .. 128 * kEG - 1
            constexpr int kET = 128 * kEG;
            constexpr int kWsPer = (kBM * 32 + kET - 1) / kET;
            float tw[kWsPer];
            const int wcnt = kBM * G, wok = (M - m0) * G;
#pragma unroll
            for (int k = 0; k < kWsPer; k++) {
                int i = et + k * kET;
                tw[k] = (i < wcnt && i < wok) ? __ldg(w_scale + (size_t)m0 * G + i) : 0.0f;
            }
            pdl_wait();
            pdl_trigger();
            constexpr int kAePer = (BN * 32 + kET - 1) / kET;
            float ta[kAePer];
            const int acnt = BN * G;
#pragma unroll
            for (int k = 0; k < kAePer; k++) {
                int i = et + k * kET;
                ta[k] = (i < acnt && n0 + i / G < n) ? act_e[(size_t)(n0 + i / G) * kEStride + i % G] : 0.0f;
            }
            epi.stage(n0, min(BN, n - n0), S.slot, S.fresh, et, kET);
#pragma unroll
            for (int k = 0; k < kWsPer; k++) {
                int i = et + k * kET;
                if (i < wcnt) {
                    int r = i / G, g = i - r * G;
                    S.ws[g * kBM + r] = tw[k];
                }
            }
#pragma unroll
            for (int k = 0; k < kAePer; k++) {
                int i = et + k * kET;
                if (i < acnt) {
                    int b = i / G, g = i - b * G;
                    S.ae[g * BN + b] = ta[k];
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kET) : "memory");  // epilogue warps only
        }
        const f2 z2 = f2_zero();     // group_accumulate2's hidden -0.0
        float acc[kSPT], tot[kSPT];  // running sum of the current split; sum of the finished splits
#pragma unroll
        for (int b = 0; b < kSPT; b++) acc[b] = tot[b] = 0.0f;
        // after group g: close the split if g is its last group (whole-row CTA: add it to tot;
        // split launch: this CTA's only split, kept in acc for the store below)
        int sp = s0, send = (G * (s0 + 1)) / NS;  // current split and its end group
        const uint32_t tile = blockIdx.y * gridDim.x + blockIdx.x;
        float* blk = sk.part + (size_t)tile * NS * (kBM * BN);  // split launch: the tile's split sums
        auto split_end = [&](int g) {
            if (g + 1 != send) return;
            if (split) {  // publish the split's sums for the tile's last CTA
                float4* mine = reinterpret_cast<float4*>(blk + ((size_t)sp * kBM + rl) * BN + half * kSPT);
#pragma unroll
                for (int q = 0; q < kSPT / 4; q++)
                    mine[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
            } else {
#pragma unroll
                for (int b = 0; b < kSPT; b++) tot[b] = sp == 0 ? acc[b] : __fadd_rn(tot[b], acc[b]);
            }
#pragma unroll
            for (int b = 0; b < kSPT; b++) acc[b] = 0.0f;
            sp++;
            send = (G * (sp + 1)) / NS;
        };
        // TMEM column of (stream block u, digit plane p, stream j of the block) = 48u + 16p + j
        if constexpr (kSPT > 16 || (MB > 1 && kSPT >= 16)) {
            // one group at a time (a double buffer would not fit in registers)
            for (int gl = 0; gl < GL; gl++) {
                const int g = gb + gl;
                const int buf = gl % kBufs;
                bool ok = __all_sync(0xffffffffu, mbar_wait(&S.tfull[buf], (gl / kBufs) & 1, abort));
                if (!ok) break;
                tc_fence_after();
                const float wsg = S.ws[g * kBM + rl];
                const uint32_t base = tmem + lane_off + (uint32_t)(buf * 3 * BN);
#pragma unroll
                for (int c = 0; c < kSPT / 16; c++) {
                    int a1[16], a2[16], a3[16];
                    tmem_ld16(base + (uint32_t)((u0 + c) * 48), a1);
                    tmem_ld16(base + (uint32_t)((u0 + c) * 48 + 16), a2);
                    tmem_ld16(base + (uint32_t)((u0 + c) * 48 + 32), a3);
                    tmem_wait_ld();
                    const f2* ae2 = reinterpret_cast<const f2*>(&S.ae[g * BN + half * kSPT + c * 16]);
#pragma unroll
                    for (int q = 0; q < 16; q += 2) {
                        const int b = c * 16 + q;
                        group_accumulate2(acc[b], acc[b + 1], a1[q], a1[q + 1], a2[q], a2[q + 1], a3[q], a3[q + 1], wsg,
                                          ae2[q >> 1], z2);
                    }
                }
                tc_fence_before();
                mbar_arrive(&S.tempty[buf]);
                split_end(g);
            }
        } else {
            // software pipeline: group g+1 is read from TMEM while group g is combined
            // (tcgen05.ld is asynchronous until tcgen05.wait::ld)
            int cur[3][kSPT], nxt[3][kSPT];
            const uint32_t ucol = (uint32_t)(u0 * 48 + j0);
            bool have = __all_sync(0xffffffffu, mbar_wait(&S.tfull[0], 0, abort));
            if (have) {
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < 3; p++) tmem_ld_n<kSPT>(tmem + lane_off + ucol + (uint32_t)(p * 16), cur[p]);
                tmem_wait_ld();
            }
            for (int gl = 0; have && gl < GL; gl++) {
                const int g = gb + gl;
                const int buf = gl % kBufs;
                bool more = false;
                if (gl + 1 < GL) {
                    const int nb = (gl + 1) % kBufs;
                    more = __all_sync(0xffffffffu, mbar_wait(&S.tfull[nb], ((gl + 1) / kBufs) & 1, abort));
                    if (more) {
                        tc_fence_after();
                        const uint32_t base = tmem + lane_off + (uint32_t)(nb * 3 * BN) + ucol;
#pragma unroll
                        for (int p = 0; p < 3; p++) tmem_ld_n<kSPT>(base + (uint32_t)(p * 16), nxt[p]);
                    }
                }
                const float wsg = S.ws[g * kBM + rl];
                const f2* ae2 = reinterpret_cast<const f2*>(&S.ae[g * BN + half * kSPT]);
#pragma unroll
                for (int b = 0; b < kSPT; b += 2)
                    group_accumulate2(acc[b], acc[b + 1], cur[0][b], cur[0][b + 1], cur[1][b], cur[1][b + 1], cur[2][b],
                                      cur[2][b + 1], wsg, ae2[b >> 1], z2);
                tc_fence_before();
                mbar_arrive(&S.tempty[buf]);
                split_end(g);
                if (gl + 1 < GL) {
                    if (!more) {
                        have = false;
                        break;
                    }
                    tmem_wait_ld();
#pragma unroll
                    for (int p = 0; p < 3; p++)
#pragma unroll
                        for (int b = 0; b < kSPT; b++) cur[p][b] = nxt[p][b];
                }
            }
        }
        bool emit = true;
        if constexpr (BN == 16) {
            static_assert(sizeof(Smem<BN, ST>::a) + sizeof(Smem<BN, ST>::b) >= (size_t)kMaxGatherSplits * kBM * BN * sizeof(float),
                          "the stage buffers hold the gathered sums of kMaxGatherSplits splits");
            if (split) {
                // this CTA's split sums are published (split_end); the tile's last CTA adds all
                // splits in order
                constexpr int kET = 128 * kEG;
                __threadfence();
                asm volatile("bar.sync 1, %0;" ::"r"(kET) : "memory");
                if (threadIdx.x == 64 && !*abort) {
                    const uint32_t old = atomicAdd(&sk.counter[tile], 1u);
                    if (old == (uint32_t)nz - 1) {
                        sk.counter[tile] = 0u;  // ready for the next launch
                        __threadfence();
                        // other CTAs' generic-proxy writes, read below by the bulk-copy (async) proxy
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        const uint32_t bytes = (uint32_t)(NS * kBM * BN * sizeof(float));
                        mbar_expect_tx(&S.gather, bytes);
                        bulk_load(&S.a[0][0], blk, bytes, &S.gather);
                        S.last = 1;
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"r"(kET) : "memory");
                emit = S.last != 0;
                if (emit) {
                    emit = __all_sync(0xffffffffu, mbar_wait(&S.gather, 0, abort));
                    const float* P = reinterpret_cast<const float*>(&S.a[0][0]);
#pragma unroll
                    for (int b = 0; b < kSPT; b++) acc[b] = P[rl * BN + half * kSPT + b];
                    for (int sp = 1; sp < NS; sp++)
#pragma unroll
                        for (int b = 0; b < kSPT; b++)
                            acc[b] = __fadd_rn(acc[b], P[((size_t)sp * kBM + rl) * BN + half * kSPT + b]);
                }
            } else {
#pragma unroll
                for (int b = 0; b < kSPT; b++) acc[b] = tot[b];
            }
        } else {
#pragma unroll
            for (int b = 0; b < kSPT; b++) acc[b] = tot[b];
        }
        if (emit && !*abort && row_ok) {
            constexpr int kCH = kSPT < 16 ? kSPT : 16;  // streams per epilogue call
#pragma unroll
            for (int c = 0; c < kSPT / kCH; c++) {
                float v[kCH];
#pragma unroll
                for (int i = 0; i < kCH; i++) v[i] = acc[c * kCH + i];
                const int tb = half * kSPT + c * kCH;  // tile-relative first stream
                const int b0 = n0 + tb;
                if (b0 < n) epi.template apply<kCH>(row, b0, min(kCH, n - b0), v, TileMeta{S.slot, S.fresh}, tb);
            }
        }
        if constexpr (TileSoftmax<Epi>::value) {
            // The tile's softmax partials: for each of this warpgroup's kSPT streams, the max over
            // the tile's 128 rows and the sum of exp(l - max) over them (the reference's Cephes exp),
            // each reduced in a fixed order (warp butterfly, then the 4 warps in order), so the
            // result depends only on the stream's own logits.  Rows past M count as -inf / 0.  The
            // head never runs split (every CTA emits its whole tile).
            __shared__ float s_part[kEG][4][kSPT];
            const int bar_id = 2 + half;
            const bool valid = emit && !*abort && row_ok;
            float mx[kSPT];
#pragma unroll
            for (int b = 0; b < kSPT; b++) mx[b] = warp_allmax(valid ? acc[b] : -INFINITY);
            if (lane == 0)
#pragma unroll
                for (int b = 0; b < kSPT; b++) s_part[half][quad][b] = mx[b];
            asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
#pragma unroll
            for (int b = 0; b < kSPT; b++)
                mx[b] = fmaxf(fmaxf(s_part[half][0][b], s_part[half][1][b]), fmaxf(s_part[half][2][b], s_part[half][3][b]));
            asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
#pragma unroll
            for (int b = 0; b < kSPT; b++) {
                const float e = (valid && mx[b] != -INFINITY) ? portable_expf(__fsub_rn(acc[b], mx[b])) : 0.0f;
                const float w = warp_allsum(e);
                if (lane == 0) s_part[half][quad][b] = w;
            }
            asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
            if (quad == 0 && lane < kSPT) {
                const int b = n0 + half * kSPT + lane;
                if (b < n && !*abort) {
                    const float tot = __fadd_rn(__fadd_rn(__fadd_rn(s_part[half][0][lane], s_part[half][1][lane]),
                                                          s_part[half][2][lane]),
                                                s_part[half][3][lane]);
                    float* r = epi.red + ((size_t)b * epi.parts + blockIdx.y) * 2;
                    r[0] = mx[lane];
                    r[1] = tot;
                }
            }
        }
    }
    if (threadIdx.x == 64 && S.last) mbar_drain(&S.gather, 0);  // a gather copy never outlives the CTA
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
