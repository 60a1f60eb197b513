// Fused small-batch decode step: every layer of one Mamba Q8 step in ONE persistent kernel.
//
// At a handful of streams each per-layer kernel of the step is latency-bound (a few MB of weights,
// a dependency on the previous kernel's complete output), so a step of 24 layers x 5 launches
// pays launch and drain latencies many times over.  This kernel keeps one resident CTA per SM (a
// cooperative launch) and walks the layers in three phases separated by grid-wide barriers:
//
//   A  norm + in_proj + causal conv/SiLU + x_proj group chains
//      job = (half of in_proj, 64 or 128 rows, 8 or 16 streams).  The CTA normalises its
//      streams itself (their digit planes never leave shared memory), multiplies them with
//      warp-level int8 MMAs, finishes each (row, stream) with the split-order combine and the
//      in_proj epilogue, and for x-half blocks evaluates the x_proj chains of that channel group.
//   B  x_proj group sums + dt_proj + selective scan + z gate + out_proj digit planes
//      job = (64-channel group, 4 or 8 streams), one thread per (channel, stream).
//   C  out_proj + residual
//      job = (16- or 32-row block, 8 streams), one accumulation split per warp.
//
// Everything a phase reads that the phase before it does not write (weights and scales, the
// conv and SSM state of earlier steps, the residual rows a job updates) is fetched into shared
// memory by a few bulk copies (cp.async.bulk, one mbarrier) and 16-byte copies issued between the
// CTA's arrival at the barrier before the phase and its wait there, so the copies overlap the
// barrier.  Weight tiles and the per-group operands are stored job-blocked in HBM (FusedLayer), so
// each is one contiguous copy.
// After the barrier a job only reads its predecessor's outputs (from L2).  After the last layer
// the final norm writes the head's digit planes; the host launches the head projection.
//
// Every value is produced by the same arithmetic, in the same order, as the per-kernel path
// (norm_apply and digit planes, the q8_splits combine, conv_silu_taps, xproj_chain, the
// one-thread scan pieces, the residual add), so a stream's bits do not depend on which path ran
// it.  The int8 products are exact int32 sums in any order; the warp-level MMA
// (mma.sync m16n8k32 s8) gives the same integers as the dp4a and tcgen05 paths.
//
// Every wait (grid barrier, bulk-copy completion) is bounded in time; one that runs out sets bit 4
// of the error word and every CTA leaves the step.
#pragma once
#include "rk_kernels.cuh"
#include "rk_tc.cuh"

namespace rk {

constexpr int kFusedMaxN = 32;           // streams handled by the fused step
constexpr int kFusedThreads = 256;
constexpr uint32_t kErrGridWait = 4u;    // error-word bit: a fused-step wait ran out

struct FusedLayer {
    const float* norm_w;
    const float* norm_b;
    const int8_t* in_q;    // tiled Q8 weights [G][mpad][64]
    const float* in_s;     // [rows][G]
    const int8_t* out_q;
    const float* out_s;
    const float* xw_blk;   // x_proj by channel group [di/64][xr][68] (4 zero floats per row)
    const float* ct_blk;   // conv taps 0..3 and bias by channel group [di/64][5][64]
    const float* sb_blk;   // dt_proj columns, A, dt bias, D by channel group [di/64][dr + 18][64]
    const int8_t* in_blk;  // in_proj by 64-row block [2 di/64][G][64][64] (tiled rows, swizzle kept)
    const int8_t* out_blk; // out_proj by 16-row block [d/16][G][16][64]
};

// Shared-memory map (byte offsets).  One prefetch region P holds the current phase's copied
// operands (A, B and C lay out their own parts in it); the work region holds the digit planes,
// exponents, split sums and staging of the running job.
struct FusedLayout {
    int a_w, a_ws, a_nw, a_xw, a_ct, a_conv;  // P, phase A
    int b_sb, b_ssm;                          // P, phase B
    int c_w, c_ws, c_x;                       // P, phase C
    int bq, ae, part, xc, zs;                 // work region
    int total;
};

struct FusedArgs {
    int n, cap, cap_pad, d, di, dr, xr, nl;
    int g_in, s_in, mpad_in;     // in_proj: groups, accumulation splits, padded rows
    int g_out, s_out, mpad_out;  // out_proj
    int sga, sgz, sgb, mc;       // streams per A job (x half, z half: 8 or 16), per B job, rows per C job
    int rz;                      // rows per z-half A job (64 or 128; x-half jobs are 64 rows)
    int pitch_a;                 // bytes per digit-plane row of phase A's planes (d + 16)
    FusedLayout lay;
    const uint32_t* slots;  // validated slots of the step (kRejected: a stream that touches no state)
    const uint32_t* rflag;
    float* x;          // [cap][d] residual stream
    float* conv;       // [L][cap][3][di]
    float* ssm;        // [L][cap][16][di]
    float* conv_out;   // [cap][di]
    float* z;          // [cap][di]
    float* xpart;      // [stream][di/64][xr] x_proj group chains
    int8_t* act_q;     // digit planes (scan output, then the final norm for the head)
    float* act_e;
    const FusedLayer* layers;
    const float* norm_f_w;
    const float* norm_f_b;
    uint32_t* bar;     // grid barrier arrivals (zeroed by k_embed of the same step)
    uint32_t* err;
};

__host__ __device__ __forceinline__ int align16(int x) { return (x + 15) & ~15; }

// Offsets for one shape and job split (host side, once per launch).
inline FusedLayout fused_layout(const FusedArgs& a) {
    // Bulk copies (async proxy) and 16-byte copies (generic proxy) land in disjoint regions, so no
    // byte is written by one proxy after the other and no proxy fence is needed between phases.
    FusedLayout L{};
    int o = 0;
    const int ra = a.rz > 64 ? a.rz : 64;
    L.a_w = o;    o += align16(ra * a.d);
    L.a_ws = o;   o += align16(ra * a.g_in * 4);
    L.a_nw = o;   o += align16(2 * a.d * 4);
    L.a_xw = o;   o += align16(a.xr * 68 * 4);
    L.a_ct = o;   o += align16(5 * 64 * 4);
    const int pa = o;
    o = 0;
    L.b_sb = o;  o += align16((a.dr + 18) * 64 * 4);
    const int pb = o;
    o = 0;
    L.c_w = o;  o += align16(a.mc * a.di);
    L.c_ws = o; o += align16(a.mc * a.g_out * 4);
    const int pc = o;
    const int big = align16(pa > pb ? (pa > pc ? pa : pc) : (pb > pc ? pb : pc));
    const int sg = a.sga > a.sgz ? a.sga : a.sgz;
    const int sa = align16(a.sga * 3 * 64 * 4), sb = align16(a.sgb * 16 * 64 * 4), sc = align16(8 * a.mc * 4);
    L.a_conv = L.b_ssm = L.c_x = big;
    o = big + (sa > sb ? (sa > sc ? sa : sc) : (sb > sc ? sb : sc));
    const int ta = sg / 8, tc = a.mc / 16;
    const int bq_a = 3 * sg * a.pitch_a, bq_c = a.g_out * 3 * 8 * 64;
    L.bq = o;   o += align16(bq_a > bq_c ? bq_a : bq_c);
    L.ae = o;   o += align16(sg * kEStride * 4);
    const int pa_n = (ta * 4 > a.rz / 16 ? ta * 4 : a.rz / 16) * a.s_in, pc_n = tc * a.s_out;
    L.part = o; o += align16((pa_n > pc_n ? pa_n : pc_n) * 128 * 4);
    L.xc = o;   o += align16(a.sga * 68 * 4);
    L.zs = o;   o += align16(a.sgb * a.xr * 4);
    L.total = o;
    return L;
}

// ---- primitives --------------------------------------------------------------------------

// D += A(16x32, s8, row) * B(32x8, s8, col), int32 accumulation.
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Grid-wide barrier of a cooperative launch, in two halves so a CTA can issue its next
// prefetch between them: grid_arrive = CTA barrier + one release arrival per CTA (ordering every
// write of the CTA before it); grid_wait = acquire spin until every CTA of this and all earlier
// barriers has arrived, then a CTA barrier.  `target` counts arrivals so far (the counter is not
// reset within a step).  grid_wait returns false when this wait, or one in another CTA, ran out
// of time.
__device__ __forceinline__ void grid_arrive(uint32_t* bar, uint32_t& target) {
    __syncthreads();
    target += gridDim.x;
    // wait test: CTA 0 withholds its first arrival, so this barrier never fills and every CTA's
    // bounded wait runs out
    if (threadIdx.x == 0 && !(blockIdx.x == 0 && target == gridDim.x && tc::take_wait_test(1)))
        red_release_gpu_add(bar, 1u);
}

__device__ __forceinline__ bool grid_wait(uint32_t* bar, uint32_t target, uint32_t* err, int* s_ok) {
    if (threadIdx.x == 0) {
        int ok = 1;
        const unsigned long long t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (ld_acquire_gpu(bar) < target) {
            if ((++spins & 31u) == 0) {
                if (ld_acquire_gpu(err) & kErrGridWait) {
                    ok = 0;
                    break;
                }
                if (globaltimer_ns() - t0 > *(volatile unsigned long long*)&tc::g_wait_ns) {
                    atomicOr(err, kErrGridWait);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// Completion of the bulk copies on `bar` (parity `par`): thread 0 waits with a time limit, the
// CTA learns the outcome.  Returns false when the wait ran out (error bit set).
__device__ __forceinline__ bool copies_wait(uint64_t* bar, uint32_t par, uint32_t* err, int* s_ok);

// One mbarrier's bulk-copy batches: at most one batch in flight.
struct CopyBatch {
    uint64_t* bar;
    uint32_t par;
    int pending;
    __device__ __forceinline__ void issued() { pending = 1; }
    __device__ __forceinline__ bool wait(uint32_t* err, int* s_ok) {
        cp_async_wait_all();  // this thread's small copies of the batch
        if (!copies_wait(bar, par, err, s_ok)) return false;
        par ^= 1u;
        pending = 0;
        return true;
    }
};

__device__ __forceinline__ bool copies_wait(uint64_t* bar, uint32_t par, uint32_t* err, int* s_ok) {
    if (threadIdx.x == 0) {
        int ok = 1;
        if (!tc::mbar_try_wait(bar, par)) {
            const unsigned long long t0 = globaltimer_ns();
            while (!tc::mbar_try_wait(bar, par)) {
                if (globaltimer_ns() - t0 > *(volatile unsigned long long*)&tc::g_wait_ns) {
                    atomicOr(err, kErrGridWait);
                    ok = 0;
                    break;
                }
            }
        }
        *s_ok = ok;
    }
    __syncthreads();
    return *s_ok != 0;
}

// ---- warp-level Q8 row tile ----------------------------------------------------------------
//
// One warp: 16 rows of a Q8 weight tile held in shared memory as [G][RT][64 B] (the global tiled
// layout of rows row0 .. row0+RT-1, row0 a multiple of 8 so the 64-byte swizzle phase of a row is
// that of its tile-local index) times 8 streams' digit planes, over groups [g0, g1) of ONE
// accumulation split.  `bword(p, g, c)` returns the thread's 4 bytes of logical 16-byte chunk c
// of group g, plane p, for stream gid at byte tig * 4.  Per group, two k-steps x three planes of
// m16n8k32 give the exact int32 digit sums of the 16 x 8 (row, stream) pairs; each thread folds
// its four pairs (rows gid, gid+8; streams 2*tig, 2*tig+1) into its split sums with digit_value /
// group_accumulate, in group order.  `ws` = the tile's scales [RT][G], `ae` = the streams'
// exponents [8][kEStride].
__device__ __forceinline__ void q8_group_frags(const int8_t* at, int RT, int ra, uint32_t sw, int g, int tig,
                                               uint32_t (&a0)[4], uint32_t (&a1)[4]) {
    const int8_t* wa = at + ((size_t)g * RT + ra) * 64 + tig * 4;
    const int8_t* wb = wa + 8 * 64;
    // k-step 0: chunks 0, 1; k-step 1: chunks 2, 3 (rows gid, gid+8)
    a0[0] = *reinterpret_cast<const uint32_t*>(wa + ((0u ^ sw) << 4));
    a0[1] = *reinterpret_cast<const uint32_t*>(wb + ((0u ^ sw) << 4));
    a0[2] = *reinterpret_cast<const uint32_t*>(wa + ((1u ^ sw) << 4));
    a0[3] = *reinterpret_cast<const uint32_t*>(wb + ((1u ^ sw) << 4));
    a1[0] = *reinterpret_cast<const uint32_t*>(wa + ((2u ^ sw) << 4));
    a1[1] = *reinterpret_cast<const uint32_t*>(wb + ((2u ^ sw) << 4));
    a1[2] = *reinterpret_cast<const uint32_t*>(wa + ((3u ^ sw) << 4));
    a1[3] = *reinterpret_cast<const uint32_t*>(wb + ((3u ^ sw) << 4));
}

template <class BWord>
__device__ __forceinline__ void q8_group_sums(const uint32_t (&a0)[4], const uint32_t (&a1)[4], BWord bword, int g,
                                              int (&dsum)[3][4]) {
#pragma unroll
    for (int p = 0; p < 3; p++) {
        dsum[p][0] = dsum[p][1] = dsum[p][2] = dsum[p][3] = 0;
        mma_s8_16832(dsum[p], a0, bword(p, g, 0), bword(p, g, 1));
        mma_s8_16832(dsum[p], a1, bword(p, g, 2), bword(p, g, 3));
    }
}

template <class BWord>
__device__ __forceinline__ void q8_tile16_split(const int8_t* at, int RT, int rl0, const float* ws, int G, int g0,
                                                int g1, BWord bword, const float* ae, int lane, float (&acc)[4]) {
    const int gid = lane >> 2, tig = lane & 3;
    const int ra = rl0 + gid;  // rows ra and ra + 8 share the swizzle phase
    const uint32_t sw = ((uint32_t)ra >> 1) & 3u;
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i] = 0.0f;
    const f2 z2 = f2_zero();
    auto fold = [&](const int (&ds)[3][4], int g) {  // (row, stream pair) on the packed pipe
        const float wsa = ws[ra * G + g], wsb = ws[(ra + 8) * G + g];
        const f2 ae2 = f2_pack(ae[(2 * tig) * kEStride + g], ae[(2 * tig + 1) * kEStride + g]);
        group_accumulate2(acc[0], acc[1], ds[0][0], ds[0][1], ds[1][0], ds[1][1], ds[2][0], ds[2][1], wsa, ae2, z2);
        group_accumulate2(acc[2], acc[3], ds[0][2], ds[0][3], ds[1][2], ds[1][3], ds[2][2], ds[2][3], wsb, ae2, z2);
    };
    int g = g0;
    for (; g + 1 < g1; g += 2) {  // two groups in flight; folded in group order
        uint32_t a0[4], a1[4], b0[4], b1[4];
        q8_group_frags(at, RT, ra, sw, g, tig, a0, a1);
        q8_group_frags(at, RT, ra, sw, g + 1, tig, b0, b1);
        int d0[3][4], d1[3][4];
        q8_group_sums(a0, a1, bword, g, d0);
        q8_group_sums(b0, b1, bword, g + 1, d1);
        fold(d0, g);
        fold(d1, g + 1);
    }
    if (g < g1) {
        uint32_t a0[4], a1[4];
        q8_group_frags(at, RT, ra, sw, g, tig, a0, a1);
        int d0[3][4];
        q8_group_sums(a0, a1, bword, g, d0);
        fold(d0, g);
    }
}

// Split sums of a 16 x 8 tile in shared memory: part[row][stream].
__device__ __forceinline__ void store_split(float* part, int lane, const float (&acc)[4]) {
    const int gid = lane >> 2, tig = lane & 3;
    part[gid * 8 + 2 * tig] = acc[0];
    part[gid * 8 + 2 * tig + 1] = acc[1];
    part[(gid + 8) * 8 + 2 * tig] = acc[2];
    part[(gid + 8) * 8 + 2 * tig + 1] = acc[3];
}

// Split sums added in split order (the q8_splits rule); splits are 128 floats apart.
__device__ __forceinline__ float sum_splits(const float* part, int S, int idx) {
    float tot = part[idx];
    for (int sp = 1; sp < S; sp++) tot = __fadd_rn(tot, part[sp * 128 + idx]);
    return tot;
}

template <int NC>
__device__ __forceinline__ void load_row_cg(const float* xb, int d, int lane, float4 (&v)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
        const int k = c * 128 + lane * 4;
        v[c] = k < d ? __ldcg(reinterpret_cast<const float4*>(xb + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// Slots and reset flags of the step's streams, staged once per CTA (they do not change during the
// step) so no loop waits on a global load of them.
struct StepMeta {
    uint32_t slot[kFusedMaxN];
    uint32_t fresh[kFusedMaxN];
};

__device__ __forceinline__ uint32_t live_slot(const FusedArgs& a, const StepMeta& m, int b) {
    const uint32_t s = m.slot[b];
    return s < (uint32_t)a.cap ? s : 0u;
}

// ---- job decompositions and prefetches ------------------------------------------------------

struct JobA {
    int h, r0, rows, g0, sg;  // half (0 = x, 1 = z), first row within the half, rows, first stream, streams
};
// x-half jobs first (64 rows x a.sga streams), then z-half jobs (a.rz rows x a.sgz streams)
__device__ __forceinline__ JobA job_a(const FusedArgs& a, int job) {
    const int nmb = a.di / 64, nx = (a.n + a.sga - 1) / a.sga, nz = (a.n + a.sgz - 1) / a.sgz;
    if (job < nmb * nx) return {0, (job / nx) * 64, 64, (job % nx) * a.sga, a.sga};
    job -= nmb * nx;
    return {1, (job / nz) * a.rz, a.rz, (job % nz) * a.sgz, a.sgz};
}
__device__ __forceinline__ int jobs_a(const FusedArgs& a) {
    return (a.di / 64) * ((a.n + a.sga - 1) / a.sga) + (a.di / a.rz) * ((a.n + a.sgz - 1) / a.sgz);
}

struct JobB {
    int g, b0;  // 64-channel group, first stream
};
__device__ __forceinline__ JobB job_b(const FusedArgs& a, int job) {
    const int nmb = a.di / 64;
    return {job % nmb, (job / nmb) * a.sgb};
}
__device__ __forceinline__ int jobs_b(const FusedArgs& a) { return (a.di / 64) * ((a.n + a.sgb - 1) / a.sgb); }

struct JobC {
    int row0, b0;
};
__device__ __forceinline__ JobC job_c(const FusedArgs& a, int job) {
    const int nt = (a.n + 7) / 8;
    return {(job / nt) * a.mc, (job % nt) * 8};
}
__device__ __forceinline__ int jobs_c(const FusedArgs& a) { return (a.d / a.mc) * ((a.n + 7) / 8); }

// Bulk copies issued by warp 0, lane-strided; lane 0 first arms `bar` with their total size.
// They read only operands no step kernel writes (weights, scales, group-blocked copies) and write
// only the bulk region of shared memory.
template <class F>
__device__ __forceinline__ void issue_copies(uint64_t* bar, uint32_t bytes, int count, F copy) {
    if (threadIdx.x >= 32) return;
    if (threadIdx.x == 0) tc::mbar_expect_tx(bar, bytes);
    __syncwarp();
    for (int k = threadIdx.x; k < count; k += 32) copy(k);
}

// Phase A operands that no earlier phase of this layer writes: the in_proj tile and its scales,
// the norm weights, and for x-half blocks the x_proj columns, the conv taps and the conv state.
__device__ __forceinline__ void prefetch_a(const FusedArgs& a, const StepMeta& m, const FusedLayer& L, int l, int job,
                                           char* P, CopyBatch& cb) {
    uint64_t* bar = cb.bar;
    cb.issued();
    const JobA jb = job_a(a, job);
    const int row0 = jb.h * a.di + jb.r0, c0 = jb.r0, mb = jb.r0 / 64;
    const int ns = min(jb.sg, a.n - jb.g0);
    const bool xh = jb.h == 0;
    const int nb = L.norm_b ? 1 : 0;
    const int nwb = jb.rows / 64;  // 64-row weight blocks, one contiguous copy each
    const int count = nwb + 2 + nb + (xh ? 2 : 0);
    const uint32_t bytes =
        a.g_in * jb.rows * 64 + jb.rows * a.g_in * 4 + a.d * 4 * (1 + nb) + (xh ? a.xr * 68 * 4 + 5 * 64 * 4 : 0);
    if (xh) {  // conv state: 256-byte pieces, as 16-byte copies spread over the CTA
        float* cv = reinterpret_cast<float*>(P + a.lay.a_conv);
        for (int i = threadIdx.x; i < ns * 3 * 16; i += kFusedThreads) {
            const int c4 = i & 15, kk = (i >> 4) % 3, s = i / 48;
            const uint32_t slot = live_slot(a, m, jb.g0 + s);
            cp_async16(cv + (s * 3 + kk) * 64 + c4 * 4, a.conv + conv_off(l, a.cap, slot, a.di, kk, c0 + c4 * 4));
        }
    }
    cp_async_commit();
    issue_copies(bar, bytes, count, [&](int k) {
        if (k < nwb) {
            tc::bulk_load(P + a.lay.a_w + k * a.g_in * 4096, L.in_blk + (size_t)(row0 / 64 + k) * a.g_in * 4096,
                          a.g_in * 4096, bar);
        } else if (k == nwb) {
            tc::bulk_load(P + a.lay.a_ws, L.in_s + (size_t)row0 * a.g_in, jb.rows * a.g_in * 4, bar);
        } else if (k == nwb + 1) {
            tc::bulk_load(P + a.lay.a_nw, L.norm_w, a.d * 4, bar);
        } else if (nb && k == nwb + 2) {
            tc::bulk_load(P + a.lay.a_nw + a.d * 4, L.norm_b, a.d * 4, bar);
        } else {
            const int q = k - (nwb + 2 + nb);
            if (q == 0) tc::bulk_load(P + a.lay.a_xw, L.xw_blk + (size_t)mb * a.xr * 68, a.xr * 68 * 4, bar);
            else tc::bulk_load(P + a.lay.a_ct, L.ct_blk + (size_t)mb * 5 * 64, 5 * 64 * 4, bar);
        }
    });
}

// Phase B operands: the channel group's dt_proj columns, A, dt bias and D, and the SSM state of
// the job's streams (written only by this phase of this layer).
__device__ __forceinline__ void prefetch_b(const FusedArgs& a, const StepMeta& m, const FusedLayer& L, int l, int job,
                                           char* P, CopyBatch& cb) {
    uint64_t* bar = cb.bar;
    cb.issued();
    const JobB jb = job_b(a, job);
    const int c0 = jb.g * 64, ns = min(a.sgb, a.n - jb.b0);
    float* st = reinterpret_cast<float*>(P + a.lay.b_ssm);
    for (int i = threadIdx.x; i < ns * 16 * 16; i += kFusedThreads) {
        const int c4 = i & 15, kk = (i >> 4) & 15, s = i >> 8;
        const uint32_t slot = live_slot(a, m, jb.b0 + s);
        cp_async16(st + (s * 16 + kk) * 64 + c4 * 4, a.ssm + ssm_off(l, a.cap, slot, a.di, kk, c0 + c4 * 4));
    }
    cp_async_commit();
    issue_copies(bar, (a.dr + 18) * 64 * 4, 1, [&](int) {
        tc::bulk_load(P + a.lay.b_sb, L.sb_blk + (size_t)jb.g * (a.dr + 18) * 64, (a.dr + 18) * 64 * 4, bar);
    });
}

// Phase C operands: the out_proj tile and scales, and the residual rows the job updates (written
// by this phase of the previous layer, so after a proxy fence).
__device__ __forceinline__ void prefetch_c(const FusedArgs& a, const FusedLayer& L, int job, char* P, CopyBatch& cb) {
    uint64_t* bar = cb.bar;
    cb.issued();
    const JobC jb = job_c(a, job);
    const int ns = min(8, a.n - jb.b0);
    float* xr = reinterpret_cast<float*>(P + a.lay.c_x);
    const int per = a.mc / 4;
    for (int i = threadIdx.x; i < ns * per; i += kFusedThreads) {
        const int s = i / per, c4 = i - s * per;
        cp_async16(xr + s * a.mc + c4 * 4, a.x + (size_t)(jb.b0 + s) * a.d + jb.row0 + c4 * 4);
    }
    cp_async_commit();
    const uint32_t bytes = a.g_out * a.mc * 64 + a.mc * a.g_out * 4;
    const int nwb = a.mc / 16;  // 16-row weight blocks, one contiguous copy each
    issue_copies(bar, bytes, nwb + 1, [&](int k) {
        if (k < nwb)
            tc::bulk_load(P + a.lay.c_w + k * a.g_out * 1024, L.out_blk + (size_t)(jb.row0 / 16 + k) * a.g_out * 1024,
                          a.g_out * 1024, bar);
        else
            tc::bulk_load(P + a.lay.c_ws, L.out_s + (size_t)jb.row0 * a.g_out, a.mc * a.g_out * 4, bar);
    });
}

// ---- phase bodies ----------------------------------------------------------------------------
// Each returns false when a bounded wait ran out (the error word says so); the kernel then leaves.

// A: norm + in_proj + conv/SiLU (x half) or gate (z half) + x_proj group chains (x half).
// Digit planes of stream s sit in 8-stream tiles: tile s/8, plane p, row s%8, pitch d + 16.
template <int NC>
__device__ __forceinline__ bool run_a(const FusedArgs& a, const StepMeta& m, const FusedLayer& L, int l, int job,
                                      char* sm, CopyBatch& pf, int* s_ok) {
    const JobA jb = job_a(a, job);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int ns = min(jb.sg, a.n - jb.g0);
    const int pitch = a.pitch_a, tile_bytes = 24 * pitch;
    int8_t* bq = reinterpret_cast<int8_t*>(sm + a.lay.bq);
    float* ae = reinterpret_cast<float*>(sm + a.lay.ae);
    float* part = reinterpret_cast<float*>(sm + a.lay.part);
    float* xc = reinterpret_cast<float*>(sm + a.lay.xc);
    if (ns == 1) {
        // one stream (batch 1): every warp computes the stream's norm and emits every eighth
        // 128-column chunk of its digit planes, so the per-chunk maxima and digit splits run on
        // eight warps instead of one; the other stream rows of the tile are zero
        float4 v[NC];
        load_row_cg<NC>(a.x + (size_t)jb.g0 * a.d, a.d, lane, v);
        if (!pf.wait(a.err, s_ok)) return false;
        NormWeights<NC> nw;
        const float* nws = reinterpret_cast<const float*>(sm + a.lay.a_nw);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int k = c * 128 + lane * 4;
            nw.w[c] = k < a.d ? *reinterpret_cast<const float4*>(nws + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            nw.b[c] = (L.norm_b && k < a.d) ? *reinterpret_cast<const float4*>(nws + a.d + k)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        norm_apply<NC>(v, a.d, nw, L.norm_b != nullptr, lane);
        int8_t* rows = bq;  // stream 0: tile 0, row 0
        norm_emit_q<NC>(v, a.d, lane, [&](int k, int p1, int p2, int p3, float gs, bool lead) {
            *reinterpret_cast<int*>(rows + k) = p1;
            *reinterpret_cast<int*>(rows + 8 * pitch + k) = p2;
            *reinterpret_cast<int*>(rows + 16 * pitch + k) = p3;
            if (lead) ae[k / kGroup] = gs;
        }, 8, warp);
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int s = warp + 8 * u;
            if (s == 0 || s >= jb.sg) continue;
            int8_t* zr = bq + (s >> 3) * tile_bytes + (s & 7) * pitch;
            for (int k = lane * 4; k < a.d; k += 128)
#pragma unroll
                for (int p = 0; p < 3; p++) *reinterpret_cast<int*>(zr + p * 8 * pitch + k) = 0;
            ae[s * kEStride + lane] = 0.0f;
        }
    } else {
        // this warp's rows (sga <= 16) are requested before anything waits
        float4 v2[2][NC];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int s = warp + 8 * u;
            if (s < ns) load_row_cg<NC>(a.x + (size_t)(jb.g0 + s) * a.d, a.d, lane, v2[u]);
        }
        if (!pf.wait(a.err, s_ok)) return false;
        NormWeights<NC> nw;
        const float* nws = reinterpret_cast<const float*>(sm + a.lay.a_nw);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int k = c * 128 + lane * 4;
            nw.w[c] = k < a.d ? *reinterpret_cast<const float4*>(nws + k) : make_float4(0.f, 0.f, 0.f, 0.f);
            nw.b[c] = (L.norm_b && k < a.d) ? *reinterpret_cast<const float4*>(nws + a.d + k)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int s = warp + 8 * u;
            if (s >= jb.sg) break;
            int8_t* rows = bq + (s >> 3) * tile_bytes + (s & 7) * pitch;  // plane p at + p * 8 * pitch
            if (s < ns) {
                float4 (&v)[NC] = v2[u];
                norm_apply<NC>(v, a.d, nw, L.norm_b != nullptr, lane);
                norm_emit_q<NC>(v, a.d, lane, [&](int k, int p1, int p2, int p3, float gs, bool lead) {
                    *reinterpret_cast<int*>(rows + k) = p1;
                    *reinterpret_cast<int*>(rows + 8 * pitch + k) = p2;
                    *reinterpret_cast<int*>(rows + 16 * pitch + k) = p3;
                    if (lead) ae[s * kEStride + k / kGroup] = gs;
                });
            } else {
                for (int k = lane * 4; k < a.d; k += 128)
#pragma unroll
                    for (int p = 0; p < 3; p++) *reinterpret_cast<int*>(rows + p * 8 * pitch + k) = 0;
                ae[s * kEStride + lane] = 0.0f;
            }
        }
    }
    __syncthreads();
    const int nmt = jb.rows >> 4;  // 16-row tiles of the job
    const int ntask = ((ns + 7) >> 3) * nmt * a.s_in;
    const int gid = lane >> 2, tig = lane & 3;
    for (int task = warp; task < ntask; task += 8) {
        const int t = task / (nmt * a.s_in), rem = task - t * nmt * a.s_in, mt = rem / a.s_in, sp = rem - mt * a.s_in;
        const int8_t* bt = bq + t * tile_bytes + gid * pitch + tig * 4;
        float acc[4];
        // weight block mt / 4 ([G][64][64]), its 16-row tile mt % 4; scales [rows][G]
        q8_tile16_split(reinterpret_cast<const int8_t*>(sm + a.lay.a_w) + (mt >> 2) * a.g_in * 4096, 64, (mt & 3) * 16,
                        reinterpret_cast<const float*>(sm + a.lay.a_ws) + (mt >> 2) * 64 * a.g_in, a.g_in,
                        a.g_in * sp / a.s_in,
                        a.g_in * (sp + 1) / a.s_in,
                        [&](int p, int g, int c) {
                            return *reinterpret_cast<const uint32_t*>(bt + p * 8 * pitch + g * 64 + c * 16);
                        },
                        ae + t * 8 * kEStride, lane, acc);
        store_split(part + (size_t)task * 128, lane, acc);
    }
    __syncthreads();
    const float* cv = reinterpret_cast<const float*>(sm + a.lay.a_conv);
    const float* ct = reinterpret_cast<const float*>(sm + a.lay.a_ct);
    const int rsh = jb.rows == 128 ? 7 : 6;
    for (int o = tid; o < (ns << rsh); o += kFusedThreads) {
        const int rl = o & (jb.rows - 1), s = o >> rsh, b = jb.g0 + s;
        const float tot =
            sum_splits(part + (size_t)((s >> 3) * nmt + (rl >> 4)) * a.s_in * 128, a.s_in, (rl & 15) * 8 + (s & 7));
        const int j = jb.r0 + rl;
        if (jb.h) {
            a.z[(size_t)b * a.di + j] = tot;
            continue;
        }
        // conv1d step + SiLU of channel j (the in_proj epilogue of the per-kernel path)
        const uint32_t slot = m.slot[b];
        float co = 0.0f;
        if (slot < (uint32_t)a.cap) {
            float s0 = 0.f, s1 = 0.f, s2 = 0.f;
            if (!m.fresh[b]) {
                s0 = cv[(s * 3 + 0) * 64 + rl];
                s1 = cv[(s * 3 + 1) * 64 + rl];
                s2 = cv[(s * 3 + 2) * 64 + rl];
            }
            float* st = a.conv + conv_off(l, a.cap, slot, a.di, 0, j);
            st[0] = s1;
            st[a.di] = s2;
            st[2 * a.di] = tot;
            co = conv_silu_taps(s0, s1, s2, tot, ct[rl], ct[64 + rl], ct[128 + rl], ct[192 + rl], ct[256 + rl]);
            a.conv_out[(size_t)b * a.di + j] = co;
        }
        xc[s * 68 + rl] = co;
    }
    if (jb.h == 0) {
        __syncthreads();
        // xproj_chain of every (row, stream) of the group, in register blocks of 2 rows x 4 streams
        // (16-byte shared loads: each weight and activation read feeds several chains)
        const float* xw = reinterpret_cast<const float*>(sm + a.lay.a_xw);
        const int nsb = (ns + 3) >> 2, nblk = ((a.xr + 1) >> 1) * nsb;
        for (int t = tid; t < nblk; t += kFusedThreads) {
            const int r0 = (t / nsb) * 2, s0 = (t % nsb) * 4;
            const float* w0 = xw + r0 * 68;
            const float* w1 = xw + min(r0 + 1, a.xr - 1) * 68;
            const float* xs[4];
#pragma unroll
            for (int j = 0; j < 4; j++) xs[j] = xc + min(s0 + j, ns - 1) * 68;
            float acc[2][4];
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
#pragma unroll 4
            for (int c = 0; c < 64; c += 4) {
                const float4 wa = *reinterpret_cast<const float4*>(w0 + c);
                const float4 wb = *reinterpret_cast<const float4*>(w1 + c);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float4 xv = *reinterpret_cast<const float4*>(xs[j] + c);
                    acc[0][j] = __fmaf_rn(wa.x, xv.x, acc[0][j]);
                    acc[0][j] = __fmaf_rn(wa.y, xv.y, acc[0][j]);
                    acc[0][j] = __fmaf_rn(wa.z, xv.z, acc[0][j]);
                    acc[0][j] = __fmaf_rn(wa.w, xv.w, acc[0][j]);
                    acc[1][j] = __fmaf_rn(wb.x, xv.x, acc[1][j]);
                    acc[1][j] = __fmaf_rn(wb.y, xv.y, acc[1][j]);
                    acc[1][j] = __fmaf_rn(wb.z, xv.z, acc[1][j]);
                    acc[1][j] = __fmaf_rn(wb.w, xv.w, acc[1][j]);
                }
            }
#pragma unroll
            for (int i = 0; i < 2; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (r0 + i < a.xr && s0 + j < ns)
                        a.xpart[((size_t)(jb.g0 + s0 + j) * (a.di / 64) + jb.r0 / 64) * a.xr + r0 + i] = acc[i][j];
        }
    }
    return true;
}

// B: x_proj group sums (group order), dt_proj, selective scan, D skip, z gate and the digit planes
// of out_proj's activation; thread = (channel tid % 64, stream tid / 64 + 4 * pass).
__device__ __forceinline__ bool run_b(const FusedArgs& a, const StepMeta& m, int l, int job, char* sm,
                                      float (*s_max)[8], CopyBatch& pf, int* s_ok) {
    const JobB jb = job_b(a, job);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int ns = min(a.sgb, a.n - jb.b0);
    float* zs = reinterpret_cast<float*>(sm + a.lay.zs);
    const int nmb = a.di / 64;
    const int ch = tid & 63, sl = tid >> 6, j = jb.g * 64 + ch;
    // this thread's (conv_out, z) for both passes, and up to 3 x_proj sums: every load in flight
    float xvp[2] = {0.f, 0.f}, zvp[2] = {0.f, 0.f};
#pragma unroll
    for (int pass = 0; pass < 2; pass++) {
        const int s = sl + 4 * pass;
        if (pass < a.sgb / 4 && s < ns) {
            xvp[pass] = __ldcg(a.conv_out + (size_t)(jb.b0 + s) * a.di + j);
            zvp[pass] = __ldcg(a.z + (size_t)(jb.b0 + s) * a.di + j);
        }
    }
    {
        // x_proj sums: thread = (stream, 4 consecutive rows); every group's 16 bytes in flight at once
        const int nq = a.xr >> 2;
        if (tid < ns * nq) {
            const int s = tid / nq, r4 = (tid - s * nq) * 4;
            const float4* pp = reinterpret_cast<const float4*>(a.xpart + ((size_t)(jb.b0 + s) * nmb) * a.xr + r4);
            float4 v[kEStride];  // [group] (stream's groups are xr floats apart)
#pragma unroll
            for (int q = 0; q < kEStride; q++)
                v[q] = q < nmb ? __ldcg(pp + (size_t)q * (a.xr >> 2)) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 t = v[0];
#pragma unroll
            for (int q = 1; q < kEStride; q++) {
                if (q < nmb) {
                    t.x = __fadd_rn(t.x, v[q].x);
                    t.y = __fadd_rn(t.y, v[q].y);
                    t.z = __fadd_rn(t.z, v[q].z);
                    t.w = __fadd_rn(t.w, v[q].w);
                }
            }
            *reinterpret_cast<float4*>(zs + s * a.xr + r4) = t;
        }
    }
    if (!pf.wait(a.err, s_ok)) return false;  // also publishes zs to the CTA
    const float* sb = reinterpret_cast<const float*>(sm + a.lay.b_sb);  // [dr + 18][64]
    const float* dtw = sb;
    const float* at = sb + a.dr * 64;
    const float dtb = sb[(a.dr + 16) * 64 + ch], dv = sb[(a.dr + 17) * 64 + ch];
    const float* pst = reinterpret_cast<const float*>(sm + a.lay.b_ssm);
    const int body = a.dr & ~7;
    for (int pass = 0; pass < a.sgb / 4; pass++) {
        const int s = sl + 4 * pass, b = jb.b0 + s;
        const bool valid = s < ns;
        bool ok = false;
        float gated = 0.0f;
        if (valid) {
            const uint32_t slot = m.slot[b];
            ok = slot < (uint32_t)a.cap;
            const bool fresh = m.fresh[b] != 0;
            float st[kDState];
#pragma unroll
            for (int k = 0; k < kDState; k++) st[k] = (ok && !fresh) ? pst[(s * kDState + k) * 64 + ch] : 0.0f;
            const float xv = pass == 0 ? xvp[0] : xvp[1];
            const float zv = pass == 0 ? zvp[0] : zvp[1];
            const float* zb = zs + s * a.xr;
            float dt = dt_dot8_body(zb, body, [&](int c) { return dtw[c * 64 + ch]; });
            for (int c = body; c < a.dr; c++) dt = __fadd_rn(dt, __fmul_rn(dtw[c * 64 + ch], zb[c]));
            dt = softplus(__fadd_rn(dt, dtb));
            const float* B = zb + a.dr;
            const float* C = zb + a.dr + kDState;
            const bool update = !(fabsf(dt) < 1e-6f);
            if (update) {  // state pairs on the packed pipe (same bits)
                const f2 z2 = f2_zero(), dt2 = f2_splat(dt), dtx2 = f2_splat(__fmul_rn(dt, xv));
#pragma unroll
                for (int k = 0; k < kDState; k += 2) {
                    const f2 arg = f2_sub(f2_splat(0.0f), f2_mulz(dt2, f2_pack(at[k * 64 + ch], at[(k + 1) * 64 + ch]), z2));
                    const f2 sn = f2_add(f2_mulz(lane_expf2(arg, z2), f2_pack(st[k], st[k + 1]), z2),
                                         f2_mulz(dtx2, f2_pack(B[k], B[k + 1]), z2));
                    f2_unpack(sn, st[k], st[k + 1]);
                }
            }
            if (ok && (update || fresh)) {
                float* sp = a.ssm + ssm_off(l, a.cap, slot, a.di, 0, j);
#pragma unroll
                for (int k = 0; k < kDState; k++) sp[k * 64] = st[k];
            }
            const float y = __fadd_rn(ssm_out16(st, C), __fmul_rn(dv, xv));
            gated = ok ? __fmul_rn(y, __fmul_rn(zv, lane_sigmoid(zv))) : 0.0f;
        }
        // digit planes over the stream's 64 channels (two warps)
        float mx = warp_allmax(fabsf(gated));
        if (lane == 0) s_max[pass & 1][warp] = mx;
        __syncthreads();
        mx = fmaxf(s_max[pass & 1][warp & ~1], s_max[pass & 1][warp | 1]);
        if (valid && ok) {
            float ginv, gs = group_scale(mx, &ginv);
            const Digits3 dg = split_digits(gated, ginv);
            a.act_q[dq_off(a.cap_pad, 0, b, j)] = (int8_t)dg.d1;
            a.act_q[dq_off(a.cap_pad, 1, b, j)] = (int8_t)dg.d2;
            a.act_q[dq_off(a.cap_pad, 2, b, j)] = (int8_t)dg.d3;
            if (ch == 0) a.act_e[(size_t)b * kEStride + jb.g] = gs;
        }
    }
    return true;
}

// B for a job of one stream (the batch-1 case): four threads per channel, each owning states
// t, t + 4, t + 8, t + 12, with the dt_proj lanes and the state-output lanes finished by quad
// shuffles in the trees of the one-thread form (scan_block<4>'s arithmetic), so the 16
// exponentials of a channel run on four threads.  Same bits as run_b.
__device__ __forceinline__ bool run_b1(const FusedArgs& a, const StepMeta& m, int l, int job, char* sm,
                                       float (*s_max)[8], CopyBatch& pf, int* s_ok) {
    const JobB jb = job_b(a, job);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    float* zs = reinterpret_cast<float*>(sm + a.lay.zs);
    const int nmb = a.di / 64;
    const int t = lane & 3, ch = warp * 8 + (lane >> 2), j = jb.g * 64 + ch;
    const int b = jb.b0;
    const float xv = __ldcg(a.conv_out + (size_t)b * a.di + j);
    const float zv = __ldcg(a.z + (size_t)b * a.di + j);
    {
        const int nq = a.xr >> 2;
        if (tid < nq) {  // x_proj sums of the stream, group order
            const int r4 = tid * 4;
            const float4* pp = reinterpret_cast<const float4*>(a.xpart + ((size_t)b * nmb) * a.xr + r4);
            float4 v[kEStride];
#pragma unroll
            for (int q = 0; q < kEStride; q++)
                v[q] = q < nmb ? __ldcg(pp + (size_t)q * (a.xr >> 2)) : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 tt = v[0];
#pragma unroll
            for (int q = 1; q < kEStride; q++) {
                if (q < nmb) {
                    tt.x = __fadd_rn(tt.x, v[q].x);
                    tt.y = __fadd_rn(tt.y, v[q].y);
                    tt.z = __fadd_rn(tt.z, v[q].z);
                    tt.w = __fadd_rn(tt.w, v[q].w);
                }
            }
            *reinterpret_cast<float4*>(zs + r4) = tt;
        }
    }
    if (!pf.wait(a.err, s_ok)) return false;  // also publishes zs to the CTA
    const float* sb = reinterpret_cast<const float*>(sm + a.lay.b_sb);  // [dr + 18][64]
    const float* dtw = sb;
    const float* at = sb + a.dr * 64;
    const float dtb = sb[(a.dr + 16) * 64 + ch], dv = sb[(a.dr + 17) * 64 + ch];
    const float* pst = reinterpret_cast<const float*>(sm + a.lay.b_ssm);  // stream 0's [16][64]
    const uint32_t slot = m.slot[b];
    const bool ok = slot < (uint32_t)a.cap;
    const bool fresh = m.fresh[b] != 0;
    float st[4];
#pragma unroll
    for (int k = 0; k < 4; k++) st[k] = (ok && !fresh) ? pst[(t + 4 * k) * 64 + ch] : 0.0f;
    // dt_proj: this thread holds 8-lane lanes t and t + 4 of dt_dot8_body's tree
    const int body = a.dr & ~7;
    float la = 0.0f, lb = 0.0f;
    for (int c = 0; c < body; c += 8) {
        la = __fadd_rn(la, __fmul_rn(dtw[(c + t) * 64 + ch], zs[c + t]));
        lb = __fadd_rn(lb, __fmul_rn(dtw[(c + t + 4) * 64 + ch], zs[c + t + 4]));
    }
    float pr = __fadd_rn(la, lb);
    pr = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 2));
    float dt = __fadd_rn(pr, __shfl_xor_sync(0xffffffffu, pr, 1));
    for (int c = body; c < a.dr; c++) dt = __fadd_rn(dt, __fmul_rn(dtw[c * 64 + ch], zs[c]));
    dt = softplus(__fadd_rn(dt, dtb));
    const float* B = zs + a.dr;
    const float* C = zs + a.dr + kDState;
    const bool update = !(fabsf(dt) < 1e-6f);
    if (update) {  // states t + 4k, t + 4k + 4 in pairs on the packed pipe (same bits)
        const f2 z2 = f2_zero(), dt2 = f2_splat(dt), dtx2 = f2_splat(__fmul_rn(dt, xv));
#pragma unroll
        for (int k = 0; k < 4; k += 2) {
            const int n2 = t + 4 * k;
            const f2 arg = f2_sub(f2_splat(0.0f), f2_mulz(dt2, f2_pack(at[n2 * 64 + ch], at[(n2 + 4) * 64 + ch]), z2));
            const f2 sn = f2_add(f2_mulz(lane_expf2(arg, z2), f2_pack(st[k], st[k + 1]), z2),
                                 f2_mulz(dtx2, f2_pack(B[n2], B[n2 + 4]), z2));
            f2_unpack(sn, st[k], st[k + 1]);
        }
    }
    if (ok && (update || fresh)) {
        float* sp = a.ssm + ssm_off(l, a.cap, slot, a.di, 0, j);
#pragma unroll
        for (int k = 0; k < 4; k++) sp[(t + 4 * k) * 64] = st[k];
    }
    // hsum_ssm: lanes t and t + 4 here, then xor 1 and xor 2 across the quad
    const float l0 = __fadd_rn(__fmul_rn(st[0], C[t]), __fmul_rn(st[2], C[t + 8]));
    const float l4 = __fadd_rn(__fmul_rn(st[1], C[t + 4]), __fmul_rn(st[3], C[t + 12]));
    float h = __fadd_rn(l0, l4);
    h = __fadd_rn(h, __shfl_xor_sync(0xffffffffu, h, 1));
    h = __fadd_rn(h, __shfl_xor_sync(0xffffffffu, h, 2));
    const float y = __fadd_rn(h, __fmul_rn(dv, xv));
    const float gated = ok ? __fmul_rn(y, __fmul_rn(zv, lane_sigmoid(zv))) : 0.0f;
    // digit planes over the group's 64 channels (all eight warps)
    float mx = warp_allmax(fabsf(gated));
    if (lane == 0) s_max[0][warp] = mx;
    __syncthreads();
    mx = s_max[0][0];
#pragma unroll
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, s_max[0][w]);
    if (ok && t == 0) {
        float ginv, gs = group_scale(mx, &ginv);
        const Digits3 dg = split_digits(gated, ginv);
        a.act_q[dq_off(a.cap_pad, 0, b, j)] = (int8_t)dg.d1;
        a.act_q[dq_off(a.cap_pad, 1, b, j)] = (int8_t)dg.d2;
        a.act_q[dq_off(a.cap_pad, 2, b, j)] = (int8_t)dg.d3;
        if (ch == 0) a.act_e[(size_t)b * kEStride + jb.g] = gs;
    }
    return true;
}

// C: out_proj + residual for mc rows x 8 streams; one (16-row tile, split) per warp task.  The
// streams' digit planes arrive as the scan wrote them (8-row halves of the tiled layout, 64-byte
// swizzled rows), one bulk copy per (group, plane).
__device__ __forceinline__ bool run_c(const FusedArgs& a, int job, char* sm, CopyBatch& pf, CopyBatch& stg,
                                      int* s_ok) {
    const JobC jb = job_c(a, job);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int ns = min(8, a.n - jb.b0);
    int8_t* bq = reinterpret_cast<int8_t*>(sm + a.lay.bq);
    float* ae = reinterpret_cast<float*>(sm + a.lay.ae);
    float* part = reinterpret_cast<float*>(sm + a.lay.part);
    // the scan's digit planes of the 8 streams (8-row halves of the tiled layout: 512 contiguous
    // bytes per group and plane) and their exponents, as 16-byte copies over the CTA
    for (int i = tid; i < a.g_out * 3 * 32; i += kFusedThreads) {
        const int k = i >> 5, c16 = i & 31, g = k / 3, p = k - 3 * g;
        cp_async16(bq + k * 512 + c16 * 16, a.act_q + dq_off(a.cap_pad, p, jb.b0, g * 64) + c16 * 16);
    }
    for (int i = tid; i < ns * (kEStride / 4); i += kFusedThreads)
        cp_async16(ae + i * 4, a.act_e + (size_t)jb.b0 * kEStride + i * 4);
    cp_async_commit();
    (void)stg;
    if (!pf.wait(a.err, s_ok)) return false;  // waits for this thread's cp.async groups too
    const int ntask = (a.mc / 16) * a.s_out;
    const int gid = lane >> 2, tig = lane & 3;
    const uint32_t bsw = ((uint32_t)gid >> 1) & 3u;  // swizzle phase of stream row gid (b0 % 8 == 0)
    const int8_t* brow = bq + gid * 64 + tig * 4;
    for (int task = warp; task < ntask; task += 8) {
        const int mt = task / a.s_out, sp = task - mt * a.s_out;
        float acc[4];
        // weight block mt ([G][16][64]); scales [rows][G]
        q8_tile16_split(reinterpret_cast<const int8_t*>(sm + a.lay.c_w) + mt * a.g_out * 1024, 16, 0,
                        reinterpret_cast<const float*>(sm + a.lay.c_ws) + mt * 16 * a.g_out, a.g_out,
                        a.g_out * sp / a.s_out,
                        a.g_out * (sp + 1) / a.s_out,
                        [&](int p, int g, int c) {
                            return *reinterpret_cast<const uint32_t*>(brow + (g * 3 + p) * 512 + ((c ^ bsw) << 4));
                        },
                        ae, lane, acc);
        store_split(part + (size_t)task * 128, lane, acc);
    }
    __syncthreads();
    const float* xr = reinterpret_cast<const float*>(sm + a.lay.c_x);
    for (int o = tid; o < a.mc * 8; o += kFusedThreads) {
        const int rr = o >> 3, s = o & 7;
        if (s < ns) {
            const float tot = sum_splits(part + (size_t)(rr >> 4) * a.s_out * 128, a.s_out, (rr & 15) * 8 + s);
            a.x[(size_t)(jb.b0 + s) * a.d + jb.row0 + rr] = __fadd_rn(xr[s * a.mc + rr], tot);
        }
    }
    return true;
}

template <int NC>
__global__ void __launch_bounds__(kFusedThreads, 1) k_step_fused(FusedArgs a) {
    extern __shared__ float4 smem_f4[];
    char* sm = reinterpret_cast<char*>(smem_f4);
    __shared__ float s_max[2][8];
    __shared__ int s_ok;
    __shared__ StepMeta meta;
    __shared__ __align__(8) uint64_t pf_bar, st_bar;
    if (threadIdx.x < a.n) {
        meta.slot[threadIdx.x] = a.slots[threadIdx.x];
        meta.fresh[threadIdx.x] = a.rflag[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        tc::mbar_init(&pf_bar, 1);
        tc::mbar_init(&st_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    uint32_t target = 0;
    CopyBatch pf{&pf_bar, 0u, 0}, stg{&st_bar, 0u, 0};
    const int ja = jobs_a(a), jbn = jobs_b(a), jc = jobs_c(a);
    const int first = blockIdx.x;
    // On an error exit, copies still in flight land before the CTA leaves (bounded waits): the
    // prefetch issued last (if its wait did not complete) and a phase-C staging copy.
    auto drain = [&]() {
        if (pf.pending) pf.wait(a.err, &s_ok);
        if (stg.pending) stg.wait(a.err, &s_ok);
    };
    if (first < ja) prefetch_a(a, meta, a.layers[0], 0, first, sm, pf);
    for (int l = 0; l < a.nl; l++) {
        const FusedLayer L = a.layers[l];
        for (int job = first; job < ja; job += gridDim.x) {
            if (job != first) {
                __syncthreads();
                prefetch_a(a, meta, L, l, job, sm, pf);
            }
            if (!run_a<NC>(a, meta, L, l, job, sm, pf, &s_ok)) return drain();
        }
        grid_arrive(a.bar, target);
        if (first < jbn) prefetch_b(a, meta, L, l, first, sm, pf);
        if (!grid_wait(a.bar, target, a.err, &s_ok)) return drain();
        for (int job = first; job < jbn; job += gridDim.x) {
            if (job != first) {
                __syncthreads();
                prefetch_b(a, meta, L, l, job, sm, pf);
            }
            const bool one = min(a.sgb, a.n - job_b(a, job).b0) == 1;
            if (!(one ? run_b1(a, meta, l, job, sm, s_max, pf, &s_ok) : run_b(a, meta, l, job, sm, s_max, pf, &s_ok)))
                return drain();
        }
        grid_arrive(a.bar, target);
        if (first < jc) prefetch_c(a, L, first, sm, pf);
        if (!grid_wait(a.bar, target, a.err, &s_ok)) return drain();
        for (int job = first; job < jc; job += gridDim.x) {
            if (job != first) {
                __syncthreads();
                prefetch_c(a, L, job, sm, pf);
            }
            if (!run_c(a, job, sm, pf, stg, &s_ok)) return drain();
        }
        grid_arrive(a.bar, target);
        if (l + 1 < a.nl && first < ja) prefetch_a(a, meta, a.layers[l + 1], l + 1, first, sm, pf);
        if (!grid_wait(a.bar, target, a.err, &s_ok)) return drain();
    }
    // final norm: the head's digit planes
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    NormWeights<NC> nw;
    nw.load(a.norm_f_w, a.norm_f_b, a.d, lane);
    const ActOut out{nullptr, a.act_q, a.act_e, a.cap_pad, a.d};
    for (int b = blockIdx.x * 8 + warp; b < a.n; b += gridDim.x * 8) {
        float4 v[NC];
        load_row_cg<NC>(a.x + (size_t)b * a.d, a.d, lane, v);
        norm_apply<NC>(v, a.d, nw, a.norm_f_b != nullptr, lane);
        zero_if_rejected<NC>(v, meta.slot[b] == kRejected);  // a rejected stream's logits are zeros
        norm_emit<NC>(b, v, a.d, out, lane);
    }
}

}  // namespace rk
