// Clustered small-batch decode step: every layer of one Mamba Q8 step in ONE kernel whose
// thread-block clusters run independently.
//
// A grid-wide barrier costs about 1.2 us on a B200 and a phase that starts after one must re-read
// its inputs from L2; a step of 24 layers with three dependent phases each pays that 72 times.
// Here the streams of the step are split over C clusters of 16 CTAs (at most 8 streams each) and a
// cluster never waits for another: every exchange inside a layer goes through distributed shared
// memory (st.shared::cluster) and a cluster barrier (about 0.2 us).  Every CTA keeps the full
// residual rows of its cluster's streams in its own shared memory.
//
// Work of CTA rank r of a cluster, per layer:
//   A  norm of every stream of the cluster (warp w: stream w) into digit planes, then for each
//      64-channel group g it owns (g = r, r + 16): the x-half in_proj rows of g (+ conv/SiLU,
//      conv state, x_proj group chains, sent to the stream-owner CTAs) and the z-half rows of g
//      (kept locally).                                                      -> cluster barrier
//   A2 CTA s (< streams) adds stream s's x_proj chains in group order and sends the sums to every
//      CTA.                                                                 -> cluster barrier
//   B  for each owned group g: dt_proj, selective scan, D skip, z gate, the digit planes of
//      out_proj's activation; the planes go to every CTA.                   -> cluster barrier
//   C  for each owned 16-row out_proj tile: out_proj + residual; the new residual rows go to every
//      CTA.                                                                 -> cluster barrier
// After the last layer CTA 0 writes the final norm's digit planes for the head kernel.
//
// Operands are streamed by one thread per CTA into a ring of shared memory, in exactly the order the
// CTA consumes them (weights of each job and accumulation split, scales, x_proj / conv / scan
// blocks, the conv and SSM state of the owned channel groups): contiguous bulk copies
// (cp.async.bulk) completing on one of 16 item mbarriers.  The ring is refilled as items are
// released, so the copies of later phases and layers overlap the current phase's arithmetic.
// Weights and the group-blocked operand copies are the fused step's (FusedLayer); the state is
// stored channel-blocked, so a (stream, channel group) state is one contiguous piece.
//
// Arithmetic is that of the per-kernel step, in the same order (norm_apply / digit planes, the
// q8_splits combine, conv_silu_taps, the x_proj group chains summed in group order, the one-thread
// scan, the residual add), so a stream's bits do not depend on which path ran it.
//
// Every wait on a copy is bounded in time (the fused step's limit); one that runs out sets bit 2
// of the error word, the CTA stops issuing copies and computes on whatever it has, still taking
// part in every cluster barrier, and drains its copies before it exits.  Nothing spins on another
// CTA except the hardware cluster barrier, which every CTA reaches on every path.
#pragma once
#include "rk_fused.cuh"

namespace rk {

constexpr int kClCTAs = 16;      // CTAs per cluster
constexpr int kClThreads = 256;
constexpr int kClMaxNS = 8;      // streams per cluster: one n8 tile of the warp-level MMA
constexpr int kClItems = 16;     // ring items in flight (one mbarrier each)
constexpr int kClMaxG = 2;       // 64-channel groups per CTA (d_inner <= 2048)
constexpr int kClMaxT = 4;       // 16-row out_proj tiles per CTA (d_model <= 1024)

struct ClLayout {
    int xs;      // f32 [8][d] residual rows of the cluster's streams
    int bq;      // int8 digit planes of the norm: [3][8][pitch]
    int ae;      // f32 [8][kEStride] their group exponents
    int part;    // f32 split sums
    int co;      // f32 [kClMaxG][8][64] conv outputs of the owned groups
    int zl;      // f32 [kClMaxG][8][64] z of the owned groups
    int rchain;  // f32 [G_out][xr] x_proj chains of this CTA's stream (stream owners)
    int xc;      // f32 [8][68] staged conv outputs for the chains
    int zs;      // f32 [8][xr] x_proj sums (dt_raw, B, C) of every stream
    int gq;      // int8 [G_out][3][8][64] out_proj digit planes (64-byte swizzle), all groups
    int ge;      // f32 [8][kEStride] their exponents
    int xn;      // f32 [kClMaxT][8][16] new residual rows of the owned tiles
    int layers;  // FusedLayer [nl]: the layer table, read by the copy issuer without a global load
    int ring;    // the operand ring
    int total;
};

struct ClArgs {
    int n, cap, cap_pad, d, di, dr, xr, nl;
    int g_in, s_in, g_out, s_out;
    int n_clusters;
    int ring;      // ring bytes
    int pitch_a;   // bytes per digit-plane row of the norm planes (d + 16)
    ClLayout lay;
    const uint32_t* slots;  // validated slots (kRejected: a stream that touches no state)
    const uint32_t* rflag;
    const float* x;         // [cap][d] embedding rows of the step (k_embed)
    float* conv;            // channel-blocked conv state
    float* ssm;             // channel-blocked SSM state
    int8_t* act_q;          // final norm's digit planes (head input)
    float* act_e;
    const FusedLayer* layers;
    const float* norm_f_w;
    const float* norm_f_b;
    uint32_t* err;
};

// Host-side shared-memory map for one shape (ring = what is left of `smem_max`).
inline ClLayout cluster_layout(const ClArgs& a, int smem_max) {
    ClLayout L{};
    int o = 0;
    L.xs = o;     o += align16(kClMaxNS * a.d * 4);
    L.bq = o;     o += align16(3 * kClMaxNS * a.pitch_a);
    L.ae = o;     o += align16(kClMaxNS * kEStride * 4);
    const int pa = 4 * a.s_in, pc = kClMaxT * a.s_out;  // split-sum tasks of a job / of the tiles
    L.part = o;   o += align16((pa > pc ? pa : pc) * 128 * 4);
    L.co = o;     o += align16(kClMaxG * kClMaxNS * 64 * 4);
    L.zl = o;     o += align16(kClMaxG * kClMaxNS * 64 * 4);
    L.rchain = o; o += align16(a.g_out * a.xr * 4);
    L.xc = o;     o += align16(kClMaxNS * 68 * 4);
    L.zs = o;     o += align16(kClMaxNS * a.xr * 4);
    L.gq = o;     o += align16(a.g_out * 3 * 512);
    L.ge = o;     o += align16(kClMaxNS * kEStride * 4);
    L.xn = o;     o += align16(kClMaxT * kClMaxNS * 16 * 4);
    L.layers = o; o += align16(a.nl * (int)sizeof(FusedLayer));
    o = (o + 127) & ~127;
    L.ring = o;
    L.total = smem_max;
    return L;
}

// ---- cluster primitives ----------------------------------------------------------------------

__device__ __forceinline__ uint32_t cl_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cl_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
// Every thread of every CTA of the cluster; release/acquire orders the DSMEM stores before it.
__device__ __forceinline__ void cl_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of this CTA's shared-memory location `p` in CTA `rank`.
__device__ __forceinline__ uint32_t cl_map(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ void cl_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cl_st4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void cl_st16(uint32_t addr, uint4 v) {
    asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}


// ---- the operand ring --------------------------------------------------------------------------
//
// Items are numbered k = layer * per_layer + j in the CTA's consumption order.  Per layer:
//   j = 0                NORM  norm weight (and bias)
//   per owned group gi:  XW[0..S_in)  x-half in_proj weights of one accumulation split each
//                                      (XW[0] first holds the job's scales [64][G_in])
//                        XE    x_proj block [xr][68], conv taps and bias [5][64], conv state of
//                              each stream [3][64]
//                        ZW[0..S_in)  z-half in_proj weights (ZW[0] with the scales)
//   per owned group gi:  SB    dt_proj columns, A, dt bias, D [dr + 18][64], SSM state of each
//                              stream [16][64]
//   per owned tile ti:   CW    out_proj weights [G_out][16][64], then scales [16][G_out]
// Thread 0 issues and releases items; every thread reads an item only after wait_items.

struct ClRing {
    uint64_t bar[kClItems];
    int start[kClItems];        // ring byte offset of item k (slot k % kClItems)
    long long endpos[kClItems]; // ring position after item k
    long long head, tail;       // positions (monotonic): next free byte, first unreleased byte
    int issued, released;       // item counts
    int abort;                  // a copy wait ran out: stop issuing, skip waits
};

struct ClCtx {
    int rank, ns, b0;      // this CTA's rank, the cluster's streams [b0, b0 + ns)
    int ng, nt;            // owned channel groups, owned out_proj tiles
    int per_layer, total;  // ring items per layer, in the whole step
};

__device__ __forceinline__ int cl_group(const ClCtx& c, int gi) { return c.rank + kClCTAs * gi; }
__device__ __forceinline__ int cl_tile(const ClCtx& c, int ti) { return c.rank + kClCTAs * ti; }

// Copies of item k: emit(byte offset in the item, source, bytes) for each piece; returns the item's
// size.  Pieces are 16-byte multiples at 16-byte offsets.
template <class Emit>
__device__ __forceinline__ int cl_item(const ClArgs& a, const ClCtx& c, const StepMeta& m, const FusedLayer* layers,
                                       int k, Emit emit) {
    const int l = k / c.per_layer;
    int j = k - l * c.per_layer;
    const FusedLayer& L = layers[l];
    int o = 0, part = 0;
    auto put = [&](const void* src, int bytes) {
        emit(part++, o, src, bytes);
        o += align16(bytes);
    };
    auto state_slot = [&](int s) -> uint32_t {
        const uint32_t sl = m.slot[s];
        return sl < (uint32_t)a.cap ? sl : 0u;  // a rejected stream's copy reads slot 0 and is ignored
    };
    if (j == 0) {
        put(L.norm_w, a.d * 4);
        if (L.norm_b) put(L.norm_b, a.d * 4);
        return o;
    }
    j -= 1;
    const int per_g = 2 * a.s_in + 1;
    if (j < c.ng * per_g) {
        const int gi = j / per_g, w = j - gi * per_g, g = cl_group(c, gi);
        if (w == a.s_in) {  // XE
            put(L.xw_blk + (size_t)g * a.xr * 68, a.xr * 68 * 4);
            put(L.ct_blk + (size_t)g * 5 * 64, 5 * 64 * 4);
            for (int s = 0; s < c.ns; s++)
                put(a.conv + conv_off(l, a.cap, state_slot(s), a.di, 0, g * 64), (kDConv - 1) * 64 * 4);
            return o;
        }
        const bool z = w > a.s_in;
        const int sp = z ? w - a.s_in - 1 : w;
        const int blk = (z ? a.di / 64 : 0) + g;  // 64-row block of in_proj
        if (sp == 0) put(L.in_s + (size_t)blk * 64 * a.g_in, 64 * a.g_in * 4);
        const int g0 = a.g_in * sp / a.s_in, g1 = a.g_in * (sp + 1) / a.s_in;
        put(L.in_blk + ((size_t)blk * a.g_in + g0) * 4096, (g1 - g0) * 4096);
        return o;
    }
    j -= c.ng * per_g;
    if (j < c.ng) {  // SB
        const int g = cl_group(c, j);
        put(L.sb_blk + (size_t)g * (a.dr + 18) * 64, (a.dr + 18) * 64 * 4);
        for (int s = 0; s < c.ns; s++) put(a.ssm + ssm_off(l, a.cap, state_slot(s), a.di, 0, g * 64), kDState * 64 * 4);
        return o;
    }
    j -= c.ng;
    const int t = cl_tile(c, j);  // CW
    put(L.out_blk + (size_t)t * a.g_out * 1024, a.g_out * 1024);
    put(L.out_s + (size_t)t * 16 * a.g_out, 16 * a.g_out * 4);
    return o;
}

// Warp 0 (all lanes, converged): issue items while a barrier slot and ring space are free.  Lane 0
// keeps the ring's books and arms the item's barrier with its total size before any lane issues one
// of the item's copies (piece i by lane i % 32).
__device__ __forceinline__ void cl_refill(const ClArgs& a, const ClCtx& c, const StepMeta& m, const FusedLayer* layers,
                                          ClRing& R, char* ring) {
    const int lane = threadIdx.x & 31;
    const long long RB = a.ring;
    for (;;) {
        int k = -1, off = 0;
        if (lane == 0 && R.issued < c.total && !R.abort && R.issued - R.released < kClItems) {
            const int kk = R.issued;
            const int size = cl_item(a, c, m, layers, kk, [](int, int, const void*, int) {});
            long long pos = R.head;
            long long o = pos % RB;
            if (o + size > RB) {  // items never wrap: skip to the ring's start
                pos += RB - o;
                o = 0;
            }
            if (pos + size - R.tail <= RB) {
                const int slot = kk % kClItems;
                R.start[slot] = (int)o;
                R.endpos[slot] = pos + size;
                R.head = pos + size;
                R.issued = kk + 1;
                tc::mbar_expect_tx(&R.bar[slot], (uint32_t)size);
                // wait test: the step's very first item never receives its bytes
                k = (kk == 0 && blockIdx.x == 0 && tc::take_wait_test(1)) ? -2 : kk;
                off = (int)o;
            }
        }
        k = __shfl_sync(0xffffffffu, k, 0);
        off = __shfl_sync(0xffffffffu, off, 0);
        if (k == -1) return;
        if (k >= 0)
            cl_item(a, c, m, layers, k, [&](int i, int o, const void* src, int bytes) {
                if ((i & 31) == lane) tc::bulk_load(ring + off + o, src, (uint32_t)bytes, &R.bar[k % kClItems]);
            });
        __syncwarp();
    }
}

// Bounded wait for item k's copies (thread 0); false when the limit ran out.
__device__ __forceinline__ bool cl_wait_one(ClRing& R, int k) {
    uint64_t* bar = &R.bar[k % kClItems];
    const uint32_t par = (uint32_t)((k / kClItems) & 1);
    if (tc::mbar_try_wait(bar, par)) return true;
    const unsigned long long t0 = globaltimer_ns();
    const unsigned long long lim = *(volatile unsigned long long*)&tc::g_wait_ns;
    while (!tc::mbar_try_wait(bar, par))
        if (globaltimer_ns() - t0 > lim) return false;
    return true;
}

// Every thread: items [k0, k1) have landed (or the CTA has aborted).  Returns nothing: after an
// abort the CTA computes on whatever the ring holds and only its error word matters.
__device__ __forceinline__ void cl_wait_items(const ClArgs& a, const ClCtx& c, const StepMeta& m,
                                              const FusedLayer* layers, ClRing& R, char* ring, int k0, int k1) {
    if (threadIdx.x < 32 && R.issued < k1) cl_refill(a, c, m, layers, R, ring);
    if (threadIdx.x == 0) {
        for (int k = k0; k < k1 && !R.abort; k++) {
            if (k >= R.issued) {  // the ring cannot hold the item: a layout error, never a wait
                R.abort = 1;
                atomicOr(a.err, kErrGridWait);
                break;
            }
            if (!cl_wait_one(R, k)) {
                R.abort = 1;
                atomicOr(a.err, kErrGridWait);
            }
        }
        // after an abort, items that were never issued read from the ring's start (in bounds:
        // every item fits the ring)
        for (int k = k0; k < k1 && R.abort; k++)
            if (k >= R.issued) R.start[k % kClItems] = 0;
    }
    __syncthreads();
}

// Warp 0, after a __syncthreads that ends every read of items < k1: release them and refill.
__device__ __forceinline__ void cl_release(const ClArgs& a, const ClCtx& c, const StepMeta& m, const FusedLayer* layers,
                                           ClRing& R, char* ring, int k1) {
    if (threadIdx.x >= 32) return;
    if (threadIdx.x == 0) {
        while (R.released < k1 && R.released < R.issued) {
            R.tail = R.endpos[R.released % kClItems];
            R.released++;
        }
    }
    __syncwarp();
    cl_refill(a, c, m, layers, R, ring);
}

__device__ __forceinline__ const char* cl_ptr(const ClRing& R, const char* ring, int k) {
    return ring + R.start[k % kClItems];
}

// ---- phases ------------------------------------------------------------------------------------

// A, one 64-row in_proj job (x half when z == false) of channel group g for the cluster's streams:
// the split MMAs over the norm's digit planes into `part`.  Items [k, k + S_in) are the job's.
__device__ __forceinline__ void cl_job_mma(const ClArgs& a, const ClRing& R, const char* ring, const char* sm, int k) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int pitch = a.pitch_a;
    const int8_t* bt = reinterpret_cast<const int8_t*>(sm + a.lay.bq) + gid * pitch + tig * 4;
    const float* ae = reinterpret_cast<const float*>(sm + a.lay.ae);
    float* part = reinterpret_cast<float*>(const_cast<char*>(sm) + a.lay.part);
    const char* x0 = cl_ptr(R, ring, k);  // XW[0]: scales [64][G_in], then split 0's weights
    const float* ws = reinterpret_cast<const float*>(x0);
    const int sc = align16(64 * a.g_in * 4);
    for (int task = warp; task < 4 * a.s_in; task += kClThreads / 32) {
        const int sp = task >> 2, mt = task & 3;
        const int g0 = a.g_in * sp / a.s_in, g1 = a.g_in * (sp + 1) / a.s_in;
        const int8_t* wsp = reinterpret_cast<const int8_t*>(cl_ptr(R, ring, k + sp) + (sp == 0 ? sc : 0));
        float acc[4];
        q8_tile16_split(wsp - (size_t)g0 * 64 * 64, 64, mt * 16, ws, a.g_in, g0, g1,
                        [&](int p, int g, int c) {
                            return *reinterpret_cast<const uint32_t*>(bt + p * 8 * pitch + g * 64 + c * 16);
                        },
                        ae, lane, acc);
        store_split(part + (size_t)(mt * a.s_in + sp) * 128, lane, acc);
    }
}

template <int NC>
__global__ void __launch_bounds__(kClThreads, 1) k_step_cluster(ClArgs a) {
    extern __shared__ __align__(128) char sm[];
    __shared__ ClRing R;
    __shared__ StepMeta meta;
    __shared__ float s_max[2][8];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    ClCtx c;
    c.rank = (int)cl_rank();
    {
        const int cid = (int)cl_id(), C = a.n_clusters, base = a.n / C, rem = a.n % C;
        c.ns = base + (cid < rem ? 1 : 0);
        c.b0 = cid * base + (cid < rem ? cid : rem);
    }
    c.ng = c.rank < a.g_out ? (a.g_out - 1 - c.rank) / kClCTAs + 1 : 0;
    c.nt = c.rank < a.d / 16 ? (a.d / 16 - 1 - c.rank) / kClCTAs + 1 : 0;
    c.per_layer = 1 + c.ng * (2 * a.s_in + 1) + c.ng + c.nt;
    c.total = c.per_layer * a.nl;
    const int ns = c.ns, b0 = c.b0, d = a.d;
    char* ring = sm + a.lay.ring;
    float* xs = reinterpret_cast<float*>(sm + a.lay.xs);
    int8_t* bq = reinterpret_cast<int8_t*>(sm + a.lay.bq);
    float* ae = reinterpret_cast<float*>(sm + a.lay.ae);
    float* part = reinterpret_cast<float*>(sm + a.lay.part);
    float* co = reinterpret_cast<float*>(sm + a.lay.co);
    float* zl = reinterpret_cast<float*>(sm + a.lay.zl);
    float* rchain = reinterpret_cast<float*>(sm + a.lay.rchain);
    float* xc = reinterpret_cast<float*>(sm + a.lay.xc);
    float* zs = reinterpret_cast<float*>(sm + a.lay.zs);
    int8_t* gq = reinterpret_cast<int8_t*>(sm + a.lay.gq);
    float* ge = reinterpret_cast<float*>(sm + a.lay.ge);
    float* xn = reinterpret_cast<float*>(sm + a.lay.xn);
    FusedLayer* lt = reinterpret_cast<FusedLayer*>(sm + a.lay.layers);

    // ---- set-up: stream metadata, zeroed exchange buffers, residual rows, the first copies ----
    if (tid < ns) {
        meta.slot[tid] = a.slots[b0 + tid];
        meta.fresh[tid] = a.rflag[b0 + tid];
    }
    for (int i = tid; i < (a.lay.layers - a.lay.bq) / 16; i += kClThreads)
        reinterpret_cast<uint4*>(sm + a.lay.bq)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < a.nl; i += kClThreads) lt[i] = a.layers[i];
    for (int i = tid; i < kClMaxNS * d; i += kClThreads) {
        const int s = i / d;
        xs[i] = s < ns ? __ldcg(a.x + (size_t)(b0 + s) * d + (i - s * d)) : 0.0f;
    }
    if (tid == 0) {
        for (int i = 0; i < kClItems; i++) tc::mbar_init(&R.bar[i], 1);
        R.head = R.tail = 0;
        R.issued = R.released = 0;
        R.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (tid < 32) cl_refill(a, c, meta, lt, R, ring);
    cl_sync();  // every CTA of the cluster is set up before any exchange writes into it

    const int G_out = a.g_out, xr = a.xr;
    const int per_g = 2 * a.s_in + 1;
    for (int l = 0; l < a.nl; l++) {
        int k = l * c.per_layer;
        // ---- A: norm of every stream into digit planes (warp w: stream w) ----
        cl_wait_items(a, c, meta, lt, R, ring, k, k + 1);
        {
            const FusedLayer& L = lt[l];
            const float* nws = reinterpret_cast<const float*>(cl_ptr(R, ring, k));
            if (warp < ns) {
                NormWeights<NC> nw;
#pragma unroll
                for (int cc = 0; cc < NC; cc++) {
                    const int kk = cc * 128 + lane * 4;
                    nw.w[cc] = kk < d ? *reinterpret_cast<const float4*>(nws + kk) : make_float4(0.f, 0.f, 0.f, 0.f);
                    nw.b[cc] = (L.norm_b && kk < d) ? *reinterpret_cast<const float4*>(nws + d + kk)
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                float4 v[NC];
#pragma unroll
                for (int cc = 0; cc < NC; cc++) {
                    const int kk = cc * 128 + lane * 4;
                    v[cc] = kk < d ? *reinterpret_cast<const float4*>(xs + warp * d + kk) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                norm_apply<NC>(v, d, nw, L.norm_b != nullptr, lane);
                int8_t* rows = bq + warp * a.pitch_a;  // plane p at + p * 8 * pitch
                norm_emit_q<NC>(v, d, lane, [&](int kk, int p1, int p2, int p3, float gs, bool lead) {
                    *reinterpret_cast<int*>(rows + kk) = p1;
                    *reinterpret_cast<int*>(rows + 8 * a.pitch_a + kk) = p2;
                    *reinterpret_cast<int*>(rows + 16 * a.pitch_a + kk) = p3;
                    if (lead) ae[warp * kEStride + kk / kGroup] = gs;
                });
            }
        }
        __syncthreads();
        cl_release(a, c, meta, lt, R, ring, k + 1);
        k += 1;
        // ---- A: the owned groups' in_proj jobs ----
        for (int gi = 0; gi < c.ng; gi++) {
            const int g = cl_group(c, gi);
            const int kx = k + gi * per_g;
            // x half: MMA, then conv/SiLU + conv state + x_proj chains
            cl_wait_items(a, c, meta, lt, R, ring, kx, kx + a.s_in);
            cl_job_mma(a, R, ring, sm, kx);
            __syncthreads();
            cl_release(a, c, meta, lt, R, ring, kx + a.s_in);
            cl_wait_items(a, c, meta, lt, R, ring, kx + a.s_in, kx + a.s_in + 1);
            {
                const char* xe = cl_ptr(R, ring, kx + a.s_in);
                const float* xw = reinterpret_cast<const float*>(xe);
                const float* ct = reinterpret_cast<const float*>(xe + align16(xr * 68 * 4));
                const float* cv = reinterpret_cast<const float*>(xe + align16(xr * 68 * 4) + align16(5 * 64 * 4));
                for (int o = tid; o < ns * 64; o += kClThreads) {
                    const int rl = o & 63, s = o >> 6, j = g * 64 + rl;
                    const float tot = sum_splits(part + (size_t)(rl >> 4) * a.s_in * 128, a.s_in, (rl & 15) * 8 + s);
                    const uint32_t slot = meta.slot[s];
                    float cov = 0.0f;
                    if (slot < (uint32_t)a.cap) {
                        float s0 = 0.f, s1 = 0.f, s2 = 0.f;
                        if (!meta.fresh[s]) {
                            s0 = cv[(s * 3 + 0) * 64 + rl];
                            s1 = cv[(s * 3 + 1) * 64 + rl];
                            s2 = cv[(s * 3 + 2) * 64 + rl];
                        }
                        float* st = a.conv + conv_off(l, a.cap, slot, a.di, 0, j);
                        st[0] = s1;
                        st[64] = s2;
                        st[128] = tot;
                        cov = conv_silu_taps(s0, s1, s2, tot, ct[rl], ct[64 + rl], ct[128 + rl], ct[192 + rl], ct[256 + rl]);
                    }
                    co[(gi * kClMaxNS + s) * 64 + rl] = cov;
                    xc[s * 68 + rl] = cov;
                }
                __syncthreads();
                // x_proj chains of the group (xproj_chain order: channels 0..63 from zero), in
                // register blocks of 2 rows x 4 streams; each chain goes to its stream's owner CTA
                const int nsb = (ns + 3) >> 2, nblk = ((xr + 1) >> 1) * nsb;
                for (int t = tid; t < nblk; t += kClThreads) {
                    const int r0 = (t / nsb) * 2, s0 = (t % nsb) * 4;
                    const float* w0 = xw + r0 * 68;
                    const float* w1 = xw + min(r0 + 1, xr - 1) * 68;
                    const float* xsr[4];
#pragma unroll
                    for (int jj = 0; jj < 4; jj++) xsr[jj] = xc + min(s0 + jj, ns - 1) * 68;
                    float acc[2][4];
#pragma unroll
                    for (int i = 0; i < 2; i++)
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) acc[i][jj] = 0.0f;
#pragma unroll 4
                    for (int cc = 0; cc < 64; cc += 4) {
                        const float4 wa = *reinterpret_cast<const float4*>(w0 + cc);
                        const float4 wb = *reinterpret_cast<const float4*>(w1 + cc);
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) {
                            const float4 xv = *reinterpret_cast<const float4*>(xsr[jj] + cc);
                            acc[0][jj] = __fmaf_rn(wa.x, xv.x, acc[0][jj]);
                            acc[0][jj] = __fmaf_rn(wa.y, xv.y, acc[0][jj]);
                            acc[0][jj] = __fmaf_rn(wa.z, xv.z, acc[0][jj]);
                            acc[0][jj] = __fmaf_rn(wa.w, xv.w, acc[0][jj]);
                            acc[1][jj] = __fmaf_rn(wb.x, xv.x, acc[1][jj]);
                            acc[1][jj] = __fmaf_rn(wb.y, xv.y, acc[1][jj]);
                            acc[1][jj] = __fmaf_rn(wb.z, xv.z, acc[1][jj]);
                            acc[1][jj] = __fmaf_rn(wb.w, xv.w, acc[1][jj]);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 2; i++)
#pragma unroll
                        for (int jj = 0; jj < 4; jj++)
                            if (r0 + i < xr && s0 + jj < ns)
                                cl_st(cl_map(rchain + g * xr + r0 + i, (uint32_t)(s0 + jj)), acc[i][jj]);
                }
            }
            __syncthreads();
            cl_release(a, c, meta, lt, R, ring, kx + a.s_in + 1);
            // z half: MMA, then z kept locally
            const int kz = kx + a.s_in + 1;
            cl_wait_items(a, c, meta, lt, R, ring, kz, kz + a.s_in);
            cl_job_mma(a, R, ring, sm, kz);
            __syncthreads();
            for (int o = tid; o < ns * 64; o += kClThreads) {
                const int rl = o & 63, s = o >> 6;
                zl[(gi * kClMaxNS + s) * 64 + rl] =
                    sum_splits(part + (size_t)(rl >> 4) * a.s_in * 128, a.s_in, (rl & 15) * 8 + s);
            }
            __syncthreads();
            cl_release(a, c, meta, lt, R, ring, kz + a.s_in);
        }
        k += c.ng * per_g;
        cl_sync();
        // ---- A2: stream owners add their chains in group order and send the sums everywhere ----
        if (c.rank < ns && tid < xr / 4) {
            const float4* cp = reinterpret_cast<const float4*>(rchain) + tid;
            float4 t = cp[0];
            for (int q = 1; q < G_out; q++) {
                const float4 v = cp[(size_t)q * (xr / 4)];
                t.x = __fadd_rn(t.x, v.x);
                t.y = __fadd_rn(t.y, v.y);
                t.z = __fadd_rn(t.z, v.z);
                t.w = __fadd_rn(t.w, v.w);
            }
            float* dst = zs + c.rank * xr + tid * 4;
            for (int r = 0; r < kClCTAs; r++) cl_st4(cl_map(dst, (uint32_t)r), t);
        }
        cl_sync();
        // ---- B: scan of the owned groups; their out_proj digit planes go to every CTA ----
        for (int gi = 0; gi < c.ng; gi++) {
            const int g = cl_group(c, gi);
            const int kb = k + gi;
            cl_wait_items(a, c, meta, lt, R, ring, kb, kb + 1);
            const char* sbi = cl_ptr(R, ring, kb);
            const float* sb = reinterpret_cast<const float*>(sbi);  // [dr + 18][64]
            const float* pst = reinterpret_cast<const float*>(sbi + align16((a.dr + 18) * 64 * 4));  // [ns][16][64]
            const int ch = tid & 63, sl = tid >> 6, j = g * 64 + ch;
            const float* dtw = sb;
            const float* at = sb + a.dr * 64;
            const float dtb = sb[(a.dr + 16) * 64 + ch], dv = sb[(a.dr + 17) * 64 + ch];
            const int body = a.dr & ~7;
            for (int pass = 0; pass < (ns + 3) / 4; pass++) {
                const int s = sl + 4 * pass;
                const bool valid = s < ns;
                bool ok = false;
                float gated = 0.0f;
                if (valid) {
                    const uint32_t slot = meta.slot[s];
                    ok = slot < (uint32_t)a.cap;
                    const bool fresh = meta.fresh[s] != 0;
                    float st[kDState];
#pragma unroll
                    for (int kk = 0; kk < kDState; kk++) st[kk] = (ok && !fresh) ? pst[(s * kDState + kk) * 64 + ch] : 0.0f;
                    const float xv = co[(gi * kClMaxNS + s) * 64 + ch];
                    const float zv = zl[(gi * kClMaxNS + s) * 64 + ch];
                    const float* zb = zs + s * xr;
                    float dt = dt_dot8_body(zb, body, [&](int cc) { return dtw[cc * 64 + ch]; });
                    for (int cc = body; cc < a.dr; cc++) dt = __fadd_rn(dt, __fmul_rn(dtw[cc * 64 + ch], zb[cc]));
                    dt = softplus(__fadd_rn(dt, dtb));
                    const float* B = zb + a.dr;
                    const float* C = zb + a.dr + kDState;
                    const bool update = !(fabsf(dt) < 1e-6f);
                    if (update) {
                        const float dtx = __fmul_rn(dt, xv);
#pragma unroll
                        for (int kk = 0; kk < kDState; kk++) {
                            const float da = lane_expf(__fsub_rn(0.0f, __fmul_rn(dt, at[kk * 64 + ch])));
                            st[kk] = __fadd_rn(__fmul_rn(da, st[kk]), __fmul_rn(dtx, B[kk]));
                        }
                    }
                    if (ok && (update || fresh)) {
                        float* sp = a.ssm + ssm_off(l, a.cap, slot, a.di, 0, j);
#pragma unroll
                        for (int kk = 0; kk < kDState; kk++) sp[kk * 64] = st[kk];
                    }
                    const float y = __fadd_rn(ssm_out16(st, C), __fmul_rn(dv, xv));
                    gated = ok ? __fmul_rn(y, __fmul_rn(zv, lane_sigmoid(zv))) : 0.0f;
                }
                // digit planes over the stream's 64 channels (warps 2q, 2q + 1)
                float mx = warp_allmax(fabsf(gated));
                if (lane == 0) s_max[pass & 1][warp] = mx;
                __syncthreads();
                mx = fmaxf(s_max[pass & 1][warp & ~1], s_max[pass & 1][warp | 1]);
                if (valid) {
                    float ginv, gs = group_scale(mx, &ginv);
                    const Digits3 dg = split_digits(gated, ginv);
                    const int sw = ((((ch >> 4) ^ ((s >> 1) & 3)) << 4) | (ch & 15)) + s * 64;
                    gq[(g * 3 + 0) * 512 + sw] = (int8_t)dg.d1;
                    gq[(g * 3 + 1) * 512 + sw] = (int8_t)dg.d2;
                    gq[(g * 3 + 2) * 512 + sw] = (int8_t)dg.d3;
                    if (ch == 0) ge[s * kEStride + g] = gs;
                }
            }
            __syncthreads();
            cl_release(a, c, meta, lt, R, ring, kb + 1);
        }
        // the owned groups' planes (3 x 8 rows x 64 B) and exponents to the other CTAs
        for (int gi = 0; gi < c.ng; gi++) {
            const int g = cl_group(c, gi);
            const uint4* src = reinterpret_cast<const uint4*>(gq + g * 1536);
            for (int i = tid; i < 96 * (kClCTAs - 1); i += kClThreads) {
                const int q = i / 96, ci = i - q * 96;
                const uint32_t r = (uint32_t)(q < c.rank ? q : q + 1);
                cl_st16(cl_map(src + ci, r), src[ci]);
            }
            for (int i = tid; i < ns * (kClCTAs - 1); i += kClThreads) {
                const int q = i / ns, s = i - q * ns;
                const uint32_t r = (uint32_t)(q < c.rank ? q : q + 1);
                cl_st(cl_map(ge + s * kEStride + g, r), ge[s * kEStride + g]);
            }
        }
        k += c.ng;
        cl_sync();
        // ---- C: out_proj + residual of the owned 16-row tiles; new rows go to every CTA ----
        {
            const int gid = lane >> 2, tig = lane & 3;
            const uint32_t bsw = ((uint32_t)gid >> 1) & 3u;
            const int8_t* brow = gq + gid * 64 + tig * 4;
            for (int ti = 0; ti < c.nt; ti++) {  // one tile at a time: its item, its splits over the warps
                cl_wait_items(a, c, meta, lt, R, ring, k + ti, k + ti + 1);
                const char* cw = cl_ptr(R, ring, k + ti);
                float* pt = part + (size_t)ti * a.s_out * 128;
                for (int sp = warp; sp < a.s_out; sp += kClThreads / 32) {
                    const int g0 = G_out * sp / a.s_out, g1 = G_out * (sp + 1) / a.s_out;
                    float acc[4];
                    q8_tile16_split(reinterpret_cast<const int8_t*>(cw), 16, 0,  // the item holds every group
                                    reinterpret_cast<const float*>(cw + G_out * 1024), G_out, g0, g1,
                                    [&](int p, int g, int cc) {
                                        return *reinterpret_cast<const uint32_t*>(brow + (g * 3 + p) * 512 +
                                                                                  ((cc ^ bsw) << 4));
                                    },
                                    ge, lane, acc);
                    store_split(pt + (size_t)sp * 128, lane, acc);
                }
                __syncthreads();
                cl_release(a, c, meta, lt, R, ring, k + ti + 1);
                if (tid < 128) {  // residual: (row rr, stream s) of the tile
                    const int rr = tid >> 3, s = tid & 7;
                    if (s < ns) {
                        const int row = cl_tile(c, ti) * 16 + rr;
                        const float tot = sum_splits(pt, a.s_out, rr * 8 + s);
                        xn[(ti * kClMaxNS + s) * 16 + rr] = __fadd_rn(xs[s * d + row], tot);
                    }
                }
            }
            __syncthreads();
            for (int i = tid; i < c.nt * ns * 4 * kClCTAs; i += kClThreads) {
                const int r = i / (c.nt * ns * 4), q = i - r * (c.nt * ns * 4);
                const int ti = q / (ns * 4), s = (q >> 2) % ns, f = q & 3;
                const float4 v = *reinterpret_cast<const float4*>(xn + (ti * kClMaxNS + s) * 16 + f * 4);
                cl_st4(cl_map(xs + s * d + cl_tile(c, ti) * 16 + f * 4, (uint32_t)r), v);
            }
        }
        cl_sync();
    }
    // ---- final norm (CTA 0): the head's digit planes; a rejected stream's are zeros ----
    if (c.rank == 0 && warp < ns) {
        NormWeights<NC> nw;
        nw.load(a.norm_f_w, a.norm_f_b, d, lane);
        float4 v[NC];
#pragma unroll
        for (int cc = 0; cc < NC; cc++) {
            const int kk = cc * 128 + lane * 4;
            v[cc] = kk < d ? *reinterpret_cast<const float4*>(xs + warp * d + kk) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        norm_apply<NC>(v, d, nw, a.norm_f_b != nullptr, lane);
        zero_if_rejected<NC>(v, meta.slot[warp] == kRejected);
        const ActOut out{nullptr, a.act_q, a.act_e, a.cap_pad, d};
        norm_emit<NC>(b0 + warp, v, d, out, lane);
    }
    // copies still in flight after an abort land before the CTA's shared memory goes away
    if (tid == 0)
        for (int kk = R.released; kk < R.issued; kk++) cl_wait_one(R, kk);
    __syncthreads();
}

}  // namespace rk
