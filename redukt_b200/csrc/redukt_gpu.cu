// libredukt_gpu.so: the C-ABI of include/redukt_gpu.h over the sm_100a decode-step kernels.
//
// Host side of the engine: .rbin loading (with Q8 quantisation on the device), the slot pool,
// argument validation with the reference's error behaviour, the launch sequence of one step
// and CUDA-graph replay of that sequence per batch size.  The reference counterpart is
// plugins/redukt-gpu-cuda/mamba_cuda.cu:385-761.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "../../include/redukt_gpu.h"
#include "rk_kernels.cuh"
#include "rk_fused.cuh"
#include "rk_rwkv7.cuh"
#include "rk_tc.cuh"
#include "rk_cdf.cuh"

namespace {

using namespace rk;

constexpr uint32_t kRbinMagic = 0x55504752u;
constexpr uint32_t kFlagNormBias = 1u << 0;
constexpr uint32_t kFlagUntiedHead = 1u << 1;
constexpr uint32_t kFlagQ8 = 1u << 2;
constexpr uint32_t kFlagQ8PerRow = 1u << 3;
constexpr uint32_t kFlagQ8Payload = 1u << 6;  // Q8 matrices stored as int8 + group scales (no quantise at load)
constexpr uint32_t kMaxStreams = 4096u;  // batch_init cap (mamba_cuda.cu:55)

enum Profile { kF32 = 0, kQ8 = 1, kQ8Row = 2 };

char g_err[1024] = "";

void set_err(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    fprintf(stderr, "[redukt-b200] %s\n", g_err);
}

#define CK(call, code)                                                                        \
    do {                                                                                      \
        cudaError_t e_ = (call);                                                              \
        if (e_ != cudaSuccess) {                                                              \
            set_err("CUDA error %s at %s:%d (%s)", cudaGetErrorString(e_), __FILE__, __LINE__, #call); \
            return (code);                                                                    \
        }                                                                                     \
    } while (0)

struct RbinHeader {
    uint32_t magic, version, vocab, d, di, ds, dc, dr, nl, flags, tokenizer;
};

// A projection matrix in the active profile.
struct Mat {
    int rows = 0, cols = 0;
    float* f = nullptr;    // F32 [rows][cols]
    int8_t* q = nullptr;   // Q8, tiled [cols/64][rows rounded up to 128][64 B] (rk_math.cuh)
    float* s = nullptr;    // Q8 scales [rows][cols/64]
};

struct Layer {
    float* norm_w = nullptr;
    float* norm_b = nullptr;
    Mat in_proj, out_proj;
    float* conv_t = nullptr;   // [4][di]
    float* conv_b = nullptr;
    float* x_proj = nullptr;   // [xr][di]
    float* dt_wt = nullptr;    // [dr][di] (transposed)
    float* dt_b = nullptr;
    float* a_t = nullptr;      // [16][di] = lane_exp(A_log)
    float* dvec = nullptr;
};

struct Pool {
    uint32_t cap = 0;
    float* conv = nullptr;       // [L][cap][3][di]
    float* ssm = nullptr;        // [L][cap][16][di]
    uint32_t* since = nullptr;   // [cap]
    // per-step scratch, indexed by batch position
    float* x = nullptr;          // [cap][d]
    float* act_f = nullptr;      // [cap][di] f32 activations (F32 profile)
    int8_t* act_q = nullptr;     // tiled digit planes [di/64][3][cap_pad][64] (Q8)
    int cap_pad = 0;             // cap rounded up to 64
    float* act_e = nullptr;      // [cap][kEStride]
    float* conv_out = nullptr;   // [cap][di]
    float* z = nullptr;          // [cap][di]
    float* logits = nullptr;     // [cap][V]
    float* red = nullptr;        // [cap][softmax partial slots] (max, sum) pairs
    float* xpart = nullptr;      // x_proj group chains [cap][di/64][xr] (k_xproj_part, fused step)
    float* zp = nullptr;         // [cap][xr] x_proj output (dt_raw, B, C)
    uint32_t* xcount = nullptr;  // [cap/16] k_xproj_part arrival counters (self-resetting)
    uint32_t* bar = nullptr;     // fused step: grid-barrier counter
    float* part = nullptr;       // split-K split sums [tiles][S][128][16] (Q8, up to 64 streams)
    size_t part_cap = 0;         // floats in `part`
    uint32_t* counter = nullptr; // split-K tile counters
    uint32_t* rflag = nullptr;   // [cap]
    uint32_t* vslot = nullptr;   // [cap] validated slot per batch position (k_embed; kRejected = bad entry)
    uint32_t* d_slots = nullptr;
    uint32_t* d_tokens = nullptr;
    uint32_t* h_slots = nullptr;   // pinned
    uint32_t* h_tokens = nullptr;  // pinned
    uint32_t* h_err = nullptr;     // pinned copy of the device error word
    std::vector<uint8_t> seen;
    std::map<uint64_t, cudaGraphExec_t> graphs;  // captured launch sequences, see graph_key()
    std::set<uint64_t> eager_done;                 // keys already run once without a graph
};

struct Model {
    RbinHeader h{};
    Profile profile = kF32;
    int V = 0, d = 0, di = 0, dr = 0, xr = 0, nl = 0;
    Mat emb, head;
    bool head_tied = true;
    float* norm_f_w = nullptr;
    float* norm_f_b = nullptr;
    std::vector<Layer> layers;
    std::vector<void*> allocs;
    cudaStream_t stream = nullptr;
    int device = 0;
    Pool v1, batch;
    uint32_t reset_every = 0;
    uint32_t* d_err = nullptr;
    int proj_path = 0;     // 0 auto, 1 CUDA cores, 2 tensor cores
    bool use_graphs = true;
    bool use_pdl = true;   // programmatic dependent launch between the step's kernels
    bool rwkv = false;     // an RWKV-7 model is loaded (rwkv7_engine.cuh) instead of Mamba
    bool ready = false;
    // fused small-batch step (rk_fused.cuh)
    bool fused = true;          // option "fused"
    bool scan_blk = true;       // option "scan_blk": stream-blocked scan above 64 streams
    bool f32_pairs = true;      // option "f32_pairs": F32 GEMV from 8 streams on as k_gemv_f32_p
    bool conv_defer = true;     // option "conv_defer": conv1d + SiLU in the x_proj kernel's staging
                                //   pass (1) or in the in_proj epilogue (0); the same bits
    int large_tile = 0;         // option "large_tile": above 256 streams, 0 = 64-stream tensor-core
                                //   tiles (one CTA per SM), 1 = 32-stream tiles, two CTAs per SM
    int fused_nc = 0;           // norm chunks of the instantiated kernel, 0 = shape not supported
    int head_ctas = 2;          // option "head_ctas": 2 = the two-CTAs-per-SM head tiles at small batch
    bool head_wide = true;      // option "head_wide": above 16 streams, 32-stream head tiles two per SM
    bool q8_payload = false;    // the loaded file stores its Q8 matrices quantised (flag bit 6)
    int num_sms = 0;
    FusedLayer* d_fused = nullptr;  // [nl] device copy of the layer pointers
};

Model G;
bool prepare_fused();

// ------------------------------------------------------------------------------------------
// Allocation helpers
// ------------------------------------------------------------------------------------------

template <class T>
bool dalloc(T** p, size_t count, bool zero = true) {
    *p = nullptr;
    if (count == 0) count = 1;
    if (cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)) != cudaSuccess) {
        *p = nullptr;
        return false;
    }
    if (zero && cudaMemset(*p, 0, count * sizeof(T)) != cudaSuccess) return false;
    return true;
}

template <class T>
bool model_alloc(T** p, size_t count) {
    if (!dalloc(p, count)) return false;
    G.allocs.push_back(*p);
    return true;
}

void pool_free(Pool* p) {
    for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
    p->graphs.clear();
    p->eager_done.clear();
    void* bufs[] = {p->conv, p->ssm, p->since, p->x, p->act_f, p->act_q, p->act_e, p->conv_out, p->z,
                    p->logits, p->red, p->part, p->counter, p->rflag, p->vslot, p->d_slots, p->d_tokens,
                    p->xpart, p->bar, p->zp, p->xcount};
    for (void* b : bufs) cudaFree(b);
    if (p->h_slots) cudaFreeHost(p->h_slots);
    if (p->h_tokens) cudaFreeHost(p->h_tokens);
    if (p->h_err) cudaFreeHost(p->h_err);
    *p = Pool();
}

constexpr int kSoftmaxTile = 2048;  // logits per partial (max, sum) of the probability pass
constexpr int kSplitMaxTiles = 1024;    // split-K tile counters
constexpr int kSplitMaxN = 256;         // split launches use the 16-stream tile (n <= 256)
int g_split_target = 148;               // CTAs a split launch may use (one wave on 148 SMs)

size_t split_part_floats(int rows, int groups, int n) {
    const size_t tiles = (size_t)((rows + tc::kBM - 1) / tc::kBM) * ((n + 15) / 16);
    return tiles * q8_splits(groups) * tc::kBM * 16;
}


bool pool_alloc(Pool* p, uint32_t cap) {
    *p = Pool();
    p->cap = cap;
    size_t n = cap, L = G.nl, d = G.d, di = G.di, V = G.V;
    size_t parts = std::max((V + kSoftmaxTile - 1) / kSoftmaxTile, (V + tc::kBM - 1) / tc::kBM);  // softmax partials
    const size_t dib = (size_t)state_blocks((int)di) * 64;  // d_inner in whole 64-channel blocks
    bool ok = dalloc(&p->conv, L * n * (kDConv - 1) * di) && dalloc(&p->ssm, L * n * kDState * dib) &&
              dalloc(&p->since, n) && dalloc(&p->x, n * d) && dalloc(&p->conv_out, n * di) &&
              dalloc(&p->z, n * di) && dalloc(&p->xpart, n * ((di + 63) / 64) * G.xr) && dalloc(&p->zp, n * G.xr) &&
              dalloc(&p->xcount, (n + 15) / 16) && dalloc(&p->logits, n * V) &&
              dalloc(&p->red, n * parts * 2) && dalloc(&p->rflag, n) && dalloc(&p->vslot, n) && dalloc(&p->d_slots, n) &&
              dalloc(&p->d_tokens, n);
    if (ok) {
        if (G.profile == kF32) ok = dalloc(&p->act_f, n * di);
        else {
            p->cap_pad = round_up((int)cap, 64);
            ok = dalloc(&p->act_q, 3 * (size_t)p->cap_pad * di) && dalloc(&p->act_e, n * kEStride);
            // split-K scratch for the layer projections (the head's many tiles never split)
            const int nn = (int)std::min<size_t>(n, kSplitMaxN);
            p->part_cap = std::max(split_part_floats(2 * (int)di, (int)d / kGroup, nn),
                                   split_part_floats((int)d, (int)di / kGroup, nn));
            ok = ok && dalloc(&p->part, p->part_cap, false) && dalloc(&p->counter, kSplitMaxTiles);
            ok = ok && dalloc(&p->bar, 1);
        }
    }
    if (ok) ok = cudaHostAlloc(reinterpret_cast<void**>(&p->h_slots), n * sizeof(uint32_t), cudaHostAllocDefault) ==
                 cudaSuccess;
    if (ok) ok = cudaHostAlloc(reinterpret_cast<void**>(&p->h_tokens), n * sizeof(uint32_t), cudaHostAllocDefault) ==
                 cudaSuccess;
    if (ok) ok = cudaHostAlloc(reinterpret_cast<void**>(&p->h_err), sizeof(uint32_t), cudaHostAllocDefault) == cudaSuccess;

    p->seen.assign(n, 0);
    if (!ok) {
        pool_free(p);
        return false;
    }
    return true;
}

void clear_dev_graphs();
namespace rwe {
void clear_graphs();
void release();
}  // namespace rwe

void free_model() {
    if (G.stream) cudaStreamSynchronize(G.stream);
    clear_dev_graphs();
    rwe::clear_graphs();
    rwe::release();
    pool_free(&G.v1);
    pool_free(&G.batch);
    for (void* a : G.allocs) cudaFree(a);
    if (G.d_err) cudaFree(G.d_err);
    if (G.stream) cudaStreamDestroy(G.stream);
    G.~Model();
    new (&G) Model();
}

// ------------------------------------------------------------------------------------------
// Weight loading
// ------------------------------------------------------------------------------------------

struct Reader {
    FILE* f = nullptr;
    float* staging = nullptr;  // pinned
    size_t staging_n = 0;
    ~Reader() {
        if (f) fclose(f);
        if (staging) cudaFreeHost(staging);
    }
    // Reads `bytes` bytes into the device buffer `dst`.
    bool read_bytes(void* dst, size_t bytes) {
        const size_t cap = staging_n * sizeof(float);
        size_t done = 0;
        while (done < bytes) {
            size_t chunk = std::min(cap, bytes - done);
            if (fread(staging, 1, chunk, f) != chunk) return false;
            if (cudaMemcpy(static_cast<char*>(dst) + done, staging, chunk, cudaMemcpyHostToDevice) != cudaSuccess)
                return false;
            done += chunk;
        }
        return true;
    }
    // Reads `count` floats into the device buffer `dst`.
    bool read_to(float* dst, size_t count) {
        size_t done = 0;
        while (done < count) {
            size_t chunk = std::min(staging_n, count - done);
            if (fread(staging, sizeof(float), chunk, f) != chunk) return false;
            if (cudaMemcpy(dst + done, staging, chunk * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
                return false;
            done += chunk;
        }
        return true;
    }
};

float* g_tmp = nullptr;  // load-time f32 staging on the device (largest matrix)

bool load_f32(Reader& r, float** dst, size_t count) { return model_alloc(dst, count) && r.read_to(*dst, count); }

// Loads a [rows][cols] matrix in the active profile.  Q8: quantised on the device with the
// reference recipe (group 64, or per-row then broadcast to the 64-column groups).
bool load_mat(Reader& r, Mat* m, int rows, int cols, bool quantise) {
    m->rows = rows;
    m->cols = cols;
    size_t count = (size_t)rows * cols;
    if (!quantise || G.profile == kF32) return load_f32(r, &m->f, count);
    int groups = cols / kGroup;
    const int rows_pad = round_up(rows, tc::kBM);
    int8_t* q_rm = nullptr;  // row-major quantised copy, then tiled
    if (!dalloc(&q_rm, count, false)) return false;
    if (!model_alloc(&m->q, (size_t)rows_pad * cols) || !model_alloc(&m->s, (size_t)rows * groups)) {
        cudaFree(q_rm);
        return false;
    }
    if (G.q8_payload) {  // stored quantised: int8 [rows][cols], then f32 scales [rows][groups]
        if (!r.read_bytes(q_rm, count) || !r.read_to(m->s, (size_t)rows * groups)) {
            cudaFree(q_rm);
            return false;
        }
    } else if (!r.read_to(g_tmp, count)) {
        cudaFree(q_rm);
        return false;
    } else if (G.profile == kQ8) {
        size_t ng = count / kGroup;
        k_quantize_q8<<<(unsigned)((ng + 7) / 8), 256>>>(g_tmp, ng, kGroup, q_rm, m->s);
    } else {
        float* row_s = nullptr;
        if (!dalloc(&row_s, (size_t)rows)) {
            cudaFree(q_rm);
            return false;
        }
        k_quantize_q8<<<(unsigned)((rows + 7) / 8), 256>>>(g_tmp, (size_t)rows, cols, q_rm, row_s);
        size_t tot = (size_t)rows * groups;
        k_broadcast_scales<<<(unsigned)((tot + 255) / 256), 256>>>(row_s, rows, groups, m->s);
        cudaDeviceSynchronize();
        cudaFree(row_s);
    }
    size_t chunks = count / 16;
    k_tile_q8<<<(unsigned)((chunks + 255) / 256), 256>>>(q_rm, rows, cols, rows_pad, m->q);
    bool ok = cudaDeviceSynchronize() == cudaSuccess;
    cudaFree(q_rm);
    return ok;
}

int validate_header(const RbinHeader& h) {
    if (h.magic != kRbinMagic || (h.version != 1 && h.version != 2)) return -1;
    if (!h.vocab || !h.d || !h.di || !h.nl || !h.dr) return -1;
    if (h.version == 2 && h.tokenizer > 1) return -1;
    if (h.version == 2 && h.tokenizer == 0 && h.vocab != 256) return -1;
    // Engine limits: d_state 16 and d_conv 4 (every Mamba-1 checkpoint redukt ships), d_inner = 2 d,
    // d a multiple of 64 (Q8 groups, 128-column vector tiles), d_inner <= 2048, dt_rank <= 256.
    if (h.ds != (uint32_t)kDState || h.dc != (uint32_t)kDConv) return -2;
    if (h.di != 2 * h.d || h.d % 64 != 0 || h.di > 2048 || h.dr > 256) return -2;
    if (h.vocab >= (1u << 30)) return -2;
    return 0;
}

int load_weights(const char* path) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) {
        set_err("cannot open %s", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    RbinHeader h;
    if (fread(&h, sizeof(h), 1, r.f) != 1) {
        set_err("%s: short header", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    int v = validate_header(h);
    if (v == -1) {
        set_err("%s: bad .rbin header", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    if (v == -2) {
        set_err("%s: model shape outside engine limits (d_state=%u d_conv=%u d=%u di=%u dr=%u)", path, h.ds, h.dc,
                h.d, h.di, h.dr);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    G.h = h;
    G.V = (int)h.vocab;
    G.d = (int)h.d;
    G.di = (int)h.di;
    G.dr = (int)h.dr;
    G.xr = (int)(h.dr + 2 * h.ds);
    G.nl = (int)h.nl;
    G.profile = (h.flags & kFlagQ8) ? ((h.flags & kFlagQ8PerRow) ? kQ8Row : kQ8) : kF32;
    if (const char* e = getenv("REDUKT_B200_PROFILE")) {
        if (!strcmp(e, "f32")) G.profile = kF32;
        else if (!strcmp(e, "q8")) G.profile = kQ8;
        else if (!strcmp(e, "q8row")) G.profile = kQ8Row;
    }
    G.q8_payload = (h.flags & kFlagQ8Payload) != 0;
    if (G.q8_payload && G.profile != kQ8) {
        set_err("%s: a Q8 payload file holds group-64 int8 weights; it loads only as the Q8 (group 64) profile", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    // expected file size
    size_t d = G.d, di = G.di, V = G.V, xr = G.xr, dr = G.dr;
    bool nb = h.flags & kFlagNormBias, untied = h.flags & kFlagUntiedHead;
    size_t per_layer = d * (nb ? 2 : 1) + 2 * di * d + di * kDConv + di + xr * di + di * dr + di + di * kDState +
                       di + d * di;
    size_t total = V * d + G.nl * per_layer + d * (nb ? 2 : 1) + (untied ? V * d : 0);
    size_t body = total * 4;
    if (G.q8_payload) {  // the Q8 matrices take 1 byte a weight + 4 bytes a 64-column group
        const size_t q8_elems = V * d * (untied ? 2 : 1) + G.nl * (2 * di * d + d * di);
        body = (total - q8_elems) * 4 + q8_elems + q8_elems / kGroup * 4;
    }
    fseek(r.f, 0, SEEK_END);
    long fsz = ftell(r.f);
    fseek(r.f, (long)sizeof(h), SEEK_SET);
    if (fsz < 0 || (size_t)fsz != sizeof(h) + body) {
        set_err("%s: size %ld does not match the header (%zu expected)", path, fsz, sizeof(h) + body);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    r.staging_n = (size_t)16 << 20;
    if (cudaHostAlloc(reinterpret_cast<void**>(&r.staging), r.staging_n * sizeof(float), cudaHostAllocDefault) !=
        cudaSuccess) {
        set_err("pinned staging allocation failed");
        return BACKEND_INIT_FAILED;
    }
    if (G.profile != kF32 && !dalloc(&g_tmp, std::max(V * d, 2 * di * d), false)) {
        set_err("device staging allocation failed");
        return BACKEND_INIT_FAILED;
    }
    bool ok = load_mat(r, &G.emb, G.V, G.d, true);
    float* a_log = nullptr;
    float* conv_w = nullptr;
    float* dt_w = nullptr;
    ok = ok && dalloc(&a_log, di * kDState, false) && dalloc(&conv_w, di * kDConv, false) &&
         dalloc(&dt_w, di * dr, false);
    G.layers.resize(G.nl);
    for (int i = 0; ok && i < G.nl; i++) {
        Layer& L = G.layers[i];
        ok = load_f32(r, &L.norm_w, d) && (!nb || load_f32(r, &L.norm_b, d)) &&
             load_mat(r, &L.in_proj, 2 * G.di, G.d, true) && r.read_to(conv_w, di * kDConv) &&
             load_f32(r, &L.conv_b, di) && load_f32(r, &L.x_proj, xr * di) && r.read_to(dt_w, di * dr) &&
             load_f32(r, &L.dt_b, di) && r.read_to(a_log, di * kDState) && load_f32(r, &L.dvec, di) &&
             load_mat(r, &L.out_proj, G.d, G.di, true);
        ok = ok && model_alloc(&L.a_t, di * kDState) && model_alloc(&L.conv_t, di * kDConv) &&
             model_alloc(&L.dt_wt, di * dr);
        if (ok) {
            k_prep_layer<<<(unsigned)((di + 255) / 256), 256>>>(a_log, conv_w, dt_w, G.di, G.dr, L.a_t, L.conv_t,
                                                                 L.dt_wt);
            ok = cudaDeviceSynchronize() == cudaSuccess;
        }
    }
    ok = ok && load_f32(r, &G.norm_f_w, d) && (!nb || load_f32(r, &G.norm_f_b, d));
    if (ok && G.profile != kF32) ok = prepare_fused();
    G.head_tied = !untied;
    if (ok && untied) ok = load_mat(r, &G.head, G.V, G.d, true);
    if (ok && !untied) G.head = G.emb;
    cudaFree(a_log);
    cudaFree(conv_w);
    cudaFree(dt_w);
    if (g_tmp) cudaFree(g_tmp);
    g_tmp = nullptr;
    if (!ok) {
        set_err("%s: reading/uploading weights failed (%s)", path, cudaGetErrorString(cudaGetLastError()));
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    return BACKEND_OK;
}

// The fused step's layer table and shape check (rk_fused.cuh).  Shapes it does not cover keep
// the per-kernel path: d and d_inner in whole 64-column groups, at most kEStride groups, and a
// norm width the kernel is instantiated for.
bool prepare_fused() {
    G.fused_nc = 0;
    const int nc = (G.d + 127) / 128;
    const bool shape_ok = G.d % 64 == 0 && G.di % 64 == 0 && G.d / 64 <= kEStride && G.di / 64 <= kEStride &&
                          (nc == 1 || nc == 2 || nc == 6 || nc == 8) && G.xr % 4 == 0 && 8 * G.xr <= 4 * kFusedThreads;
    std::vector<FusedLayer> h(G.nl);
    const int ng = G.di / 64, xr = G.xr, dr = G.dr;
    if (shape_ok) {
        // per-channel-group copies of the small per-layer operands, so the fused step fetches each
        // group's share with one contiguous copy: x_proj [ng][xr][68], conv taps + bias [ng][5][64],
        // dt_proj columns + A + dt bias + D [ng][dr + 18][64]
        for (int i = 0; i < G.nl; i++) {
            const Layer& L = G.layers[i];
            float *xw = nullptr, *ct = nullptr, *sb = nullptr;
            if (!model_alloc(&xw, (size_t)ng * xr * 68) || !model_alloc(&ct, (size_t)ng * 5 * 64) ||
                !model_alloc(&sb, (size_t)ng * (dr + 18) * 64))
                return false;
            bool ok = true;
            const size_t row = 64 * sizeof(float), src_pitch = (size_t)G.di * sizeof(float);
            for (int g = 0; ok && g < ng; g++) {
                const size_t c0 = (size_t)g * 64;
                ok = cudaMemcpy2D(xw + (size_t)g * xr * 68, 68 * sizeof(float), L.x_proj + c0, src_pitch, row, xr,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess &&
                     cudaMemcpy2D(ct + (size_t)g * 5 * 64, row, L.conv_t + c0, src_pitch, row, 4,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess &&
                     cudaMemcpy(ct + (size_t)g * 5 * 64 + 4 * 64, L.conv_b + c0, row, cudaMemcpyDeviceToDevice) ==
                         cudaSuccess &&
                     cudaMemcpy2D(sb + (size_t)g * (dr + 18) * 64, row, L.dt_wt + c0, src_pitch, row, dr,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess &&
                     cudaMemcpy2D(sb + ((size_t)g * (dr + 18) + dr) * 64, row, L.a_t + c0, src_pitch, row, kDState,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess &&
                     cudaMemcpy(sb + ((size_t)g * (dr + 18) + dr + 16) * 64, L.dt_b + c0, row,
                                cudaMemcpyDeviceToDevice) == cudaSuccess &&
                     cudaMemcpy(sb + ((size_t)g * (dr + 18) + dr + 17) * 64, L.dvec + c0, row,
                                cudaMemcpyDeviceToDevice) == cudaSuccess;
            }
            if (!ok) return false;
            // in_proj by 64-row block and out_proj by 16-row block, every group of a block adjacent,
            // so a fused-step job's weight tile is one contiguous copy per block
            int8_t *ib = nullptr, *ob = nullptr;
            const int gi = G.d / 64, go = G.di / 64;
            const size_t mi = (size_t)round_up(2 * G.di, 128), mo = (size_t)round_up(G.d, 128);
            if (!model_alloc(&ib, (size_t)2 * G.di * G.d) || !model_alloc(&ob, (size_t)G.d * G.di)) return false;
            for (int b = 0; ok && b < 2 * G.di / 64; b++)
                ok = cudaMemcpy2D(ib + (size_t)b * gi * 4096, 4096, L.in_proj.q + (size_t)b * 64 * 64, mi * 64, 4096, gi,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess;
            for (int b = 0; ok && b < G.d / 16; b++)
                ok = cudaMemcpy2D(ob + (size_t)b * go * 1024, 1024, L.out_proj.q + (size_t)b * 16 * 64, mo * 64, 1024, go,
                                  cudaMemcpyDeviceToDevice) == cudaSuccess;
            if (!ok) return false;
            h[i] = FusedLayer{L.norm_w, L.norm_b, L.in_proj.q, L.in_proj.s, L.out_proj.q, L.out_proj.s, xw, ct, sb,
                              ib, ob};
        }
    }
    if (!model_alloc(&G.d_fused, (size_t)G.nl)) return false;
    if (cudaMemcpy(G.d_fused, h.data(), h.size() * sizeof(FusedLayer), cudaMemcpyHostToDevice) != cudaSuccess) return false;
    cudaDeviceGetAttribute(&G.num_sms, cudaDevAttrMultiProcessorCount, G.device);
    if (shape_ok && G.num_sms > 0) G.fused_nc = nc;
    return true;
}

// ------------------------------------------------------------------------------------------
// Launch helpers
// ------------------------------------------------------------------------------------------

// Launches a step kernel; with PDL the kernel may start while its predecessor drains (every step
// kernel calls griddepcontrol.wait before touching data an earlier kernel wrote).
template <class... KArgs, class... Args>
void launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = G.use_pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <class Kern>
void allow_smem(Kern k, size_t bytes) {
    if (bytes > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

template <int RW, int NS, int NCH, class Epi>
void gemv_f32_nch(int M, int K, const float* W, const float* act, int ld, int n, Epi epi, cudaStream_t st) {
    size_t smem = (size_t)NS * K * sizeof(float);
    auto k = k_gemv_f32<RW, NS, NCH, Epi>;
    allow_smem(k, smem);
    dim3 grid((n + NS - 1) / NS, (M + 8 * RW - 1) / (8 * RW));
    launch(k, grid, dim3(256), smem, st, M, K, W, act, ld, n, epi);
}

// K <= 128 * NCH; the chunk loop is unrolled so every weight load of a row is issued at once.
template <int RW, int NS, class Epi>
void gemv_f32_ns(int M, int K, const float* W, const float* act, int ld, int n, Epi epi, cudaStream_t st) {
    if (RW > 1) {  // many rows per warp: a rolled chunk loop keeps the register count moderate
        gemv_f32_nch<RW, NS, 0>(M, K, W, act, ld, n, epi, st);
        return;
    }
    int nch = (K + 127) / 128;
    if (nch <= 1) gemv_f32_nch<RW, NS, 1>(M, K, W, act, ld, n, epi, st);
    else if (nch <= 2) gemv_f32_nch<RW, NS, 2>(M, K, W, act, ld, n, epi, st);
    else if (nch <= 6) gemv_f32_nch<RW, NS, 6>(M, K, W, act, ld, n, epi, st);
    else if (nch <= 12) gemv_f32_nch<RW, NS, 12>(M, K, W, act, ld, n, epi, st);
    else gemv_f32_nch<RW, NS, 16>(M, K, W, act, ld, n, epi, st);
}

template <int RW, class Epi>
void gemv_f32(int M, int K, const float* W, const float* act, int ld, int n, Epi epi, cudaStream_t st) {
    if (RW == 4 && n >= 8 && G.f32_pairs) {  // 4 rows x 8 streams per warp on the packed pipe (same bits)
        const size_t smem = (size_t)8 * ((K + 127) / 128) * 128 * sizeof(float);
        allow_smem(k_gemv_f32_p<Epi>, smem);
        launch(k_gemv_f32_p<Epi>, dim3((n + 7) / 8, (M + 31) / 32), dim3(256), smem, st, M, K, W, act, ld, n, epi);
        return;
    }
    if (n >= 8) gemv_f32_ns<RW, 8>(M, K, W, act, ld, n, epi, st);
    else if (n >= 4) gemv_f32_ns<RW, 4>(M, K, W, act, ld, n, epi, st);
    else if (n >= 2) gemv_f32_ns<RW, 2>(M, K, W, act, ld, n, epi, st);
    else gemv_f32_ns<RW, 1>(M, K, W, act, ld, n, epi, st);
}

// x_proj of every profile: group chains into p.xpart[b][g][r], summed in group order into p.zp.
// Above 512 streams, 64-stream tiles (the group's weights staged once per 64 streams, 4 x 8
// register blocks; below that they leave SMs idle); the chains and their group-order sums are the
// same either way.
// The in_proj epilogue of layer li: with conv_defer the x-branch is stored before the conv and
// launch_xproj runs conv1d + SiLU in its staging pass (same arithmetic, same bits).
EpiInProj in_proj_epi(const Layer& L, int li, const Pool& p, const uint32_t* vs) {
    EpiInProj e{G.di, (int)p.cap, li, vs, p.rflag, p.conv, L.conv_t, L.conv_b, p.conv_out, p.z};
    e.defer = G.conv_defer;
    return e;
}

void launch_xproj(const Layer& L, int li, const Pool& p, int n, const uint32_t* vs, cudaStream_t st) {
    const int ng = (G.di + kXGroup - 1) / kXGroup;
    XConv cv{G.conv_defer, (int)p.cap, li, vs, p.rflag, p.conv, L.conv_t, L.conv_b, p.conv_out};
    if (n > 512) {
        const size_t smem = ((size_t)G.xr * 68 + 64 * 68) * sizeof(float);
        allow_smem(k_xproj_part<64, 4, 8>, smem);
        launch(k_xproj_part<64, 4, 8>, dim3(ng, (n + 63) / 64), dim3(256), smem, st, G.xr, G.di, (const float*)L.x_proj,
               (const float*)p.conv_out, n, p.xpart, p.zp, p.xcount, cv);
        return;
    }
    const size_t smem = ((size_t)G.xr * 68 + 16 * 68) * sizeof(float);
    allow_smem(k_xproj_part<16, 2, 4>, smem);
    launch(k_xproj_part<16, 2, 4>, dim3(ng, (n + 15) / 16), dim3(256), smem, st, G.xr, G.di, (const float*)L.x_proj,
           (const float*)p.conv_out, n, p.xpart, p.zp, p.xcount, cv);
}

template <int NS, int GI, class Epi>
void gemv_q8_ns(const Mat& m, const int8_t* q, const float* e, int cap_pad, int n, Epi epi, cudaStream_t st) {
    constexpr int RW = 4;
    int K = m.cols;
    size_t smem = (size_t)NS * 3 * K + (size_t)NS * (K / kGroup) * sizeof(float);
    auto k = k_gemv_q8<RW, NS, GI, Epi>;
    allow_smem(k, smem);
    dim3 grid((n + NS - 1) / NS, (m.rows + 8 * RW - 1) / (8 * RW));
    launch(k, grid, dim3(256), smem, st, m.rows, K, (const int8_t*)m.q, (const float*)m.s, q, e, cap_pad, n, epi);
}

template <int GI, class Epi>
void gemv_q8_gi(const Mat& m, const int8_t* q, const float* e, int cap_pad, int n, Epi epi, cudaStream_t st) {
    if (n >= 8) gemv_q8_ns<8, GI>(m, q, e, cap_pad, n, epi, st);
    else if (n >= 4) gemv_q8_ns<4, GI>(m, q, e, cap_pad, n, epi, st);
    else if (n >= 2) gemv_q8_ns<2, GI>(m, q, e, cap_pad, n, epi, st);
    else gemv_q8_ns<1, GI>(m, q, e, cap_pad, n, epi, st);
}

template <class Epi>
void gemv_q8(const Mat& m, const int8_t* q, const float* e, int cap_pad, int n, Epi epi, cudaStream_t st) {
    int G8 = (m.cols / kGroup + 7) / 8;
    if (G8 <= 1) gemv_q8_gi<1>(m, q, e, cap_pad, n, epi, st);
    else if (G8 == 2) gemv_q8_gi<2>(m, q, e, cap_pad, n, epi, st);
    else if (G8 == 3) gemv_q8_gi<3>(m, q, e, cap_pad, n, epi, st);
    else gemv_q8_gi<4>(m, q, e, cap_pad, n, epi, st);
}

// Tensor cores for the Q8 projections once the batch makes them worthwhile (or when forced).
bool use_tc(int n) {
    if (G.profile == kF32 || G.proj_path == 1) return false;
    if (G.proj_path == 2) return true;
    return n >= tc::kAutoMinStreams;
}

// Split-K of a tensor-core projection: when a small batch leaves fewer (row, stream) tiles than
// g_split_target, each tile runs its q8_splits(G) accumulation splits in parallel CTAs.  The
// accumulation order is the same either way (q8_splits), so this is purely a latency choice.
// Split only while the split launch still fits one wave: the tile kernel runs one CTA per SM
// (registers and the TMEM guard), so tiles x S must stay within g_split_target (the SM count).
int split_for(int tiles, int rows, int groups, int n, size_t part_cap) {
    if (n > kSplitMaxN || tiles > kSplitMaxTiles) return 1;
    const int S = q8_splits(groups);
    if (S <= 1 || S > tc::kMaxGatherSplits || split_part_floats(rows, groups, n) > part_cap) return 1;
    for (int z = S; z > 1; z--)  // the most CTAs per tile that divide S and keep one wave
        if (S % z == 0 && (long)tiles * z <= g_split_target) return z;
    return 1;
}

template <int BN, class Epi, int ST = tc::stages_for<BN>(), int MB = 1>
void project_tc_bn(const Mat& m, const Pool& p, int n, Epi epi, cudaStream_t st) {
    auto k = tc::k_proj_q8_tc<BN, Epi, ST, MB>;
    size_t smem = tc::launch_smem<BN, ST>();
    allow_smem(k, smem);
    const int gx = (n + BN - 1) / BN, gy = (m.rows + tc::kBM - 1) / tc::kBM;
    tc::SplitK sk{1, p.part, p.counter};
    // the head's softmax partials need every CTA to hold its whole tile: never split it
    if (BN == 16 && p.part && !TileSoftmax<Epi>::value) sk.splits = split_for(gx * gy, m.rows, m.cols / kGroup, n, p.part_cap);
    dim3 grid(gx, gy, sk.splits);
    launch(k, grid, dim3(tc::TileCfg<BN, ST, MB>::kThreads), smem, st, (const int8_t*)m.q, (const int8_t*)p.act_q, m.rows, m.cols,
           p.cap_pad, n, (const float*)m.s, (const float*)p.act_e, G.d_err, epi, sk);
}

template <class Epi>
void project(const Mat& m, const Pool& p, int n, Epi epi, cudaStream_t st) {
    if (G.profile == kF32) {
        // below 8 streams, fewer rows per warp when 4 would leave the GPU short of CTAs (out_proj:
        // 24 CTAs at one stream); the per-(row, stream) arithmetic does not depend on it
        const long ct = (long)((n + 7) / 8) * ((m.rows + 31) / 32);
        if (n >= 8 || ct >= 2 * G.num_sms) gemv_f32<4>(m.rows, m.cols, m.f, p.act_f, m.cols, n, epi, st);
        else if (2 * ct >= 2 * G.num_sms) gemv_f32<2>(m.rows, m.cols, m.f, p.act_f, m.cols, n, epi, st);
        else gemv_f32<1>(m.rows, m.cols, m.f, p.act_f, m.cols, n, epi, st);
    } else if (use_tc(n)) {
        // narrow stream tiles at small n put more CTAs on the weights (re-reads hit L2)
        const int rt = (m.rows + tc::kBM - 1) / tc::kBM;
        if (n <= 64) {
            project_tc_bn<16>(m, p, n, epi, st);
        } else if (n <= 256) {
            // few row tiles (out_proj): 16-stream tiles whose K splits run in parallel CTAs, when
            // that fills the GPU better; else the narrowest tile that still fits one wave
            if (p.part && split_for(((n + 15) / 16) * rt, m.rows, m.cols / kGroup, n, p.part_cap) > 1)
                project_tc_bn<16>(m, p, n, epi, st);
            else if (((n + 31) / 32) * rt > G.num_sms && ((n + 63) / 64) * rt <= G.num_sms)
                project_tc_bn<64>(m, p, n, epi, st);
            else
                project_tc_bn<32>(m, p, n, epi, st);
        }
        else if (G.large_tile == 1) project_tc_bn<32, Epi, 6, 2>(m, p, n, epi, st);  // two CTAs per SM
        else project_tc_bn<64>(m, p, n, epi, st);
    } else {
        gemv_q8(m, p.act_q, p.act_e, p.cap_pad, n, epi, st);
    }
}

// The LM head: hundreds of row tiles, so at small batch a shallower pipeline (6 stages) that lets
// two CTAs share an SM (TMEM: 2 x 256 columns) keeps more tiles in flight than one deep CTA.
// Above 16 streams the head's hundreds of row tiles run as 32-stream tiles two CTAs per SM
// (option head_wide 1, default; 0: 16-stream tiles up to 64 streams, then the layer projections'
// tile choice), which keeps two tiles' epilogues and copies in flight per SM.
void project_head(const Pool& p, int n, float* out, cudaStream_t st) {
    const bool tc = G.profile != kF32 && use_tc(n);
    if (tc && n > 16 && G.head_wide)
        project_tc_bn<32, EpiStore, 6, 2>(G.head, p, n, EpiStore{out, G.V}, st);
    else if (tc && n <= 64 && G.head_ctas == 2)
        project_tc_bn<16, EpiStore, 6, 2>(G.head, p, n, EpiStore{out, G.V}, st);
    else
        project(G.head, p, n, EpiStore{out, G.V}, st);
}

// The head with the softmax partials of its 128-row tiles (EpiStoreSoftmax); the tile shapes are
// project_head's, so the logits are the same bits.
void project_head_softmax(const Pool& p, int n, float* out, int tiles, cudaStream_t st) {
    EpiStoreSoftmax e{};
    e.out = out;
    e.ld = G.V;
    e.red = p.red;
    e.parts = tiles;
    if (n > 16 && G.head_wide) project_tc_bn<32, EpiStoreSoftmax, 6, 2>(G.head, p, n, e, st);
    else if (n <= 64 && G.head_ctas == 2) project_tc_bn<16, EpiStoreSoftmax, 6, 2>(G.head, p, n, e, st);
    else if (n <= 64) project_tc_bn<16>(G.head, p, n, e, st);
    else if (G.large_tile == 1) project_tc_bn<32, EpiStoreSoftmax, 6, 2>(G.head, p, n, e, st);
    else if (n <= 256) project_tc_bn<32>(G.head, p, n, e, st);
    else project_tc_bn<64>(G.head, p, n, e, st);
}

// Four threads per channel while the batch is small (latency), one when it is large (no repeated
// per-channel work); both give the same bits.
// Above 64 streams, stream blocks of 16 or 32 per CTA with the group's weights staged once
// (k_scan_blk, same bits) where d_inner is a multiple of 64 and dt_rank and x_proj's rows are
// multiples of 4 (its 16-byte shared loads).
void launch_scan(const ScanArgs& sc, const ActOut& ao, int n, cudaStream_t st) {
    if (n <= 64) {
        launch(k_scan<4>, dim3(G.di / 64, n), dim3(256), G.xr * sizeof(float), st, sc, ao);
    } else if (G.di % 64 == 0 && G.dr % 4 == 0 && G.xr % 4 == 0 && G.scan_blk) {
        const int sb = n >= 512 ? 32 : 16;
        const size_t smem =
            ((size_t)64 * (scan_blk_wstride(G.dr) + kScanAStride + 2) + (size_t)sb * G.xr) * sizeof(float);
        if (sb == 32) {
            allow_smem(k_scan_blk<32>, smem);
            launch(k_scan_blk<32>, dim3(G.di / 64, (n + 31) / 32), dim3(256), smem, st, sc, ao, n);
        } else {
            allow_smem(k_scan_blk<16>, smem);
            launch(k_scan_blk<16>, dim3(G.di / 64, (n + 15) / 16), dim3(256), smem, st, sc, ao, n);
        }
    } else {
        launch(k_scan<1>, dim3((G.di + 255) / 256, n), dim3(256), G.xr * sizeof(float), st, sc, ao);
    }
}

// vslot: the final norm's validated slots (rejected streams give zero rows), nullptr for a layer norm.
void launch_norm(const Pool& p, int n, const float* w, const float* b, int K_out, cudaStream_t st,
                 const uint32_t* vslot = nullptr) {
    ActOut out{p.act_f, p.act_q, p.act_e, p.cap_pad, K_out};
    if (G.profile != kF32) out.f = nullptr;
    else out.q = nullptr;
    dim3 grid((n + 3) / 4);
    int nc = (G.d + 127) / 128;
    switch (nc) {
        case 1: launch(k_norm<1>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 2: launch(k_norm<2>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 3: launch(k_norm<3>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 4: launch(k_norm<4>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 5: launch(k_norm<5>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 6: launch(k_norm<6>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        case 7: launch(k_norm<7>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
        default: launch(k_norm<8>, grid, dim3(128), 0, st, n, (const float*)p.x, G.d, w, b, out, vslot); break;
    }
}

// Softmax over each row of `logits` written to `out` (may alias), softmax_into's semantics
// (src/domain/tensor.rs:1917-1933): p = exp(l - max) / max(sum, FLT_EPSILON) with the reference's
// Cephes exp, and a row whose logits are all -inf becomes uniform.  Two passes: a (max, sum of
// exp(l - max)) partial per tile of logits (k_softmax_partial over 2048-logit tiles, or the
// tensor-core head's own 128-row tiles, EpiStoreSoftmax), then k_softmax_final combines the
// partials in a fixed order (lane-strided, then a butterfly) and normalises.
__global__ void k_softmax_partial(const float* __restrict__ logits, int V, float* __restrict__ red, int parts) {
    pdl_wait();
    pdl_trigger();
    int b = blockIdx.y, t = blockIdx.x;
    const float* l = logits + (size_t)b * V;
    int v0 = t * kSoftmaxTile, v1 = min(V, v0 + kSoftmaxTile);
    __shared__ float s_m[8], s_s[8];
    float m = -INFINITY;
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) m = fmaxf(m, l[v]);
    m = warp_allmax(m);
    int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) s_m[w] = m;
    __syncthreads();
    m = s_m[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, s_m[i]);
    float s = 0.0f;
    if (m != -INFINITY)
        for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) s = __fadd_rn(s, portable_expf(__fsub_rn(l[v], m)));
    s = warp_allsum(s);
    if (lane == 0) s_s[w] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.0f;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot = __fadd_rn(tot, s_s[i]);
        red[((size_t)b * parts + t) * 2] = m;
        red[((size_t)b * parts + t) * 2 + 1] = tot;
    }
}

__global__ void k_softmax_final(const float* __restrict__ logits, int V, const float* __restrict__ red, int parts,
                                float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float s_ms[2];
    const int b = blockIdx.y;
    const float* rb = red + (size_t)b * parts * 2;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        float M = -INFINITY;
        for (int t = lane; t < parts; t += 32) M = fmaxf(M, rb[2 * t]);
        M = warp_allmax(M);
        float S = 0.0f;
        if (M != -INFINITY)
            for (int t = lane; t < parts; t += 32) {
                const float mt = rb[2 * t];
                if (mt != -INFINITY) S = __fadd_rn(S, __fmul_rn(rb[2 * t + 1], portable_expf(__fsub_rn(mt, M))));
            }
        S = warp_allsum(S);
        if (lane == 0) {
            s_ms[0] = M;
            s_ms[1] = fmaxf(S, 1.1920928955078125e-07f);  // sum.max(f32::EPSILON)
        }
    }
    __syncthreads();
    const float M = s_ms[0], D = s_ms[1];
    const float* l = logits + (size_t)b * V;
    float* o = out + (size_t)b * V;
    const float uni = __fdiv_rn(1.0f, (float)V);
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < V; v += gridDim.x * blockDim.x)
        o[v] = M == -INFINITY ? uni : __fdiv_rn(portable_expf(__fsub_rn(l[v], M)), D);
}

// Kernel classes for the optional per-launch CUDA-event timing (redukt_b200_kernel_times).
enum KClass { kKEmbed = 0, kKNorm, kKInProj, kKXProj, kKScan, kKOutProj, kKHead, kKSoftmax, kKStep, kKClasses };

struct KTiming {
    bool on = false;
    std::vector<cudaEvent_t> pool;  // created lazily, reused
    std::vector<std::pair<int, size_t>> marks;  // (class, index of the start event; stop = +1)
    size_t used = 0;
    cudaEvent_t next() {
        if (used == pool.size()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            pool.push_back(e);
        }
        return pool[used++];
    }
};
KTiming g_kt;

// Brackets the launches of one kernel class with events when timing is on (eager path only).
struct KScope {
    int cls;
    cudaStream_t st;
    size_t idx = 0;
    bool active;
    KScope(int c, cudaStream_t s) : cls(c), st(s), active(g_kt.on) {
        if (active) {
            idx = g_kt.used;
            cudaEventRecord(g_kt.next(), st);
        }
    }
    ~KScope() {
        if (active) {
            cudaEventRecord(g_kt.next(), st);
            g_kt.marks.push_back({cls, idx});
        }
    }
};

int g_launches_per_step = 0;

// ---- fused small-batch step (rk_fused.cuh) ----

bool use_fused(int n) {
    return G.profile != kF32 && G.fused && G.fused_nc > 0 && G.proj_path == 0 && !g_kt.on && n >= 1 &&
           n <= kFusedMaxN;
}

template <int NC>
void launch_fused_nc(const FusedArgs& fa, size_t smem, cudaStream_t st) {
    auto k = k_step_fused<NC>;
    allow_smem(k, smem);
    // one CTA per SM (the job shapes are sized for that grid); a cooperative launch reports a grid
    // that cannot be co-resident
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G.num_sms);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k, fa);
}

void launch_fused(Pool& p, int n, const uint32_t* d_slots, cudaStream_t st) {
    FusedArgs fa{};
    fa.n = n;
    fa.cap = (int)p.cap;
    fa.cap_pad = p.cap_pad;
    fa.d = G.d;
    fa.di = G.di;
    fa.dr = G.dr;
    fa.xr = G.xr;
    fa.nl = G.nl;
    fa.g_in = G.d / kGroup;
    fa.s_in = q8_splits(fa.g_in);
    fa.mpad_in = round_up(2 * G.di, 128);
    fa.g_out = G.di / kGroup;
    fa.s_out = q8_splits(fa.g_out);
    fa.mpad_out = round_up(G.d, 128);
    const int grid = G.num_sms;  // the launch grid: one CTA per SM
    const int nmb = G.di / 64, nt = (n + 7) / 8;
    // phase A: x-half jobs (conv and x_proj work) take 8 streams while they fit; z-half jobs grow
    // to 16 streams first
    fa.sga = 8;
    fa.sgz = 8;
    fa.rz = 64;
    if (2 * nmb * nt > grid && G.di % 128 == 0) fa.rz = 128;  // z half: 128 rows x 8 streams
    if (nmb * nt + (G.di / fa.rz) * nt > grid) fa.sgz = 16;
    if (nmb * nt + (G.di / fa.rz) * ((n + fa.sgz - 1) / fa.sgz) > grid) fa.sga = 16;
    fa.sgb = nmb * ((n + 3) / 4) <= grid ? 4 : 8;
    fa.mc = (G.d / 16) * nt <= grid ? 16 : 32;
    fa.pitch_a = G.d + 16;
    fa.slots = d_slots;
    fa.rflag = p.rflag;
    fa.x = p.x;
    fa.conv = p.conv;
    fa.ssm = p.ssm;
    fa.conv_out = p.conv_out;
    fa.z = p.z;
    fa.xpart = p.xpart;
    fa.act_q = p.act_q;
    fa.act_e = p.act_e;
    fa.layers = G.d_fused;
    fa.norm_f_w = G.norm_f_w;
    fa.norm_f_b = G.norm_f_b;
    fa.bar = p.bar;
    fa.err = G.d_err;
    fa.lay = fused_layout(fa);
    const size_t smem = (size_t)fa.lay.total;
    switch (G.fused_nc) {
        case 1: launch_fused_nc<1>(fa, smem, st); break;
        case 2: launch_fused_nc<2>(fa, smem, st); break;
        case 6: launch_fused_nc<6>(fa, smem, st); break;
        default: launch_fused_nc<8>(fa, smem, st); break;
    }
}

// Enqueues one decode step for n streams whose slots/tokens are already on the device.
int enqueue_step(Pool& p, int n, const uint32_t* d_slots, const uint32_t* d_tokens, float* d_out, bool probs,
                 cudaStream_t st) {
    const bool fused = use_fused(n);
    StepArgs sa{n, (int)p.cap, d_slots, d_tokens, p.rflag, p.since, G.reset_every, G.d_err, p.vslot,
                fused ? p.bar : nullptr};
    // every kernel after the embedding reads the validated slots, never the caller's
    const uint32_t* vs = p.vslot;
    const Mat& emb = G.emb;
    int launches = 0;
    {
        KScope k(kKEmbed, st);
        launch(k_embed, dim3(n), dim3(256), 0, st, sa, (const float*)emb.f, (const int8_t*)emb.q, (const float*)emb.s, G.d,
               G.V, p.x);
        launches++;
    }
    if (fused) {  // every layer and the final norm in one kernel
        launch_fused(p, n, vs, st);
        launches++;
    }
    for (int li = 0; !fused && li < G.nl; li++) {
        const Layer& L = G.layers[li];
        {
            KScope k(kKNorm, st);
            launch_norm(p, n, L.norm_w, L.norm_b, G.d, st);
            launches++;
        }
        {
            KScope k(kKInProj, st);
            project(L.in_proj, p, n, in_proj_epi(L, li, p, vs), st);
        }
        {
            KScope k(kKXProj, st);
            launch_xproj(L, li, p, n, vs, st);
        }
        {
            KScope k(kKScan, st);
            ScanArgs sc{G.di, G.dr, G.xr, (int)p.cap, li, vs, p.rflag, p.zp, p.conv_out, p.z,
                        L.dt_wt, L.dt_b, L.a_t, L.dvec, p.ssm};
            sc.x_late = G.conv_defer;
            ActOut ao{p.act_f, p.act_q, p.act_e, p.cap_pad, G.di};
            if (G.profile != kF32) ao.f = nullptr;
            else ao.q = nullptr;
            launch_scan(sc, ao, n, st);
        }
        {
            KScope k(kKOutProj, st);
            project(L.out_proj, p, n, EpiResidual{p.x, G.d}, st);
        }
        launches += 4;
    }
    if (!fused) {
        KScope k(kKNorm, st);
        launch_norm(p, n, G.norm_f_w, G.norm_f_b, G.d, st, vs);
        launches++;
    }
    float* lo = probs ? p.logits : d_out;
    const bool fused_softmax = probs && G.profile != kF32 && use_tc(n);
    const int head_tiles = (G.V + tc::kBM - 1) / tc::kBM;
    {
        KScope k(kKHead, st);
        if (fused_softmax) project_head_softmax(p, n, lo, head_tiles, st);
        else project_head(p, n, lo, st);
    }
    launches += 1;
    if (probs) {
        KScope k(kKSoftmax, st);
        int parts = head_tiles;
        if (!fused_softmax) {
            parts = (G.V + kSoftmaxTile - 1) / kSoftmaxTile;
            launch(k_softmax_partial, dim3(parts, n), dim3(256), 0, st, (const float*)lo, G.V, p.red, parts);
            launches++;
        }
        launch(k_softmax_final, dim3(std::max(1, std::min(64, G.V / 1024)), n), dim3(256), 0, st, (const float*)lo, G.V,
               (const float*)p.red, parts, d_out);
        launches++;
    }
    g_launches_per_step = launches;
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// Captures `enqueue_step` with these exact pointers into an executable graph.
int capture_step(Pool& p, int n, const uint32_t* d_slots, const uint32_t* d_tokens, float* d_out, bool probs,
                 cudaGraphExec_t* exec_out) {
    cudaStream_t cs = G.stream;
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), BACKEND_FORWARD_FAILED);
    int rc = enqueue_step(p, n, d_slots, d_tokens, d_out, probs, cs);
    cudaError_t e = cudaStreamEndCapture(cs, &graph);
    if (rc != BACKEND_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    CK(e, BACKEND_FORWARD_FAILED);
    e = cudaGraphInstantiate(exec_out, graph, 0);
    cudaGraphDestroy(graph);
    CK(e, BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

uint64_t graph_key(int n, bool probs) {
    return (uint64_t)n | ((uint64_t)probs << 13) | ((uint64_t)G.proj_path << 14) | ((uint64_t)G.reset_every << 16) |
           ((uint64_t)G.fused << 60);
}

// Enqueue one step for this pool's fixed buffers.  The first call for a (n, probs, options)
// key runs eagerly (it also sets every kernel attribute); later calls replay a CUDA graph of the
// same launch sequence captured on the second call.  Timing mode always runs eagerly.
int enqueue_pool_step(Pool& p, int n, bool probs) {
    float* out = p.logits;
    uint64_t key = graph_key(n, probs);
    if (!G.use_graphs || g_kt.on || !p.eager_done.count(key)) {
        int rc = enqueue_step(p, n, p.d_slots, p.d_tokens, out, probs, G.stream);
        if (rc == BACKEND_OK) p.eager_done.insert(key);
        return rc;
    }
    auto it = p.graphs.find(key);
    if (it == p.graphs.end()) {
        cudaGraphExec_t exec = nullptr;
        int rc = capture_step(p, n, p.d_slots, p.d_tokens, out, probs, &exec);
        if (rc != BACKEND_OK) return rc;
        it = p.graphs.emplace(key, exec).first;
    }
    CK(cudaGraphLaunch(it->second, G.stream), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// Graphs of the device-resident entry point, keyed by the caller's pointers as well.
struct DevKey {
    uint64_t key;
    const void *s, *t, *o;
    bool operator<(const DevKey& b) const {
        if (key != b.key) return key < b.key;
        if (s != b.s) return s < b.s;
        if (t != b.t) return t < b.t;
        return o < b.o;
    }
};
std::map<DevKey, cudaGraphExec_t> g_dev_graphs;
std::set<DevKey> g_dev_eager;

void clear_dev_graphs() {
    for (auto& kv : g_dev_graphs) cudaGraphExecDestroy(kv.second);
    g_dev_graphs.clear();
    g_dev_eager.clear();
}

// Validates, uploads slots/tokens, runs the step and copies logits or probabilities to `out`
// (mamba_cuda.cu:604-635 semantics: INVALID_ARGUMENT before any launch, synchronous return).
int pool_forward(Pool& p, uint32_t n, const uint32_t* slots, const uint32_t* tokens, float* out, bool probs) {
    std::fill(p.seen.begin(), p.seen.end(), 0);
    for (uint32_t b = 0; b < n; b++) {
        if (slots[b] >= p.cap || p.seen[slots[b]] || tokens[b] >= (uint32_t)G.V) return BACKEND_INVALID_ARGUMENT;
        p.seen[slots[b]] = 1;
        p.h_slots[b] = slots[b];
        p.h_tokens[b] = tokens[b];
    }
    size_t ib = (size_t)n * sizeof(uint32_t);
    CK(cudaMemcpyAsync(p.d_slots, p.h_slots, ib, cudaMemcpyHostToDevice, G.stream), BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(p.d_tokens, p.h_tokens, ib, cudaMemcpyHostToDevice, G.stream), BACKEND_FORWARD_FAILED);
    int rc = enqueue_pool_step(p, (int)n, probs);
    if (rc != BACKEND_OK) return rc;
    CK(cudaMemcpyAsync(out, p.logits, (size_t)n * G.V * sizeof(float), cudaMemcpyDeviceToHost, G.stream),
       BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(p.h_err, G.d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, G.stream), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    if (*p.h_err) {
        set_err("device error word 0x%x (1 = bad slot/token, 2 = a tensor-core pipeline wait ran out, "
                "4 = a fused-step wait ran out)", *p.h_err);
        cudaMemset(G.d_err, 0, sizeof(uint32_t));
        if (p.counter) cudaMemset(p.counter, 0, kSplitMaxTiles * sizeof(uint32_t));  // an aborted tile keeps its count
        return BACKEND_FORWARD_FAILED;
    }
    return BACKEND_OK;
}

int pool_reset(Pool& p, const uint32_t* slots, uint32_t n) {
    if (!slots) {
        size_t L = G.nl, cap = p.cap, di = G.di;
        const size_t dib = (size_t)state_blocks((int)di) * 64;
        CK(cudaMemsetAsync(p.conv, 0, L * cap * (kDConv - 1) * di * sizeof(float), G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.ssm, 0, L * cap * kDState * dib * sizeof(float), G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.since, 0, cap * sizeof(uint32_t), G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
        return BACKEND_OK;
    }
    for (uint32_t b = 0; b < n; b++) {
        if (slots[b] >= p.cap) return BACKEND_INVALID_ARGUMENT;
        p.h_slots[b] = slots[b];
    }
    if (n == 0) return BACKEND_OK;
    CK(cudaMemcpyAsync(p.d_slots, p.h_slots, (size_t)n * sizeof(uint32_t), cudaMemcpyHostToDevice, G.stream),
       BACKEND_FORWARD_FAILED);
    int per = 3 * G.di + kDState * state_blocks(G.di) * 64;
    k_zero_slots<<<dim3((per + 255) / 256, n, G.nl), 256, 0, G.stream>>>(p.d_slots, (int)n, (int)p.cap, G.nl, G.di,
                                                                         p.conv, p.ssm, p.since);
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

std::string rbin_path(const uint8_t* weights_path) {
    std::string p(reinterpret_cast<const char*>(weights_path));
    if (p.size() < 5 || p.compare(p.size() - 5, 5, ".rbin") != 0) p += "/model.rbin";
    return p;
}

#include "rwkv7_engine.cuh"

// ------------------------------------------------------------------------------------------
// Probability pass without allocation (redukt_b200_softmax_noalloc).
//
// The pass needs scratch for one (max, sum) partial per 2048-logit tile of each row.  Here that
// scratch is a fixed array in the library's own device memory, so the entry point never calls
// cudaMalloc.  The array exists once per GPU that loads the library, for the life of the process.
// ------------------------------------------------------------------------------------------
constexpr uint32_t kNoAllocMaxRows = 1024;
constexpr uint32_t kNoAllocMaxVocab = 65536;
constexpr uint32_t kNoAllocMaxParts = kNoAllocMaxVocab / kSoftmaxTile;  // 32 tiles of 2048 logits
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxRows * kNoAllocMaxParts * 2];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};  // device address of g_noalloc_scratch, per device

// Device buffers of the host-buffer CDF entry point (redukt_b200_cdf), grown on demand.
struct CdfHostBuffers {
    std::mutex mu;
    int device = -1;
    cudaStream_t stream = nullptr;
    float* logits = nullptr;
    uint32_t* cdf = nullptr;
    uint32_t* query_in = nullptr;
    uint32_t* query_out = nullptr;
    uint32_t* slots = nullptr;    // forward_batch_cdf: the step's slots and tokens
    uint32_t* tokens = nullptr;
    uint32_t* h_err = nullptr;    // pinned copy of the engine's device error word
    size_t logit_cap = 0, cdf_cap = 0, row_cap = 0;
};
CdfHostBuffers g_cdf_host;

// Grows the host entry points' device buffers to n_rows rows of vocab logits; caller holds B.mu.
int32_t cdf_buffers(uint32_t n_rows, uint32_t vocab) {
    CdfHostBuffers& B = g_cdf_host;
    int dev = 0;
    CK(cudaGetDevice(&dev), BACKEND_FORWARD_FAILED);
    if (B.device != dev) {   // buffers belong to one device: start over on another
        if (B.stream) { cudaStreamDestroy(B.stream); B.stream = nullptr; }
        cudaFree(B.logits); cudaFree(B.cdf); cudaFree(B.query_in); cudaFree(B.query_out);
        cudaFree(B.slots); cudaFree(B.tokens);
        B.logits = nullptr; B.cdf = nullptr; B.query_in = B.query_out = nullptr;
        B.slots = B.tokens = nullptr;
        B.logit_cap = B.cdf_cap = B.row_cap = 0;
        B.device = dev;
        CK(cudaStreamCreateWithFlags(&B.stream, cudaStreamNonBlocking), BACKEND_FORWARD_FAILED);
    }
    const size_t nl = (size_t)n_rows * vocab, nc = (size_t)n_rows * (vocab + 1);
    if (nl > B.logit_cap) {
        cudaFree(B.logits); B.logits = nullptr; B.logit_cap = 0;
        CK(cudaMalloc(&B.logits, nl * sizeof(float)), BACKEND_FORWARD_FAILED);
        B.logit_cap = nl;
    }
    if (nc > B.cdf_cap) {
        cudaFree(B.cdf); B.cdf = nullptr; B.cdf_cap = 0;
        CK(cudaMalloc(&B.cdf, nc * sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
        B.cdf_cap = nc;
    }
    if (n_rows > B.row_cap) {
        cudaFree(B.query_in); cudaFree(B.query_out); cudaFree(B.slots); cudaFree(B.tokens);
        B.query_in = B.query_out = B.slots = B.tokens = nullptr;
        B.row_cap = 0;
        CK(cudaMalloc(&B.query_in, (size_t)n_rows * sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
        CK(cudaMalloc(&B.query_out, (size_t)n_rows * 3 * sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
        CK(cudaMalloc(&B.slots, (size_t)n_rows * sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
        CK(cudaMalloc(&B.tokens, (size_t)n_rows * sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
        B.row_cap = n_rows;
    }
    return BACKEND_OK;
}

int32_t check_cdf_args(uint32_t n_rows, uint32_t vocab, uint32_t ld_logits, uint32_t ld_cdf) {
    if (vocab == 0 || vocab >= cdf::kTotal) {
        set_err("cdf: vocab %u outside [1, 2^24)", vocab);
        return BACKEND_INVALID_ARGUMENT;
    }
    if (ld_logits < vocab || ld_cdf < vocab + 1) {
        set_err("cdf: strides %u / %u too small for %u logits", ld_logits, ld_cdf, vocab);
        return BACKEND_INVALID_ARGUMENT;
    }
    if (ld_logits > 0x7fffffffu || ld_cdf > 0x7fffffffu) {  // the kernel indexes rows with int strides
        set_err("cdf: strides %u / %u exceed 2^31 - 1", ld_logits, ld_cdf);
        return BACKEND_INVALID_ARGUMENT;
    }
    if (n_rows > 0x7fffffffu) {
        set_err("cdf: %u rows", n_rows);
        return BACKEND_INVALID_ARGUMENT;
    }
    return BACKEND_OK;
}

}  // namespace

// ==========================================================================================
// C ABI
// ==========================================================================================
extern "C" {

BackendResult redukt_backend_init(const uint8_t* weights_path, int32_t device_id, BackendInfo* info_out) {
    if (!weights_path || !info_out) return BACKEND_INIT_FAILED;
    if (G.ready || G.stream) free_model();
    g_err[0] = 0;
    std::string path = rbin_path(weights_path);
    G.device = device_id >= 0 ? device_id : 0;
    if (cudaSetDevice(G.device) != cudaSuccess ||
        cudaStreamCreateWithFlags(&G.stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_err("no CUDA device %d (%s)", G.device, cudaGetErrorString(cudaGetLastError()));
        free_model();
        return BACKEND_INIT_FAILED;
    }
    int maj = 0, min = 0;
    cudaDeviceGetAttribute(&G.num_sms, cudaDevAttrMultiProcessorCount, G.device);  // launch shapes, every profile
    cudaDeviceGetAttribute(&maj, cudaDevAttrComputeCapabilityMajor, G.device);
    cudaDeviceGetAttribute(&min, cudaDevAttrComputeCapabilityMinor, G.device);
    if (maj != 10 || min != 0) {
        set_err("device %d is sm_%d%d; this library is built for sm_100a (B200) only", G.device, maj, min);
        free_model();
        return BACKEND_INIT_FAILED;
    }
    const int kind = rwe::peek_kind(path.c_str());
    G.rwkv = kind == 1;
    int rc = G.rwkv ? rwe::load_weights(path.c_str()) : load_weights(path.c_str());
    if (rc != BACKEND_OK) {
        free_model();
        return (BackendResult)rc;
    }
    if (!dalloc(&G.d_err, 1) || !(G.rwkv ? rwe::pool_alloc(&rwe::M.v1, 1) : pool_alloc(&G.v1, 1))) {
        set_err("device allocation failed");
        free_model();
        return BACKEND_INIT_FAILED;
    }
    if (const char* e = getenv("REDUKT_B200_GRAPHS")) G.use_graphs = atoi(e) != 0;
    if (const char* e = getenv("REDUKT_B200_PROJ")) G.proj_path = atoi(e);
    if (const char* e = getenv("REDUKT_B200_PDL")) G.use_pdl = atoi(e) != 0;
    G.ready = true;
    memset(info_out, 0, sizeof(*info_out));
    info_out->ffi_version = BACKEND_FFI_VERSION;
    info_out->vocab_size = (uint32_t)G.V;
    info_out->hidden_dim = (uint32_t)G.d;
    const char* name = G.rwkv ? "b200-rwkv7-w8a8"
                              : (G.profile == kF32 ? "b200-mamba-f32" : (G.profile == kQ8 ? "b200-mamba-q8" : "b200-mamba-q8row"));
    memcpy(info_out->name, name, strlen(name));
    return BACKEND_OK;
}

BackendResult redukt_backend_forward(uint32_t token, float* out_logits, uint32_t vocab_size) {
    if (!G.ready || !out_logits || vocab_size != (uint32_t)G.V) return BACKEND_FORWARD_FAILED;
    uint32_t slot = 0;
    int rc = G.rwkv ? rwe::pool_forward(rwe::M.v1, 1, &slot, &token, out_logits, false)
                    : pool_forward(G.v1, 1, &slot, &token, out_logits, false);
    return rc == BACKEND_OK ? BACKEND_OK : BACKEND_FORWARD_FAILED;
}

void redukt_backend_reset_state(void) {
    if (!G.ready) return;
    uint32_t slot = 0;
    int rc = G.rwkv ? rwe::pool_reset(rwe::M.v1, &slot, 1) : pool_reset(G.v1, &slot, 1);
    if (rc != BACKEND_OK) fprintf(stderr, "[redukt-b200] reset_state failed\n");
}

void redukt_backend_free(void) { free_model(); }

uint32_t redukt_backend_abi_version(void) { return BACKEND_ABI_VERSION; }

int32_t redukt_backend_batch_init(uint32_t max_streams) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    if (max_streams > kMaxStreams) return BACKEND_INVALID_ARGUMENT;
    CK(cudaStreamSynchronize(G.stream), BACKEND_INIT_FAILED);
    clear_dev_graphs();
    rwe::clear_graphs();
    pool_free(&G.batch);
    rwe::pool_free(&rwe::M.batch);
    if (max_streams == 0) return BACKEND_OK;
    if (!(G.rwkv ? rwe::pool_alloc(&rwe::M.batch, max_streams) : pool_alloc(&G.batch, max_streams))) {
        set_err("batch pool of %u streams: device allocation failed", max_streams);
        return BACKEND_INIT_FAILED;
    }
    return BACKEND_OK;
}

static uint32_t batch_cap() { return G.rwkv ? rwe::M.batch.cap : G.batch.cap; }

int32_t redukt_backend_batch_reset(const uint32_t* slots, uint32_t n_slots) {
    if (!G.ready || batch_cap() == 0) return BACKEND_INIT_FAILED;
    if (slots && n_slots > batch_cap()) return BACKEND_INVALID_ARGUMENT;
    return G.rwkv ? rwe::pool_reset(rwe::M.batch, slots, n_slots) : pool_reset(G.batch, slots, n_slots);
}

static int32_t forward_batch_impl(uint32_t n, const uint32_t* slots, const uint32_t* tokens, float* out,
                                  uint32_t vocab, bool probs) {
    if (!G.ready || batch_cap() == 0) return BACKEND_INIT_FAILED;
    if (vocab != (uint32_t)G.V || n > batch_cap()) return BACKEND_INVALID_ARGUMENT;
    if (n == 0) return BACKEND_OK;
    if (!slots || !tokens || !out) return BACKEND_INVALID_ARGUMENT;
    return G.rwkv ? rwe::pool_forward(rwe::M.batch, n, slots, tokens, out, probs)
                  : pool_forward(G.batch, n, slots, tokens, out, probs);
}

int32_t redukt_backend_forward_batch(uint32_t n_streams, const uint32_t* slots, const uint32_t* tokens,
                                     float* out_logits, uint32_t vocab_size) {
    return forward_batch_impl(n_streams, slots, tokens, out_logits, vocab_size, false);
}

int32_t redukt_backend_forward_batch_probs(uint32_t n_streams, const uint32_t* slots, const uint32_t* tokens,
                                           float* out_probs, uint32_t vocab_size) {
    return forward_batch_impl(n_streams, slots, tokens, out_probs, vocab_size, true);
}

int32_t redukt_backend_set_reset_every(uint32_t every) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    if (every > (1u << 31)) return BACKEND_INVALID_ARGUMENT;
    G.reset_every = every;
    return BACKEND_OK;
}

int32_t redukt_b200_forward_batch_device(uint32_t n, const uint32_t* d_slots, const uint32_t* d_tokens, float* d_out,
                                         uint32_t vocab, int32_t probs, void* cuda_stream) {
    if (!G.ready || batch_cap() == 0) return BACKEND_INIT_FAILED;
    if (vocab != (uint32_t)G.V || n > batch_cap()) return BACKEND_INVALID_ARGUMENT;
    if (n == 0) return BACKEND_OK;
    if (!d_slots || !d_tokens || !d_out) return BACKEND_INVALID_ARGUMENT;
    cudaStream_t st = cuda_stream ? reinterpret_cast<cudaStream_t>(cuda_stream) : G.stream;
    if (G.rwkv) return rwe::forward_device(n, d_slots, d_tokens, d_out, probs != 0, st);
    DevKey k{graph_key((int)n, probs != 0), d_slots, d_tokens, d_out};
    if (!G.use_graphs || g_kt.on || !g_dev_eager.count(k)) {
        int rc = enqueue_step(G.batch, (int)n, d_slots, d_tokens, d_out, probs != 0, st);
        if (rc == BACKEND_OK) g_dev_eager.insert(k);
        return rc;
    }
    auto it = g_dev_graphs.find(k);
    if (it == g_dev_graphs.end()) {
        if (g_dev_graphs.size() >= 64) clear_dev_graphs();
        // capture on the library stream, ordered after the caller's stream
        cudaEvent_t ev;
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), BACKEND_FORWARD_FAILED);
        cudaEventRecord(ev, st);
        cudaStreamWaitEvent(G.stream, ev, 0);
        cudaEventDestroy(ev);
        cudaGraphExec_t exec = nullptr;
        int rc = capture_step(G.batch, (int)n, d_slots, d_tokens, d_out, probs != 0, &exec);
        if (rc != BACKEND_OK) return rc;
        it = g_dev_graphs.emplace(k, exec).first;
    }
    CK(cudaGraphLaunch(it->second, st), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

int32_t redukt_b200_kernel_times(int32_t enable, double* ms, uint32_t* launches, uint32_t n_classes) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    CK(cudaDeviceSynchronize(), BACKEND_FORWARD_FAILED);
    if (ms && launches) {
        for (uint32_t c = 0; c < n_classes; c++) {
            ms[c] = 0.0;
            launches[c] = 0;
        }
        for (auto& m : g_kt.marks) {
            if ((uint32_t)m.first >= n_classes) continue;
            float t = 0.f;
            if (cudaEventElapsedTime(&t, g_kt.pool[m.second], g_kt.pool[m.second + 1]) == cudaSuccess) {
                ms[m.first] += t;
                launches[m.first] += 1;
            }
        }
    }
    g_kt.marks.clear();
    g_kt.used = 0;
    g_kt.on = enable != 0;
    return BACKEND_OK;
}

int32_t redukt_b200_device_error(uint32_t* out_word) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    uint32_t w = 0;
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    CK(cudaMemcpy(&w, G.d_err, sizeof(w), cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
    CK(cudaMemset(G.d_err, 0, sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
    if (out_word) *out_word = w;
    return BACKEND_OK;
}

int32_t redukt_b200_get_state(uint32_t slot, float* conv, float* ssm) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    if (G.rwkv) return BACKEND_INVALID_ARGUMENT;
    Pool* p = &G.batch;
    if (slot == 0xffffffffu) {
        p = &G.v1;
        slot = 0;
    }
    if (slot >= p->cap) return BACKEND_INVALID_ARGUMENT;
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    const int di = G.di, cap = (int)p->cap;
    const size_t dib = (size_t)state_blocks(di) * 64;
    std::vector<float> tmp((size_t)kDState * dib);
    for (int l = 0; l < G.nl; l++) {  // channel-blocked device layout -> the reference's [di][k]
        if (conv) {
            CK(cudaMemcpy(tmp.data(), p->conv + conv_off(l, cap, slot, di, 0, 0), (size_t)(kDConv - 1) * di * sizeof(float),
                          cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
            for (int j = 0; j < di; j++)
                for (int k = 0; k < kDConv - 1; k++)
                    conv[((size_t)l * di + j) * (kDConv - 1) + k] = tmp[conv_off(0, 1, 0, di, k, j)];
        }
        if (ssm) {
            CK(cudaMemcpy(tmp.data(), p->ssm + ssm_off(l, cap, slot, di, 0, 0), (size_t)kDState * dib * sizeof(float),
                          cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
            for (int j = 0; j < di; j++)
                for (int k = 0; k < kDState; k++) ssm[((size_t)l * di + j) * kDState + k] = tmp[ssm_off(0, 1, 0, di, k, j)];
        }
    }
    return BACKEND_OK;
}

int32_t redukt_b200_rwkv_get_state(uint32_t slot, float* x_att, float* wkv, float* x_ffn, float* v_first) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    if (!G.rwkv) return BACKEND_INVALID_ARGUMENT;
    return rwe::get_state(slot, x_att, wkv, x_ffn, v_first);
}

int32_t redukt_b200_get_q8(int32_t which, uint32_t layer, int8_t* q, float* scales) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    if (G.rwkv) return rwe::get_q8(which, layer, q, scales);
    if (G.profile == kF32) return BACKEND_INVALID_ARGUMENT;
    const Mat* m = nullptr;
    if (which == 0) m = &G.emb;
    else if (which == 1) m = &G.head;
    else if ((which == 2 || which == 3) && layer < (uint32_t)G.nl)
        m = which == 2 ? &G.layers[layer].in_proj : &G.layers[layer].out_proj;
    if (!m) return BACKEND_INVALID_ARGUMENT;
    size_t count = (size_t)m->rows * m->cols;
    if (q) {
        const int rows_pad = round_up(m->rows, tc::kBM);
        std::vector<int8_t> tiled((size_t)rows_pad * m->cols);
        CK(cudaMemcpy(tiled.data(), m->q, tiled.size(), cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
        for (int r = 0; r < m->rows; r++)
            for (int k = 0; k < m->cols; k++) q[(size_t)r * m->cols + k] = tiled[wq_off(rows_pad, r, k)];
    }
    (void)count;
    if (scales)
        CK(cudaMemcpy(scales, m->s, (size_t)m->rows * (m->cols / kGroup) * sizeof(float), cudaMemcpyDeviceToHost),
           BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// Times one kernel class in isolation: the class's launches for every layer of one step (the
// head or embedding once) are captured into a CUDA graph over the batch pool's buffers with
// slots 0..n-1; each replay follows an L2 flush (a 256 MiB memset) so weights come from HBM as
// in a real step.  Overwrites the pool's scratch and the state of slots 0..n-1.
int32_t redukt_b200_time_kernel(int32_t cls, uint32_t n, uint32_t reps, float* ms_per_launch) {
    if (!G.ready || batch_cap() == 0) return BACKEND_INIT_FAILED;
    if (G.rwkv) {
        set_err("time_kernel: per-class timing is implemented for the Mamba engine only");
        return BACKEND_INVALID_ARGUMENT;
    }
    if (n == 0 || n > G.batch.cap || !ms_per_launch || cls < 0 || cls >= (int)kKClasses || cls == (int)kKSoftmax)
        return BACKEND_INVALID_ARGUMENT;
    if (cls == (int)kKStep && !use_fused((int)n)) {
        set_err("time_kernel: the fused step does not run for %u streams with the current options", n);
        return BACKEND_INVALID_ARGUMENT;
    }
    Pool& p = G.batch;
    std::vector<uint32_t> idx(n);
    for (uint32_t i = 0; i < n; i++) idx[i] = i;
    CK(cudaMemcpy(p.d_slots, idx.data(), n * 4, cudaMemcpyHostToDevice), BACKEND_FORWARD_FAILED);
    std::fill(idx.begin(), idx.end(), 1u);
    CK(cudaMemcpy(p.d_tokens, idx.data(), n * 4, cudaMemcpyHostToDevice), BACKEND_FORWARD_FAILED);
    void* flush = nullptr;
    const size_t flush_bytes = (size_t)256 << 20;
    CK(cudaMalloc(&flush, flush_bytes), BACKEND_FORWARD_FAILED);
    cudaStream_t st = G.stream;
    int nn = (int)n;
    int launches = 0;
    auto body = [&]() {
        StepArgs sa{nn, (int)p.cap, p.d_slots, p.d_tokens, p.rflag, p.since, 0u, G.d_err, p.vslot};
        launches = 0;
        if (cls == kKEmbed) {
            launch(k_embed, dim3(nn), dim3(256), 0, st, sa, (const float*)G.emb.f, (const int8_t*)G.emb.q,
                   (const float*)G.emb.s, G.d, G.V, p.x);
            launches = 1;
        } else if (cls == kKHead) {
            project_head(p, nn, p.logits, st);
            launches = 1;
        } else if (cls == kKStep) {  // every layer + the final norm in the fused kernel
            cudaMemsetAsync(p.bar, 0, sizeof(uint32_t), st);
            launch_fused(p, nn, p.d_slots, st);
            launches = 1;
        } else {
            for (int li = 0; li < G.nl; li++) {
                const Layer& L = G.layers[li];
                if (cls == kKNorm) launch_norm(p, nn, L.norm_w, L.norm_b, G.d, st);
                if (cls == kKInProj) {
                    project(L.in_proj, p, nn, in_proj_epi(L, li, p, p.d_slots), st);
                }
                if (cls == kKXProj) launch_xproj(L, li, p, nn, p.d_slots, st);
                if (cls == kKScan) {
                    ScanArgs sc{G.di, G.dr, G.xr, (int)p.cap, li, p.d_slots, p.rflag, p.zp, p.conv_out, p.z,
                                L.dt_wt, L.dt_b, L.a_t, L.dvec, p.ssm};
                    sc.x_late = G.conv_defer;
                    ActOut ao{p.act_f, p.act_q, p.act_e, p.cap_pad, G.di};
                    if (G.profile != kF32) ao.f = nullptr;
                    else ao.q = nullptr;
                    launch_scan(sc, ao, nn, st);
                }
                if (cls == kKOutProj) project(L.out_proj, p, nn, EpiResidual{p.x, G.d}, st);
                launches++;
            }
        }
    };
    body();  // eager once: sets kernel attributes, fills rflag via embed-free path
    CK(cudaMemsetAsync(p.rflag, 0, n * sizeof(uint32_t), st), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(st), BACKEND_FORWARD_FAILED);
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal), BACKEND_FORWARD_FAILED);
    body();
    CK(cudaStreamEndCapture(st, &graph), BACKEND_FORWARD_FAILED);
    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(e, BACKEND_FORWARD_FAILED);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    double total = 0.0;
    uint32_t R = reps ? reps : 5;
    for (uint32_t r = 0; r <= R; r++) {
        cudaMemsetAsync(flush, r & 0xff, flush_bytes, st);
        cudaEventRecord(e0, st);
        cudaGraphLaunch(exec, st);
        cudaEventRecord(e1, st);
        cudaError_t se = cudaEventSynchronize(e1);
        if (se != cudaSuccess) {
            set_err("time_kernel: %s", cudaGetErrorString(se));
            break;
        }
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        if (r > 0) total += ms;  // replay 0 warms the graph
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    cudaFree(flush);
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    *ms_per_launch = (float)(total / R / launches);
    return BACKEND_OK;
}

int32_t redukt_b200_info(uint32_t* out, uint32_t n) {
    if (!G.ready) return BACKEND_INIT_FAILED;
    uint32_t v[13] = {(uint32_t)G.V, (uint32_t)G.d, (uint32_t)G.di, G.h.ds, G.h.dc, (uint32_t)G.dr, (uint32_t)G.nl,
                      G.h.flags, (uint32_t)G.profile, G.batch.cap, G.reset_every, (uint32_t)G.proj_path,
                      (uint32_t)g_launches_per_step};
    if (G.rwkv) {  // RWKV-7: words 2..5 are d_ffn, n_head, head size, sum of LoRA ranks; profile 3 = W8A8
        const rwe::Model& m = rwe::M;
        uint32_t w[13] = {(uint32_t)m.V, (uint32_t)m.D, (uint32_t)m.F, (uint32_t)m.H, 64u, (uint32_t)m.R,
                          (uint32_t)m.L, m.flags, 3u, m.batch.cap, G.reset_every, (uint32_t)G.proj_path,
                          (uint32_t)g_launches_per_step};
        for (int i = 0; i < 13; i++) v[i] = w[i];
    }
    for (uint32_t i = 0; i < n && i < 13; i++) out[i] = v[i];
    return BACKEND_OK;
}

int32_t redukt_b200_set_option(const char* key, int64_t value) {
    if (!key) return BACKEND_INVALID_ARGUMENT;
    if (!strcmp(key, "proj_path")) {
        if (value < 0 || value > 2) return BACKEND_INVALID_ARGUMENT;
        G.proj_path = (int)value;
        return BACKEND_OK;
    }
    if (!strcmp(key, "graphs")) {
        G.use_graphs = value != 0;
        return BACKEND_OK;
    }
    if (!strcmp(key, "wait_limit_us")) {  // test setting: limit of every bounded device wait (0 = default)
        if (value < 0 || value > 10 * 1000 * 1000) return BACKEND_INVALID_ARGUMENT;
        long long cyc = value ? (long long)value * 2000 : tc::kWaitLimitCycles;  // ~2 cycles per ns
        unsigned long long ns = value ? (unsigned long long)value * 1000 : 200ull * 1000 * 1000;
        CK(cudaMemcpyToSymbol(tc::g_wait_cycles, &cyc, sizeof(cyc)), BACKEND_FORWARD_FAILED);
        CK(cudaMemcpyToSymbol(tc::g_wait_ns, &ns, sizeof(ns)), BACKEND_FORWARD_FAILED);
        return BACKEND_OK;
    }
    if (!strcmp(key, "reset_counters")) {  // bench setting: every batch slot has run `value` forwards
        if (value < 0 || value > 0xffffffffll || batch_cap() == 0) return BACKEND_INVALID_ARGUMENT;
        uint32_t* since = G.rwkv ? rwe::M.batch.since : G.batch.since;
        std::vector<uint32_t> h(batch_cap(), (uint32_t)value);
        CK(cudaMemcpyAsync(since, h.data(), h.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, G.stream),
           BACKEND_FORWARD_FAILED);
        CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
        return BACKEND_OK;
    }
    if (!strcmp(key, "wait_test")) {  // test setting: one bounded wait of the next step runs out
        if (value < 0 || value > 2) return BACKEND_INVALID_ARGUMENT;
        int v = (int)value;
        CK(cudaMemcpyToSymbol(tc::g_wait_test, &v, sizeof(v)), BACKEND_FORWARD_FAILED);
        return BACKEND_OK;
    }
    if (!strcmp(key, "split_target")) {
        if (value < 0 || value > 4096) return BACKEND_INVALID_ARGUMENT;
        g_split_target = (int)value;
        for (Pool* p : {&G.v1, &G.batch}) {  // captured graphs hold the old grids
            for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
            p->graphs.clear();
        }
        clear_dev_graphs();
        return BACKEND_OK;
    }
    if (!strcmp(key, "scan_blk") || !strcmp(key, "large_tile") || !strcmp(key, "conv_defer") ||
        !strcmp(key, "f32_pairs")) {
        if (!strcmp(key, "scan_blk")) G.scan_blk = value != 0;
        else if (!strcmp(key, "f32_pairs")) G.f32_pairs = value != 0;
        else if (!strcmp(key, "conv_defer")) G.conv_defer = value != 0;
        else if (value < 0 || value > 1) return BACKEND_INVALID_ARGUMENT;
        else G.large_tile = (int)value;
        for (Pool* p : {&G.v1, &G.batch}) {
            for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
            p->graphs.clear();
            p->eager_done.clear();
        }
        clear_dev_graphs();
        return BACKEND_OK;
    }
    if (!strcmp(key, "fused") || !strcmp(key, "head_ctas") || !strcmp(key, "head_wide")) {
        if (!strcmp(key, "fused")) G.fused = value != 0;
        else if (!strcmp(key, "head_wide")) G.head_wide = value != 0;
        else {
            if (value < 1 || value > 2) return BACKEND_INVALID_ARGUMENT;
            G.head_ctas = (int)value;
        }
        for (Pool* p : {&G.v1, &G.batch}) {  // captured graphs hold the old launch sequence
            for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
            p->graphs.clear();
            p->eager_done.clear();
        }
        clear_dev_graphs();
        return BACKEND_OK;
    }
    if (!strcmp(key, "pdl")) {
        G.use_pdl = value != 0;
        for (Pool* p : {&G.v1, &G.batch}) {  // captured graphs hold the old launch attributes
            for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
            p->graphs.clear();
        }
        clear_dev_graphs();
        rwe::clear_graphs();
        return BACKEND_OK;
    }
    return BACKEND_INVALID_ARGUMENT;
}

// See include/redukt_gpu.h.  The first call on a device looks up the scratch array's device
// address on that device (cudaGetSymbolAddress, with that device current) and caches it.
int32_t redukt_b200_softmax_noalloc(const float* d_logits, uint32_t n_rows, uint32_t vocab, float* d_probs,
                                    void* cuda_stream) {
    if (!d_logits || !d_probs) return BACKEND_INVALID_ARGUMENT;
    if (n_rows == 0) return BACKEND_OK;
    if (n_rows > kNoAllocMaxRows || vocab == 0 || vocab > kNoAllocMaxVocab) {
        set_err("softmax_noalloc: %u rows x %u logits exceeds the fixed scratch (at most %u rows of at most %u logits)",
                n_rows, vocab, kNoAllocMaxRows, kNoAllocMaxVocab);
        return BACKEND_INVALID_ARGUMENT;
    }
    int dev = -1;
    CK(cudaGetDevice(&dev), BACKEND_FORWARD_FAILED);
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        set_err("softmax_noalloc: device ordinal %d is out of range", dev);
        return BACKEND_INVALID_ARGUMENT;
    }
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* addr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_scratch);
            if (e != cudaSuccess || !addr) {
                set_err("softmax_noalloc: cudaGetSymbolAddress failed on device %d (%s)", dev, cudaGetErrorString(e));
                return BACKEND_FORWARD_FAILED;
            }
            g_noalloc_ptr[dev] = static_cast<float*>(addr);
        }
        scratch = g_noalloc_ptr[dev];
    }
    // every (row, tile) partial is written by the first kernel before the second reads it, so
    // nothing left in the array by an earlier call is ever read
    const int parts = (int)((vocab + kSoftmaxTile - 1) / kSoftmaxTile);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(cuda_stream);
    k_softmax_partial<<<dim3(parts, n_rows), 256, 0, st>>>(d_logits, (int)vocab, scratch, parts);
    k_softmax_final<<<dim3(std::max(1, std::min(64, (int)vocab / 1024)), n_rows), 256, 0, st>>>(
        d_logits, (int)vocab, scratch, parts, d_probs);
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

int32_t redukt_b200_cdf_device(const float* d_logits, uint32_t n_rows, uint32_t vocab, uint32_t ld_logits,
                               uint32_t* d_cdf, uint32_t ld_cdf, const uint32_t* d_symbols,
                               const uint32_t* d_cum_freqs, uint32_t* d_query_out, void* cuda_stream) {
    if (!d_logits || !d_cdf) return BACKEND_INVALID_ARGUMENT;
    if (int32_t rc = check_cdf_args(n_rows, vocab, ld_logits, ld_cdf)) return rc;
    if ((d_symbols || d_cum_freqs) && !d_query_out) return BACKEND_INVALID_ARGUMENT;
    if (d_symbols && d_cum_freqs) {
        set_err("cdf: give symbols or cum_freqs, not both");
        return BACKEND_INVALID_ARGUMENT;
    }
    if (n_rows == 0) return BACKEND_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(cuda_stream);
    const size_t dyn = cdf::cdf_dyn_smem((int)vocab);
    if (dyn > 0) {   // per device, the attribute is set once
        static std::mutex mu;
        static bool done[kNoAllocMaxDevices] = {};
        int dev = 0;
        CK(cudaGetDevice(&dev), BACKEND_FORWARD_FAILED);
        std::lock_guard<std::mutex> lock(mu);
        if (dev >= 0 && dev < kNoAllocMaxDevices && !done[dev]) {
            CK(cudaFuncSetAttribute(cdf::k_cdf_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)cdf::cdf_dyn_smem(cdf::kSmemVocab)), BACKEND_FORWARD_FAILED);
            done[dev] = true;
        }
    }
    cdf::k_cdf_rows<<<n_rows, cdf::kThreads, dyn, st>>>(d_logits, (int)vocab, (int)ld_logits, d_cdf, (int)ld_cdf,
                                                       d_symbols, d_cum_freqs,
                                                       (d_symbols || d_cum_freqs) ? d_query_out : nullptr);
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

int32_t redukt_b200_cdf(const float* logits, uint32_t n_rows, uint32_t vocab, uint32_t* cdf_out,
                        const uint32_t* symbols, const uint32_t* cum_freqs, uint32_t* query_out) {
    if (!logits) return BACKEND_INVALID_ARGUMENT;
    if (int32_t rc = check_cdf_args(n_rows, vocab, vocab, vocab + 1)) return rc;
    const bool query = symbols || cum_freqs;
    if ((query && !query_out) || (symbols && cum_freqs)) return BACKEND_INVALID_ARGUMENT;
    if (n_rows == 0) return BACKEND_OK;
    CdfHostBuffers& B = g_cdf_host;
    std::lock_guard<std::mutex> lock(B.mu);
    if (int32_t rc = cdf_buffers(n_rows, vocab)) return rc;
    const size_t nl = (size_t)n_rows * vocab, nc = (size_t)n_rows * (vocab + 1);
    CK(cudaMemcpyAsync(B.logits, logits, nl * sizeof(float), cudaMemcpyHostToDevice, B.stream), BACKEND_FORWARD_FAILED);
    if (query)
        CK(cudaMemcpyAsync(B.query_in, symbols ? symbols : cum_freqs, (size_t)n_rows * sizeof(uint32_t),
                           cudaMemcpyHostToDevice, B.stream), BACKEND_FORWARD_FAILED);
    int32_t rc = redukt_b200_cdf_device(B.logits, n_rows, vocab, vocab, B.cdf, vocab + 1,
                                        symbols ? B.query_in : nullptr, cum_freqs ? B.query_in : nullptr,
                                        B.query_out, B.stream);
    if (rc != BACKEND_OK) return rc;
    if (cdf_out)
        CK(cudaMemcpyAsync(cdf_out, B.cdf, nc * sizeof(uint32_t), cudaMemcpyDeviceToHost, B.stream), BACKEND_FORWARD_FAILED);
    if (query)
        CK(cudaMemcpyAsync(query_out, B.query_out, (size_t)n_rows * 3 * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                           B.stream), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(B.stream), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

int32_t redukt_b200_forward_batch_cdf(uint32_t n, const uint32_t* slots, const uint32_t* tokens,
                                      const uint32_t* symbols, const uint32_t* cum_freqs, uint32_t* query_out,
                                      uint32_t* cdf_out) {
    if (!G.ready || batch_cap() == 0) return BACKEND_INIT_FAILED;
    if (n > batch_cap()) return BACKEND_INVALID_ARGUMENT;
    if (n == 0) return BACKEND_OK;
    const bool query = symbols || cum_freqs;
    if (!slots || !tokens || (query && !query_out) || (symbols && cum_freqs) || (!query && !cdf_out))
        return BACKEND_INVALID_ARGUMENT;
    const uint32_t V = (uint32_t)G.V;
    {   // the host path's checks (pool_forward): slots in the pool and distinct, tokens in the vocabulary
        std::vector<uint8_t> seen(batch_cap(), 0);
        for (uint32_t b = 0; b < n; b++) {
            if (slots[b] >= batch_cap() || seen[slots[b]] || tokens[b] >= V) return BACKEND_INVALID_ARGUMENT;
            seen[slots[b]] = 1;
        }
    }
    CdfHostBuffers& B = g_cdf_host;
    std::lock_guard<std::mutex> lock(B.mu);
    CK(cudaSetDevice(G.device), BACKEND_FORWARD_FAILED);
    if (int32_t rc = cdf_buffers(n, V)) return rc;
    cudaStream_t st = G.stream;
    const size_t ib = (size_t)n * sizeof(uint32_t);
    CK(cudaMemcpyAsync(B.slots, slots, ib, cudaMemcpyHostToDevice, st), BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(B.tokens, tokens, ib, cudaMemcpyHostToDevice, st), BACKEND_FORWARD_FAILED);
    if (query)
        CK(cudaMemcpyAsync(B.query_in, symbols ? symbols : cum_freqs, ib, cudaMemcpyHostToDevice, st),
           BACKEND_FORWARD_FAILED);
    int32_t rc = redukt_b200_forward_batch_device(n, B.slots, B.tokens, B.logits, V, 0, st);
    if (rc != BACKEND_OK) return rc;
    rc = redukt_b200_cdf_device(B.logits, n, V, V, B.cdf, V + 1, symbols ? B.query_in : nullptr,
                                cum_freqs ? B.query_in : nullptr, B.query_out, st);
    if (rc != BACKEND_OK) return rc;
    if (query)
        CK(cudaMemcpyAsync(query_out, B.query_out, ib * 3, cudaMemcpyDeviceToHost, st), BACKEND_FORWARD_FAILED);
    if (cdf_out)
        CK(cudaMemcpyAsync(cdf_out, B.cdf, (size_t)n * (V + 1) * sizeof(uint32_t), cudaMemcpyDeviceToHost, st),
           BACKEND_FORWARD_FAILED);
    if (!B.h_err) CK(cudaMallocHost(&B.h_err, sizeof(uint32_t)), BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(B.h_err, G.d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(st), BACKEND_FORWARD_FAILED);
    if (*B.h_err) {
        set_err("forward_batch_cdf: device error word 0x%x (2 = a tensor-core pipeline wait ran out, "
                "4 = a fused-step wait ran out)", *B.h_err);
        cudaMemset(G.d_err, 0, sizeof(uint32_t));
        return BACKEND_FORWARD_FAILED;
    }
    return BACKEND_OK;
}

const char* redukt_b200_last_error(void) { return g_err; }

}  // extern "C"
