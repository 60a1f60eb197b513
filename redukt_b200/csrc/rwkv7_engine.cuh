// RWKV-7 engine behind the same C ABI: loaded when the .rbin header says version 3 with the
// RWKV-7 model-kind flag.  Host counterpart of the reference's Rwkv7Model (rwkv7/model.rs:249-698)
// for n lockstep streams; the reference itself has only a single-stream path
// (src/application/model_loader.rs:218-223).
//
// Included inside redukt_gpu.cu's anonymous namespace: it shares the device, stream, error word,
// launch helpers, graph policy and allocation list of the Mamba engine (G), and only one model of
// either kind is loaded at a time.
//
// Device layout (per layer, slot-major):
//   x_att, x_ffn   [L][cap][D]        token-shift states
//   wkv            [L][cap][H][16][64][4]  64x64 state per head, row i's 16-byte chunk q at q*64+i
//   v_first        [cap][D]
//   since          [cap]
// Weights: LayerNorm / mix / bias vectors f32; the four LoRA down-projections concatenated into
// one [R][D] matrix and the four up-projections into a head-major [H][R][64] (R = sum of the
// ranks); the W8A8
// matrices as per-row-quantised int8 in the tiled layout of the tensor-core projection.

namespace rwe {

using namespace rk::rw;

constexpr uint32_t kVersion = 3u;
constexpr uint32_t kFlagRwkv7 = 1u << 4;
constexpr uint32_t kFlagG1k = 1u << 5;
constexpr int kHeaderWords = 19;
constexpr int kMaxR = 640;     // sum of LoRA ranks (shared-memory tile of k_rw_wkv)
constexpr int kTcMinStreams = 9;  // below this the dp4a projection is used

struct W8 {
    int rows = 0, cols = 0, rows_pad = 0;
    int8_t* q = nullptr;  // tiled [cols/64][rows_pad][64]
    float* s = nullptr;   // [rows]
};

struct Layer {
    float *ln1_w = nullptr, *ln1_b = nullptr, *ln2_w = nullptr, *ln2_b = nullptr;
    float* mix6 = nullptr;  // [6][D] x_r, x_w, x_k, x_v, x_a, x_g
    float *w0 = nullptr, *a0 = nullptr, *v0 = nullptr, *k_k = nullptr, *k_a = nullptr, *r_k = nullptr;
    float *lnx_w = nullptr, *lnx_b = nullptr, *ffn_xk = nullptr;
    float* w1cat = nullptr;  // [R][D]
    float* w2cat = nullptr;  // [H][R][64] (head-major, k_rw_put_up)
    W8 r, k, v, o, fk, fv;
};

struct Pool {
    uint32_t cap = 0;
    int cap_pad = 0;
    float *x_att = nullptr, *x_ffn = nullptr, *wkv = nullptr, *v_first = nullptr;
    uint32_t* since = nullptr;
    float *x = nullptr, *lora_in = nullptr, *rkv = nullptr, *h1 = nullptr, *gated = nullptr, *ffn = nullptr;
    float *logits = nullptr, *red = nullptr, *as = nullptr;
    int8_t *aq0 = nullptr, *aq1 = nullptr, *aq2 = nullptr;
    uint32_t *rflag = nullptr, *vslot = nullptr, *d_slots = nullptr, *d_tokens = nullptr;
    uint32_t *h_slots = nullptr, *h_tokens = nullptr, *h_err = nullptr;
    std::vector<uint8_t> seen;
    std::map<uint64_t, cudaGraphExec_t> graphs;
    std::set<uint64_t> eager_done;
};

struct Model {
    int V = 0, D = 0, H = 0, F = 0, L = 0, R = 0, g1k = 0;
    uint32_t flags = 0;
    int seg_off[4] = {}, seg_len[4] = {}, tiles_before[5] = {};
    float* emb = nullptr;  // [V][D], LayerNorm ln0 applied at load
    float *ln_out_w = nullptr, *ln_out_b = nullptr;
    W8 head;
    std::vector<Layer> layers;
    Pool v1, batch;
};

Model M;

void pool_free(Pool* p) {
    for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
    void* bufs[] = {p->x_att, p->x_ffn, p->wkv, p->v_first, p->since, p->x, p->lora_in, p->rkv, p->h1, p->gated,
                    p->ffn, p->logits, p->red, p->as, p->aq0, p->aq1, p->aq2, p->rflag, p->vslot, p->d_slots, p->d_tokens};
    for (void* b : bufs) cudaFree(b);
    if (p->h_slots) cudaFreeHost(p->h_slots);
    if (p->h_tokens) cudaFreeHost(p->h_tokens);
    if (p->h_err) cudaFreeHost(p->h_err);
    *p = Pool();
}

bool pool_alloc(Pool* p, uint32_t cap) {
    *p = Pool();
    p->cap = cap;
    p->cap_pad = round_up((int)cap, 64);
    const size_t n = cap, L = M.L, D = M.D, F = M.F, V = M.V, cp = p->cap_pad;
    const size_t parts = (V + kSoftmaxTile - 1) / kSoftmaxTile;
    bool ok = dalloc(&p->x_att, L * n * D) && dalloc(&p->x_ffn, L * n * D) &&
              dalloc(&p->wkv, L * n * (size_t)M.H * kHS * kHS) && dalloc(&p->v_first, n * D) && dalloc(&p->since, n) &&
              dalloc(&p->x, n * D) && dalloc(&p->lora_in, 4 * n * D) && dalloc(&p->rkv, 3 * n * D) &&
              dalloc(&p->h1, n * (size_t)M.R) && dalloc(&p->gated, n * D) && dalloc(&p->ffn, n * F) &&
              dalloc(&p->logits, n * V) && dalloc(&p->red, n * parts * 2) && dalloc(&p->as, 3 * n) &&
              dalloc(&p->aq0, std::max(D, F) * cp) && dalloc(&p->aq1, D * cp) && dalloc(&p->aq2, D * cp) &&
              dalloc(&p->rflag, n) && dalloc(&p->vslot, n) && dalloc(&p->d_slots, n) && dalloc(&p->d_tokens, n);
    ok = ok && cudaHostAlloc(reinterpret_cast<void**>(&p->h_slots), n * 4, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(reinterpret_cast<void**>(&p->h_tokens), n * 4, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc(reinterpret_cast<void**>(&p->h_err), 4, cudaHostAllocDefault) == cudaSuccess;
    p->seen.assign(n, 0);
    if (!ok) pool_free(p);
    return ok;
}

void release() {
    pool_free(&M.v1);
    pool_free(&M.batch);
    M = Model();
}

// ---- Loading ----------------------------------------------------------------------------------

// Per-row W8 quantisation with the reference recipe (Q8Tensor::from_f32, tensor.rs:113-135), then
// the tiled layout.
bool load_w8(Reader& r, W8* m, int rows, int cols) {
    m->rows = rows;
    m->cols = cols;
    m->rows_pad = round_up(rows, tc::kBM);
    const size_t count = (size_t)rows * cols;
    if (!r.read_to(g_tmp, count)) return false;
    int8_t* q_rm = nullptr;
    if (!dalloc(&q_rm, count, false)) return false;
    bool ok = model_alloc(&m->q, (size_t)m->rows_pad * cols) && model_alloc(&m->s, (size_t)rows);
    if (ok) {
        k_quantize_q8<<<(unsigned)((rows + 7) / 8), 256>>>(g_tmp, (size_t)rows, cols, q_rm, m->s);
        k_tile_q8<<<(unsigned)((count / 16 + 255) / 256), 256>>>(q_rm, rows, cols, m->rows_pad, m->q);
        ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(q_rm);
    return ok;
}

// A LoRA up-projection [D][len] into columns [off, off + len) of the layer's head-major [H][R][64]
// up-projection matrix.
bool load_up(Reader& r, float* w2cat, int len, int off) {
    const size_t count = (size_t)M.D * len;
    if (!r.read_to(g_tmp, count)) return false;
    k_rw_put_up<<<(unsigned)((count + 255) / 256), 256>>>(g_tmp, M.D, len, M.R, off, w2cat);
    return cudaDeviceSynchronize() == cudaSuccess;
}

// 0 = Mamba (.rbin v1/v2), 1 = RWKV-7, -1 = unreadable.
int peek_kind(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return -1;
    uint32_t w[10] = {};
    size_t got = fread(w, 4, 10, f);
    fclose(f);
    if (got != 10) return -1;
    return (w[0] == kRbinMagic && w[1] == kVersion && (w[9] & kFlagRwkv7)) ? 1 : 0;
}

int load_weights(const char* path) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) {
        set_err("cannot open %s", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    uint32_t h[kHeaderWords];
    if (fread(h, 4, kHeaderWords, r.f) != (size_t)kHeaderWords || h[0] != kRbinMagic || h[1] != kVersion ||
        !(h[9] & kFlagRwkv7)) {
        set_err("%s: bad RWKV-7 .rbin header", path);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    M = Model();
    M.V = (int)h[2];
    M.D = (int)h[3];
    M.F = (int)h[4];
    M.H = (int)h[6];
    M.L = (int)h[8];
    M.flags = h[9];
    M.g1k = (h[9] & kFlagG1k) ? 1 : 0;
    const int ranks[4] = {(int)h[11], (int)h[12], (int)h[13], (int)h[14]};
    M.R = 0;
    for (int i = 0; i < 4; i++) {
        M.seg_off[i] = M.R;
        M.seg_len[i] = ranks[i];
        M.tiles_before[i + 1] = M.tiles_before[i] + (ranks[i] + kLoraRows - 1) / kLoraRows;
        M.R += ranks[i];
    }
    // Engine limits: head size 64, d and d_ffn multiples of 64 (int8 K slices), every LoRA rank
    // at least 1 and their sum within the k_rw_wkv shared-memory tile.
    if (h[5] != (uint32_t)kHS || (uint32_t)M.H * kHS != (uint32_t)M.D || M.D == 0 || M.D % 64 || M.D > 4096 ||
        M.F == 0 || M.F % 64 || M.F > 16384 || M.L == 0 || M.V == 0 || h[2] >= (1u << 30) || ranks[0] < 1 ||
        ranks[1] < 1 || ranks[2] < 1 || ranks[3] < 1 || M.R > kMaxR) {
        set_err("%s: RWKV-7 shape outside engine limits (V=%u D=%u F=%u N=%u H=%u L=%u R=%d)", path, h[2], h[3], h[4],
                h[5], h[6], h[8], M.R);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    const size_t D = M.D, F = M.F, V = M.V, R = M.R;
    const size_t per_layer = 10 * D + 3 * D + 2 * R * D + 3 * D + 4 * D * D + 3 * D + 2 * F * D;
    const size_t total = V * D + 2 * D + M.L * per_layer + 2 * D + V * D;
    fseek(r.f, 0, SEEK_END);
    long fsz = ftell(r.f);
    fseek(r.f, (long)(kHeaderWords * 4), SEEK_SET);
    if (fsz < 0 || (size_t)fsz != kHeaderWords * 4 + total * 4) {
        set_err("%s: size %ld does not match the header (%zu expected)", path, fsz, kHeaderWords * 4 + total * 4);
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    r.staging_n = (size_t)16 << 20;
    if (cudaHostAlloc(reinterpret_cast<void**>(&r.staging), r.staging_n * sizeof(float), cudaHostAllocDefault) !=
        cudaSuccess) {
        set_err("pinned staging allocation failed");
        return BACKEND_INIT_FAILED;
    }
    if (!dalloc(&g_tmp, std::max(std::max(V * D, D * D), std::max(F * D, R * D)), false)) {
        set_err("device staging allocation failed");
        return BACKEND_INIT_FAILED;
    }
    float* ln0 = nullptr;
    bool ok = model_alloc(&M.emb, V * D) && r.read_to(M.emb, V * D) && dalloc(&ln0, 2 * D, false) &&
              r.read_to(ln0, 2 * D);
    if (ok) {
        const size_t smem = 8 * D * sizeof(float);
        allow_smem(k_rw_emb_norm, smem);
        k_rw_emb_norm<<<(unsigned)((V + 7) / 8), 256, smem>>>(M.emb, M.V, M.D, ln0, ln0 + D);
        ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(ln0);
    M.layers.resize(M.L);
    const int lw = ranks[0], la = ranks[1], lv = ranks[2], lg = ranks[3];
    for (int i = 0; ok && i < M.L; i++) {
        Layer& Y = M.layers[i];
        ok = load_f32(r, &Y.ln1_w, D) && load_f32(r, &Y.ln1_b, D) && load_f32(r, &Y.ln2_w, D) &&
             load_f32(r, &Y.ln2_b, D) && load_f32(r, &Y.mix6, 6 * D) && model_alloc(&Y.w1cat, R * D) &&
             model_alloc(&Y.w2cat, D * R);
        ok = ok && load_f32(r, &Y.w0, D) && r.read_to(Y.w1cat, lw * D) && load_up(r, Y.w2cat, lw, M.seg_off[0]);
        ok = ok && load_f32(r, &Y.a0, D) && r.read_to(Y.w1cat + M.seg_off[1] * D, la * D) &&
             load_up(r, Y.w2cat, la, M.seg_off[1]);
        ok = ok && load_f32(r, &Y.v0, D) && r.read_to(Y.w1cat + M.seg_off[2] * D, lv * D) &&
             load_up(r, Y.w2cat, lv, M.seg_off[2]);
        ok = ok && r.read_to(Y.w1cat + M.seg_off[3] * D, lg * D) && load_up(r, Y.w2cat, lg, M.seg_off[3]);
        ok = ok && load_f32(r, &Y.k_k, D) && load_f32(r, &Y.k_a, D) && load_f32(r, &Y.r_k, D);
        ok = ok && load_w8(r, &Y.r, M.D, M.D) && load_w8(r, &Y.k, M.D, M.D) && load_w8(r, &Y.v, M.D, M.D) &&
             load_w8(r, &Y.o, M.D, M.D);
        ok = ok && load_f32(r, &Y.lnx_w, D) && load_f32(r, &Y.lnx_b, D) && load_f32(r, &Y.ffn_xk, D) &&
             load_w8(r, &Y.fk, M.F, M.D) && load_w8(r, &Y.fv, M.D, M.F);
    }
    ok = ok && load_f32(r, &M.ln_out_w, D) && load_f32(r, &M.ln_out_b, D) && load_w8(r, &M.head, M.V, M.D);
    cudaFree(g_tmp);
    g_tmp = nullptr;
    if (!ok) {
        set_err("%s: reading/uploading RWKV-7 weights failed (%s)", path, cudaGetErrorString(cudaGetLastError()));
        return BACKEND_WEIGHTS_NOT_FOUND;
    }
    G.V = M.V;
    G.d = M.D;
    G.nl = M.L;
    return BACKEND_OK;
}

// ---- One step -----------------------------------------------------------------------------------

W8Job job(const W8& m, const int8_t* aq, const float* as, float* out, int ldo, int epi) {
    return W8Job{m.q, m.s, m.rows, m.rows_pad, aq, as, out, ldo, epi};
}

template <int NS>
void w8_dp4a(const W8Args& wa, int njobs, int maxM, cudaStream_t st) {
    const size_t smem = (size_t)NS * wa.K;
    allow_smem(k_rw_w8a8_dp4a<NS>, smem);
    launch(k_rw_w8a8_dp4a<NS>, dim3((maxM + 15) / 16, (wa.n + NS - 1) / NS, njobs), dim3(256), smem, st, wa);
}

template <int BN>
void w8_tc(const W8Args& wa, int njobs, int maxM, cudaStream_t st) {
    const size_t smem = w8_smem<BN>();
    allow_smem(k_rw_w8a8_tc<BN>, smem);
    launch(k_rw_w8a8_tc<BN>, dim3((wa.n + BN - 1) / BN, (maxM + tc::kBM - 1) / tc::kBM, njobs), dim3(192), smem, st,
           wa, G.d_err);
}

bool use_tc(int n) { return G.proj_path == 2 || (G.proj_path == 0 && n >= kTcMinStreams); }

void project(const W8Args& wa, int njobs, cudaStream_t st) {
    int maxM = 0;
    for (int i = 0; i < njobs; i++) maxM = std::max(maxM, wa.job[i].M);
    const int n = wa.n;
    if (use_tc(n)) {
        if (n <= 16) w8_tc<16>(wa, njobs, maxM, st);
        else if (n <= 32) w8_tc<32>(wa, njobs, maxM, st);
        else w8_tc<64>(wa, njobs, maxM, st);
    } else {
        if (n == 1) w8_dp4a<1>(wa, njobs, maxM, st);
        else if (n == 2) w8_dp4a<2>(wa, njobs, maxM, st);
        else if (n <= 4) w8_dp4a<4>(wa, njobs, maxM, st);
        else w8_dp4a<8>(wa, njobs, maxM, st);
    }
}

W8Args w8args(int K, int n, const Pool& p) {
    W8Args wa{};
    wa.K = K;
    wa.n = n;
    wa.cap_pad = p.cap_pad;
    return wa;
}

int enqueue_step(Pool& p, int n, const uint32_t* d_slots, const uint32_t* d_tokens, float* d_out, bool probs,
                 cudaStream_t st) {
    // the first kernel checks the caller's slots and tokens; every later one reads the validated slots
    const RwStep sa0{n, (int)p.cap, p.cap_pad, M.V, d_slots, d_tokens, p.rflag, p.since, G.reset_every, G.d_err, p.vslot};
    const RwStep sa{n, (int)p.cap, p.cap_pad, M.V, p.vslot, d_tokens, p.rflag, p.since, G.reset_every, G.d_err, p.vslot};
    const int D = M.D, F = M.F;
    const size_t cap = p.cap;
    const size_t ln_smem = (size_t)D * sizeof(float);
    const dim3 ln_block(D / 4), q_grid(n);
    const size_t wkv_sm = wkv_smem(M.R);
    allow_smem(k_rw_ln_mix, ln_smem);
    allow_smem(k_rw_wkv, wkv_sm);
    allow_smem(k_rw_lora1, lora1_smem());
    int launches = 0;
    for (int li = 0; li < M.L; li++) {
        const Layer& Y = M.layers[li];
        float* x_att = p.x_att + (size_t)li * cap * D;
        float* x_ffn = p.x_ffn + (size_t)li * cap * D;
        float* wkv = p.wkv + (size_t)li * cap * M.H * kHS * kHS;
        {
            KScope k(kKNorm, st);
            LnMixArgs la{D, kLnTime, li == 0 ? M.emb : nullptr, p.x, Y.ln1_w, Y.ln1_b, x_att, Y.mix6,
                         p.aq0, p.aq1, p.aq2, p.as, p.lora_in};
            launch(k_rw_ln_mix, dim3(n), ln_block, ln_smem, st, li == 0 ? sa0 : sa, la);
        }
        {
            KScope k(kKInProj, st);
            W8Args wa = w8args(D, n, p);
            wa.job[0] = job(Y.r, p.aq0, p.as, p.rkv, D, kW8Store);
            wa.job[1] = job(Y.k, p.aq1, p.as + cap, p.rkv + cap * D, D, kW8Store);
            wa.job[2] = job(Y.v, p.aq2, p.as + 2 * cap, p.rkv + 2 * cap * D, D, kW8Store);
            project(wa, 3, st);
        }
        {
            KScope k(kKXProj, st);
            Lora1Args a1{};
            a1.D = D;
            a1.R = M.R;
            a1.layer0 = li == 0;
            a1.act_body = std::max(std::max(M.seg_len[0], M.seg_len[1]), std::max(M.seg_len[2], M.seg_len[3])) & ~7;
            for (int i = 0; i < 4; i++) {
                a1.seg_off[i] = M.seg_off[i];
                a1.seg_len[i] = M.seg_len[i];
            }
            for (int i = 0; i < 5; i++) a1.tiles_before[i] = M.tiles_before[i];
            a1.xin = p.lora_in;
            a1.w1cat = Y.w1cat;
            a1.h1 = p.h1;
            launch(k_rw_lora1, dim3(M.tiles_before[4], (n + kLoraStreams - 1) / kLoraStreams), dim3(256), lora1_smem(),
                   st, sa, a1);
        }
        {
            KScope k(kKScan, st);
            WkvArgs wk{};
            wk.D = D;
            wk.H = M.H;
            wk.R = M.R;
            wk.layer0 = li == 0;
            wk.g1k = M.g1k;
            for (int i = 0; i < 4; i++) {
                wk.seg_off[i] = M.seg_off[i];
                wk.seg_len[i] = M.seg_len[i];
            }
            wk.rkv = p.rkv;
            wk.h1 = p.h1;
            wk.w2cat = Y.w2cat;
            wk.w0 = Y.w0;
            wk.a0 = Y.a0;
            wk.v0 = Y.v0;
            wk.k_k = Y.k_k;
            wk.k_a = Y.k_a;
            wk.r_k = Y.r_k;
            wk.lnx_w = Y.lnx_w;
            wk.lnx_b = Y.lnx_b;
            wk.wkv = wkv;
            wk.v_first = p.v_first;
            wk.gated = p.gated;
            launch(k_rw_wkv, dim3(M.H, (n + kWkvSB - 1) / kWkvSB), dim3(kHS * kWkvSB), wkv_sm, st, sa, wk);
            launch(k_rw_quant, q_grid, dim3(256), 0, st, sa, (const float*)p.gated, D, p.aq0, p.as);
        }
        {
            KScope k(kKOutProj, st);
            W8Args wa = w8args(D, n, p);
            wa.job[0] = job(Y.o, p.aq0, p.as, p.x, D, kW8Add);
            project(wa, 1, st);
        }
        {
            KScope k(kKNorm, st);
            LnMixArgs lc{D, kLnChannel, nullptr, p.x, Y.ln2_w, Y.ln2_b, x_ffn, Y.ffn_xk,
                         p.aq0, nullptr, nullptr, p.as, nullptr};
            launch(k_rw_ln_mix, dim3(n), ln_block, ln_smem, st, sa, lc);
        }
        {
            KScope k(kKOutProj, st);
            W8Args wa = w8args(D, n, p);
            wa.job[0] = job(Y.fk, p.aq0, p.as, p.ffn, F, kW8ReluSq);
            project(wa, 1, st);
            launch(k_rw_quant, q_grid, dim3(256), 0, st, sa, (const float*)p.ffn, F, p.aq0, p.as);
            W8Args wv = w8args(F, n, p);
            wv.job[0] = job(Y.fv, p.aq0, p.as, p.x, D, kW8Add);
            project(wv, 1, st);
        }
        launches += 10;
    }
    {
        KScope k(kKNorm, st);
        LnMixArgs lf{D, kLnFinal, nullptr, p.x, M.ln_out_w, M.ln_out_b, nullptr, nullptr,
                     p.aq0, nullptr, nullptr, p.as, nullptr};
        launch(k_rw_ln_mix, dim3(n), ln_block, ln_smem, st, sa, lf);
    }
    float* lo = probs ? p.logits : d_out;
    {
        KScope k(kKHead, st);
        W8Args wa = w8args(D, n, p);
        wa.job[0] = job(M.head, p.aq0, p.as, lo, M.V, kW8Store);
        project(wa, 1, st);
    }
    launches += 2;
    if (probs) {
        KScope k(kKSoftmax, st);
        int parts = (M.V + kSoftmaxTile - 1) / kSoftmaxTile;
        launch(k_softmax_partial, dim3(parts, n), dim3(256), 0, st, (const float*)lo, M.V, p.red, parts);
        launch(k_softmax_final, dim3(std::max(1, std::min(64, M.V / 1024)), n), dim3(256), 0, st, (const float*)lo, M.V,
               (const float*)p.red, parts, d_out);
        launches += 2;
    }
    g_launches_per_step = launches;
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

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

int enqueue_pool_step(Pool& p, int n, bool probs) {
    const uint64_t key = graph_key(n, probs);
    if (!G.use_graphs || g_kt.on || !p.eager_done.count(key)) {
        int rc = enqueue_step(p, n, p.d_slots, p.d_tokens, p.logits, probs, G.stream);
        if (rc == BACKEND_OK) p.eager_done.insert(key);
        return rc;
    }
    auto it = p.graphs.find(key);
    if (it == p.graphs.end()) {
        cudaGraphExec_t exec = nullptr;
        int rc = capture_step(p, n, p.d_slots, p.d_tokens, p.logits, probs, &exec);
        if (rc != BACKEND_OK) return rc;
        it = p.graphs.emplace(key, exec).first;
    }
    CK(cudaGraphLaunch(it->second, G.stream), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

int pool_forward(Pool& p, uint32_t n, const uint32_t* slots, const uint32_t* tokens, float* out, bool probs) {
    std::fill(p.seen.begin(), p.seen.end(), 0);
    for (uint32_t b = 0; b < n; b++) {
        if (slots[b] >= p.cap || p.seen[slots[b]] || tokens[b] >= (uint32_t)M.V) return BACKEND_INVALID_ARGUMENT;
        p.seen[slots[b]] = 1;
        p.h_slots[b] = slots[b];
        p.h_tokens[b] = tokens[b];
    }
    const size_t ib = (size_t)n * sizeof(uint32_t);
    CK(cudaMemcpyAsync(p.d_slots, p.h_slots, ib, cudaMemcpyHostToDevice, G.stream), BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(p.d_tokens, p.h_tokens, ib, cudaMemcpyHostToDevice, G.stream), BACKEND_FORWARD_FAILED);
    int rc = enqueue_pool_step(p, (int)n, probs);
    if (rc != BACKEND_OK) return rc;
    CK(cudaMemcpyAsync(out, p.logits, (size_t)n * M.V * sizeof(float), cudaMemcpyDeviceToHost, G.stream),
       BACKEND_FORWARD_FAILED);
    CK(cudaMemcpyAsync(p.h_err, G.d_err, sizeof(uint32_t), cudaMemcpyDeviceToHost, G.stream), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    if (*p.h_err) {
        set_err("device error word 0x%x (2 = a tensor-core pipeline wait timed out)", *p.h_err);
        cudaMemset(G.d_err, 0, sizeof(uint32_t));
        return BACKEND_FORWARD_FAILED;
    }
    return BACKEND_OK;
}

// Rwkv7State::reset (model.rs:136-141) of the listed slots (all slots when `slots` is null), and
// the periodic-reset counter.
__global__ void k_rw_zero_slots(const uint32_t* __restrict__ slots, int cap, int L, int D, int HNN, float* x_att,
                                float* x_ffn, float* wkv, float* v_first, uint32_t* since) {
    const uint32_t slot = slots[blockIdx.y];
    if (slot >= (uint32_t)cap) return;
    const int l = blockIdx.z;
    const size_t ls = (size_t)l * cap + slot;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < HNN; i += gridDim.x * blockDim.x) {
        wkv[ls * HNN + i] = 0.0f;
        if (i < D) {
            x_att[ls * D + i] = 0.0f;
            x_ffn[ls * D + i] = 0.0f;
            if (l == 0) v_first[(size_t)slot * D + i] = 0.0f;
        }
        if (i == 0 && l == 0) since[slot] = 0u;
    }
}

int pool_reset(Pool& p, const uint32_t* slots, uint32_t n) {
    const size_t cap = p.cap, D = M.D, L = M.L, HNN = (size_t)M.H * kHS * kHS;
    if (!slots) {
        CK(cudaMemsetAsync(p.x_att, 0, L * cap * D * 4, G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.x_ffn, 0, L * cap * D * 4, G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.wkv, 0, L * cap * HNN * 4, G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.v_first, 0, cap * D * 4, G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaMemsetAsync(p.since, 0, cap * 4, G.stream), BACKEND_FORWARD_FAILED);
        CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
        return BACKEND_OK;
    }
    for (uint32_t b = 0; b < n; b++) {
        if (slots[b] >= p.cap) return BACKEND_INVALID_ARGUMENT;
        p.h_slots[b] = slots[b];
    }
    if (n == 0) return BACKEND_OK;
    CK(cudaMemcpyAsync(p.d_slots, p.h_slots, (size_t)n * 4, cudaMemcpyHostToDevice, G.stream), BACKEND_FORWARD_FAILED);
    k_rw_zero_slots<<<dim3(8, n, M.L), 256, 0, G.stream>>>(p.d_slots, (int)p.cap, M.L, M.D, (int)HNN, p.x_att, p.x_ffn,
                                                          p.wkv, p.v_first, p.since);
    CK(cudaGetLastError(), BACKEND_FORWARD_FAILED);
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// Device-resident step on the caller's stream (graphs keyed by the caller's pointers).
std::map<DevKey, cudaGraphExec_t> dev_graphs;
std::set<DevKey> dev_eager;

void clear_graphs() {
    for (auto& kv : dev_graphs) cudaGraphExecDestroy(kv.second);
    dev_graphs.clear();
    dev_eager.clear();
    for (Pool* p : {&M.v1, &M.batch}) {
        for (auto& kv : p->graphs) cudaGraphExecDestroy(kv.second);
        p->graphs.clear();
    }
}

int forward_device(uint32_t n, const uint32_t* d_slots, const uint32_t* d_tokens, float* d_out, bool probs,
                   cudaStream_t st) {
    DevKey k{graph_key((int)n, probs), d_slots, d_tokens, d_out};
    if (!G.use_graphs || g_kt.on || !dev_eager.count(k)) {
        int rc = enqueue_step(M.batch, (int)n, d_slots, d_tokens, d_out, probs, st);
        if (rc == BACKEND_OK) dev_eager.insert(k);
        return rc;
    }
    auto it = dev_graphs.find(k);
    if (it == dev_graphs.end()) {
        if (dev_graphs.size() >= 64) clear_graphs();
        cudaEvent_t ev;
        CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), BACKEND_FORWARD_FAILED);
        cudaEventRecord(ev, st);
        cudaStreamWaitEvent(G.stream, ev, 0);
        cudaEventDestroy(ev);
        cudaGraphExec_t exec = nullptr;
        int rc = capture_step(M.batch, (int)n, d_slots, d_tokens, d_out, probs, &exec);
        if (rc != BACKEND_OK) return rc;
        it = dev_graphs.emplace(k, exec).first;
    }
    CK(cudaGraphLaunch(it->second, st), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// State of one slot in the reference's layout (Rwkv7State, model.rs:113-120).
int get_state(uint32_t slot, float* x_att, float* wkv, float* x_ffn, float* v_first) {
    Pool* p = &M.batch;
    if (slot == 0xffffffffu) {
        p = &M.v1;
        slot = 0;
    }
    if (slot >= p->cap) return BACKEND_INVALID_ARGUMENT;
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    const size_t D = M.D, cap = p->cap, HNN = (size_t)M.H * kHS * kHS;
    std::vector<float> tmp(HNN);
    for (int l = 0; l < M.L; l++) {
        const size_t ls = (size_t)l * cap + slot;
        if (x_att)
            CK(cudaMemcpy(x_att + l * D, p->x_att + ls * D, D * 4, cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
        if (x_ffn)
            CK(cudaMemcpy(x_ffn + l * D, p->x_ffn + ls * D, D * 4, cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
        if (wkv) {
            CK(cudaMemcpy(tmp.data(), p->wkv + ls * HNN, HNN * 4, cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
            float* dst = wkv + l * HNN;
            for (int h = 0; h < M.H; h++)
                for (int i = 0; i < kHS; i++)
                    for (int j = 0; j < kHS; j++)
                        dst[((size_t)h * kHS + i) * kHS + j] = tmp[(size_t)h * kHS * kHS + ((j >> 2) * kHS + i) * 4 + (j & 3)];
        }
    }
    if (v_first)
        CK(cudaMemcpy(v_first, p->v_first + (size_t)slot * D, D * 4, cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

// which: 0 receptance, 1 key, 2 value, 3 output, 4 FFN key, 5 FFN value, 6 head; scales per row.
int get_q8(int which, uint32_t layer, int8_t* q, float* scales) {
    const W8* m = nullptr;
    if (which == 6) m = &M.head;
    else if (which >= 0 && which < 6 && layer < (uint32_t)M.L) {
        const Layer& Y = M.layers[layer];
        const W8* t[6] = {&Y.r, &Y.k, &Y.v, &Y.o, &Y.fk, &Y.fv};
        m = t[which];
    }
    if (!m) return BACKEND_INVALID_ARGUMENT;
    CK(cudaStreamSynchronize(G.stream), BACKEND_FORWARD_FAILED);
    if (q) {
        std::vector<int8_t> tiled((size_t)m->rows_pad * m->cols);
        CK(cudaMemcpy(tiled.data(), m->q, tiled.size(), cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
        for (int r = 0; r < m->rows; r++)
            for (int k = 0; k < m->cols; k++) q[(size_t)r * m->cols + k] = tiled[wq_off(m->rows_pad, r, k)];
    }
    if (scales) CK(cudaMemcpy(scales, m->s, (size_t)m->rows * 4, cudaMemcpyDeviceToHost), BACKEND_FORWARD_FAILED);
    return BACKEND_OK;
}

}  // namespace rwe
