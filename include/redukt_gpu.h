/*
 * redukt_gpu.h -- C ABI of libredukt_gpu.so, the B200 (sm_100a) backbone engine.
 *
 * The library is a drop-in for redukt's GPU backbone plugin: it exports the FFI v1 and v2
 * symbols with the reference's names, argument meaning and result codes, so the Rust host
 * (src/infrastructure/plugin_backend/loader.rs:157-216) loads it unchanged.  Everything after
 * the v2 block is additive: optional symbols an old host never looks up.
 *
 * Threading: like the reference plugin, one model per process (a global singleton), calls are
 * single-threaded and not reentrant (docs/api/PLUGIN-FFI-V2.md section 3).  Select the GPU of a
 * process with CUDA_VISIBLE_DEVICES; the host always passes device_id 0
 * (src/application/model_loader.rs:436).
 *
 * Plain C types only: no torch or CUDA types cross this boundary.
 */
#ifndef REDUKT_GPU_H
#define REDUKT_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Result codes: BackendResult, src/domain/backend_ffi.rs:25-41 (v2 adds 5). */
typedef enum {
    BACKEND_OK = 0,
    BACKEND_INIT_FAILED = 1,
    BACKEND_FORWARD_FAILED = 2,
    BACKEND_VERSION_MISMATCH = 3,
    BACKEND_WEIGHTS_NOT_FOUND = 4,
    BACKEND_INVALID_ARGUMENT = 5
} BackendResult;

#define BACKEND_FFI_VERSION 1 /* BackendInfo.ffi_version (src/domain/backend_ffi.rs:16) */
#define BACKEND_ABI_VERSION 2 /* redukt_backend_abi_version() (src/domain/backend_ffi.rs:19) */
#define BACKEND_NAME_MAX 64

/* BackendInfo, src/domain/backend_ffi.rs:61-72. */
typedef struct {
    uint32_t ffi_version;
    uint32_t vocab_size;
    uint32_t hidden_dim;
    uint8_t name[BACKEND_NAME_MAX];
} BackendInfo;

/* ---- FFI v1 (src/domain/backend_ffi.rs:91-114; plugins/redukt-gpu-cuda/mamba_cuda.cu:675-731) ---- */

/* Loads `weights_path` (a *.rbin file, or a directory holding model.rbin: mamba_cuda.cu:664-671)
 * onto device `device_id` and allocates the private single-stream state.  WEIGHTS_NOT_FOUND for
 * a missing/invalid file, INIT_FAILED for a CUDA failure.  Replaces mamba_cuda.cu:675-708.
 * Two model kinds: a Mamba .rbin (version 1/2, the reference plugin's format) or an RWKV-7 .rbin
 * (version 3 with flag bit 4, this engine's model-kind extension; W8A8 like the reference's
 * default RWKV-7 quantisation, src/infrastructure/rwkv7/model.rs:245).  Every entry point below
 * serves both kinds unless its comment says otherwise; BackendInfo.name says which is loaded
 * ("b200-mamba-*" or "b200-rwkv7-w8a8").  Mamba header flag bits 2/3 select the Q8 profile, and bit 6
 * (with bit 2) marks Q8 matrices stored as int8 + group scales in the file (no quantisation at load). */
BackendResult redukt_backend_init(const uint8_t* weights_path, int32_t device_id, BackendInfo* info_out);

/* One step of the v1 stream; writes vocab_size logits.  Replaces mamba_cuda.cu:710-715. */
BackendResult redukt_backend_forward(uint32_t token, float* out_logits, uint32_t vocab_size);

/* Zeroes the v1 stream's recurrent state.  Replaces mamba_cuda.cu:717-722. */
void redukt_backend_reset_state(void);

/* Releases every device allocation, including the batch pool.  Replaces mamba_cuda.cu:724-727. */
void redukt_backend_free(void);

/* ---- FFI v2 (src/domain/backend_ffi.rs:137-177; docs/api/PLUGIN-FFI-V2.md; mamba_cuda.cu:731-761) ---- */

/* Returns 2.  Replaces mamba_cuda.cu:731. */
uint32_t redukt_backend_abi_version(void);

/* (Re)allocates `max_streams` zeroed state slots (0 = release).  INVALID_ARGUMENT above 4096,
 * INIT_FAILED without a model or on allocation failure.  Replaces mamba_cuda.cu:733-745. */
int32_t redukt_backend_batch_init(uint32_t max_streams);

/* Zeroes the state (and the periodic-reset counter) of the listed slots; NULL = every slot.
 * Replaces mamba_cuda.cu:747-752. */
int32_t redukt_backend_batch_reset(const uint32_t* slots, uint32_t n_slots);

/* Advances each listed slot by one token and writes row b of out_logits [n_streams * vocab_size]
 * for batch position b.  Synchronous.  INVALID_ARGUMENT (vocab mismatch, n > pool, slot >= pool,
 * duplicate slot, token >= vocab, NULL pointer) returns before any launch with no state change.
 * A stream's logits are bit-identical for every batch size, batch position and slot.
 * Replaces mamba_cuda.cu:754-761. */
int32_t redukt_backend_forward_batch(uint32_t n_streams, const uint32_t* slots, const uint32_t* tokens,
                                     float* out_logits, uint32_t vocab_size);

/* ---- Additive extensions (optional symbols; absent from the reference) ---- */

/* Device-side periodic state reset: before a slot's token enters the model, the slot restarts
 * from zero state if it has run `every` forwards since its last reset (0 = never, the default).
 * The schedule is MambaState::maybe_periodic_reset (src/infrastructure/mamba/model.rs:315-320) and
 * PluginState::tick (src/infrastructure/plugin_backend/model.rs:44-49); a host that sets it must
 * stop calling batch_reset from its own tick.  Applies to the v1 stream and every batch slot. */
int32_t redukt_backend_set_reset_every(uint32_t every);

/* forward_batch that returns softmax probabilities (per row: exp(l - max) / sum) instead of
 * logits, computed on the device from the same logits; used for parity and benchmarks. */
int32_t redukt_backend_forward_batch_probs(uint32_t n_streams, const uint32_t* slots, const uint32_t* tokens,
                                           float* out_probs, uint32_t vocab_size);

/* forward_batch on device-resident inputs: d_slots/d_tokens/d_out are device pointers and the
 * work is enqueued on `cuda_stream` (a cudaStream_t, NULL = the library's stream) without a host
 * synchronisation.  Slots/tokens are checked on the device.  A bad entry (slot >= pool or
 * token >= vocab) sets bit 0 of the error word read by redukt_b200_device_error() and rejects only
 * its own stream: no state is read or written for it (its slot, if valid, keeps its state and its
 * periodic-reset counter bit for bit), its output row is all zeros (logits; with probs != 0 the row
 * is the uniform distribution), and every other stream of the call is computed as if the bad one
 * were absent.  Duplicate slots are the caller's responsibility.  probs != 0 writes probabilities
 * instead of logits. */
int32_t redukt_b200_forward_batch_device(uint32_t n_streams, const uint32_t* d_slots, const uint32_t* d_tokens,
                                         float* d_out, uint32_t vocab_size, int32_t probs, void* cuda_stream);

/* Reads and clears the device error word set by redukt_b200_forward_batch_device (0 = none). */
int32_t redukt_b200_device_error(uint32_t* out_word);

/* Copies one batch slot's recurrent state in the reference layout (MambaState,
 * src/infrastructure/mamba/model.rs:278-284): conv [n_layer][d_inner][d_conv-1] and
 * ssm [n_layer][d_inner][d_state].  Either pointer may be NULL.  slot = UINT32_MAX reads the v1 state. */
int32_t redukt_b200_get_state(uint32_t slot, float* conv, float* ssm);

/* Copies one quantised matrix as the engine holds it: which = 0 embedding, 1 head, 2 in_proj,
 * 3 out_proj (layer).  q [rows][cols] int8, scales [rows][cols/64] f32 (per-row scales repeated).
 * RWKV-7: which = 0 receptance, 1 key, 2 value, 3 output, 4 FFN key, 5 FFN value (layer), 6 head;
 * scales [rows] (Q8Tensor::from_f32, src/domain/tensor.rs:113-135). */
int32_t redukt_b200_get_q8(int32_t which, uint32_t layer, int8_t* q, float* scales);

/* RWKV-7 only: one slot's recurrent state in the reference layout (Rwkv7State,
 * src/infrastructure/rwkv7/model.rs:113-120): x_att [n_layer][d], wkv [n_layer][n_head][64][64],
 * x_ffn [n_layer][d], v_first [d].  Any pointer may be NULL.  slot = UINT32_MAX reads the v1 state.
 * INVALID_ARGUMENT when a Mamba model is loaded (use redukt_b200_get_state). */
int32_t redukt_b200_rwkv_get_state(uint32_t slot, float* x_att, float* wkv, float* x_ffn, float* v_first);

/* Model and engine facts: out[0..12] = vocab, d_model, d_inner, d_state, d_conv, dt_rank, n_layer,
 * flags, profile (0 F32, 1 Q8-g64, 2 Q8 per-row), pool capacity, reset_every, projection path,
 * kernel launches of the last enqueued step.  RWKV-7: words 2..5 are d_ffn, n_head, head size (64)
 * and the sum of the four LoRA ranks, and profile is 3 (W8A8). */
int32_t redukt_b200_info(uint32_t* out, uint32_t n);

/* Engine switches for tests and benchmarks:
 *   "proj_path"    0 = automatic, 1 = CUDA-core projections, 2 = tensor-core projections
 *   "graphs"       0/1 = replay each batch size's launch sequence from a captured CUDA graph
 *   "pdl"          0/1 = programmatic dependent launch between the step's kernels
 *   "split_target" CTAs a split-K tensor-core launch may use (0 = never split)
 *   "fused"        0/1 = run Q8 batches of up to 32 streams as one persistent step kernel
 *                  (only with proj_path 0; same bits as the per-kernel step)
 *   "head_ctas"    1 or 2 = tensor-core head tiles per SM at up to 64 streams (2: a 6-stage pipeline
 *                  so two CTAs share an SM; 1: the 12-stage tile of the other projections)
 *   "head_wide"    0/1 = above 16 streams, the head as 32-stream tensor-core tiles two CTAs per SM
 *                  (1, default) or 16-stream tiles up to 64 streams, then the layer projections'
 *                  tile choice (0); same bits
 *   "scan_blk"     0/1 = above 64 streams, scan blocks of 16-32 streams per CTA with the channel
 *                  group's weights staged once (1, default) or one stream per CTA (0); same bits
 *   "large_tile"   0/1 = above 256 streams, tensor-core tiles of 64 streams, one CTA per SM (0) or
 *                  of 32 streams, two CTAs per SM (1); same bits
 *   "f32_pairs"    0/1 = F32 projections of 8 or more streams on packed stream-pair FMAs with a
 *                  reduce-scatter butterfly (1, default) or the plain CUDA-core GEMV (0); same bits
 *   "conv_defer"   0/1 = outside the fused step, conv1d + SiLU runs in the x_proj kernel's staging
 *                  pass with in_proj storing the x-branch before the conv (1, default) or in the
 *                  in_proj epilogue (0); same bits
 *   "reset_counters" sets every batch slot's periodic-reset counter to `value` (forwards since its
 *                  last reset), e.g. to time the steps around a reset boundary without running the
 *                  window up to it; for benchmarks
 *   "wait_limit_us" limit of every bounded device wait in microseconds (0 = the defaults: 200 ms for
 *                  the fused step, about 2 s for the tensor-core pipelines); for tests
 *   "wait_test"    1 or 2 = make one bounded wait of the next step run out (1: the fused step's first
 *                  grid barrier misses one arrival; 2: a tensor-core projection tile misses one
 *                  activation copy); the step then returns FORWARD_FAILED with error-word bit 2
 *                  (fused) or bit 1 (tensor core) set and the device stays usable.  One-shot; for
 *                  tests of the error path
 * Returns INVALID_ARGUMENT for an unknown key or value. */
int32_t redukt_b200_set_option(const char* key, int64_t value);

/* Per-kernel-class device time: returns the CUDA-event time (ms) and launch count accumulated per
 * class since the previous call (0 embed, 1 norm, 2 in_proj, 3 x_proj, 4 scan, 5 out_proj, 6 head,
 * 7 softmax, 8 the fused small-batch step), then turns event bracketing on (enable != 0) or off.  While on, steps run without
 * CUDA graphs so each launch can be bracketed, and the per-kernel step replaces the fused one (class 8
 * stays 0).  Synchronises the device.  RWKV-7 classes: 1 the
 * LayerNorm/shift/quantise kernels, 2 the r/k/v projections, 3 the LoRA down-projections, 4 the WKV
 * head update and its quantisation, 5 the output and FFN projections, 6 head, 7 softmax. */
int32_t redukt_b200_kernel_times(int32_t enable, double* ms, uint32_t* launches, uint32_t n_classes);

/* Device time of one kernel class in isolation, in ms per launch: the class's launches of one
 * step for n streams (every layer; the embedding and head once) replayed as a CUDA graph after an
 * L2 flush, `reps` times.  cls as in redukt_b200_kernel_times (0-6, or 8: the fused step kernel, all
 * layers and the final norm in one launch, when it runs for n streams).  Needs a batch pool of at
 * least n slots and overwrites its scratch and the state of slots 0..n-1.  Mamba only. */
int32_t redukt_b200_time_kernel(int32_t cls, uint32_t n, uint32_t reps, float* ms_per_launch);

/* Softmax of n_rows rows of vocab logits, device memory in and out, with no allocation.
 * No counterpart in the reference: redukt's plugin ABI returns logits and the host does the
 * softmax.  This entry point is for callers that must not allocate device memory while they
 * run: code recording a CUDA graph (cudaMalloc cannot be captured), hosts that run on a fixed
 * device-memory budget or a caching allocator and forbid allocation on the decode path.
 * Its per-row scratch lives in a fixed array inside the library (256 KiB on every GPU that
 * loads it, held until the process exits), so it handles at most 1024 rows of at most 65536
 * logits; larger requests return INVALID_ARGUMENT.  Results are the same as the probability pass
 * of redukt_backend_forward_batch_probs.  Work is enqueued on cuda_stream (a cudaStream_t; NULL =
 * the legacy default stream) and not synchronised.  The first call on a device looks up the
 * array's address on that device; make that first call before any stream capture.  All calls
 * share the one array: calls whose work overlaps on the GPU (other streams, other threads)
 * race and must be serialised by the caller.  Needs no model loaded. */
int32_t redukt_b200_softmax_noalloc(const float* d_logits, uint32_t n_rows, uint32_t vocab, float* d_probs,
                                    void* cuda_stream);

/* The range coder's frequency table, computed on the device: for each of n_rows rows of vocab f32
 * logits, the vocab + 1 cumulative frequencies (cdf[0] = 0, cdf[vocab] = 2^24, every symbol >= 1)
 * that the reference host builds with cdf_from_logits_with(row, NumericContract::FmathV1)
 * (src/application/codec.rs:785-798: max, binary64 exp of fmath v1, sequential binary64 sum,
 * f32 probabilities) and Cdf::from_probs (src/domain/coder.rs:43-82).  Bit-identical to it.
 * It replaces the host CDF pass that follows the plugin's forward_batch
 * (src/application/lockstep.rs:315,330).
 * d_logits: device rows at stride ld_logits (>= vocab); d_cdf: device rows at stride ld_cdf
 * (>= vocab + 1), also used as the row's workspace.  Optional queries, three uint32 per row in
 * d_query_out (device): with d_symbols (encoder), {symbol, cdf[symbol], cdf[symbol + 1]}; with
 * d_cum_freqs (decoder), {Cdf::lookup(cum), cdf[sym], cdf[sym + 1]} (coder.rs:100-114); an
 * out-of-range symbol or a cum >= 2^24 gives {.., UINT32_MAX, UINT32_MAX}.  At most one of
 * d_symbols / d_cum_freqs.  Work is enqueued on cuda_stream (NULL = the legacy default stream),
 * not synchronised, and allocates nothing.  The first call on a device sets the kernel's
 * shared-memory limit (rows of up to 53,248 logits keep their workspace in shared memory): make it
 * before any stream capture.  INVALID_ARGUMENT when vocab is 0 or >= 2^24 or a stride is too
 * small.  Needs no model loaded. */
int32_t redukt_b200_cdf_device(const float* d_logits, uint32_t n_rows, uint32_t vocab, uint32_t ld_logits,
                               uint32_t* d_cdf, uint32_t ld_cdf, const uint32_t* d_symbols,
                               const uint32_t* d_cum_freqs, uint32_t* d_query_out, void* cuda_stream);

/* redukt_b200_cdf_device on host buffers (contiguous rows): copies the logits in, computes on the
 * library's stream, and copies back whatever is asked for: cdf_out (n_rows x (vocab + 1), may be
 * NULL) and, with symbols or cum_freqs (host), query_out (n_rows x 3).  Synchronous.  Device
 * buffers are kept by the library between calls and grown when a call needs more. */
int32_t redukt_b200_cdf(const float* logits, uint32_t n_rows, uint32_t vocab, uint32_t* cdf_out,
                        const uint32_t* symbols, const uint32_t* cum_freqs, uint32_t* query_out);

/* One lockstep step followed by the coder CDF of its logits, all on the device, with only the
 * coder's words coming back: forward_batch's slots/tokens (checked on the host, as forward_batch
 * does), then per stream r the query of redukt_b200_cdf_device on that step's logits row:
 * symbols[r] (encoder) or cum_freqs[r] (decoder) -> query_out[3r..3r+2].  cdf_out (NULL, or
 * n_streams x (vocab + 1)) also returns the whole tables; with neither query it is required.
 * This replaces forward_batch + the host's cdf_from_logits for each stream
 * (src/application/lockstep.rs:297-337, without the host CM ensemble): 12 bytes per stream come
 * back instead of vocab logits.  Synchronous, on the library's stream. */
int32_t redukt_b200_forward_batch_cdf(uint32_t n_streams, const uint32_t* slots, const uint32_t* tokens,
                                      const uint32_t* symbols, const uint32_t* cum_freqs, uint32_t* query_out,
                                      uint32_t* cdf_out);

/* Last error message of this library (empty string when none). */
const char* redukt_b200_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* REDUKT_GPU_H */
