// libxtg_cuda: the Dory looped-nGPT verify / decode step on one NVIDIA B200 (sm_100a), behind the C ABI of XTier
// Go's NPU plugin. Every session entry point below replaces the xtg_npu_* function of npu/xtg_npu.h cited beside
// it, with the same arguments, return values and error convention (0 / -1 with the reason in `err`, NULL from
// open), so packs/dory/npu.cpp's dlopen loader (npu.cpp:40-78) binds it with the prefix changed. One handle is one
// session: it owns the model's weights on the device, every KV instance, the ring's slot -> position table, the
// snapshots and the scratch. A handle is used by one thread at a time.
//
// The kernel-level entry points at the end are the device forms of the reference's CPU kernels (matmul_nvfp4,
// attention, KvCache::store, the NVFP4 quantizer) on caller-owned device memory, for parity checks and single-op
// benchmarks. They have no counterpart in xtg_npu.h.
#pragma once

#include <stdint.h>

#if defined(__GNUC__)
#define XTG_CUDA_API __attribute__((visibility("default")))
#else
#define XTG_CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct xtg_cuda xtg_cuda;

// row: index in this call's tokens; logits: vocab floats, valid during the callback (npu/xtg_npu.h:16-17)
typedef void (*xtg_cuda_logits_fn)(int row, const float* logits, void* user);

// Open a session (replaces xtg_npu_open, npu/xtg_npu.h:19-23). model_path: a Dory checkpoint directory (config.json +
// model.safetensors, ModelOpt W4A16_NVFP4), or "synthetic": the seeded synthetic Dory of options "model", built on
// the device. options: JSON, may be empty: "model" {hidden, ffn, heads, kv_heads, head_dim (128 | 256), vocab, n_in,
// n_rec, n_out, loops, window, ring, global_every, theta_sliding, theta_global, weight_std, lr_lo, lr_hi, qs_lo,
// qs_hi, gs_lo, gs_hi, suv_lo, suv_hi, ls_lo, ls_hi, kvs_lo, kvs_hi, seed} (synthetic only); "context" (tier,
// default 8192); "kv_dtype" ("int8" | "fp8", default int8);
// "snapshots" (ring snapshots kept, default 2); "decode_rows" (rows per step, 1..8, default 8); "device" (CUDA
// device, default 0); "graph" (1: replay the step as a CUDA graph, default 1); "pdl" (1: programmatic dependent
// launches, default 1). NULL on failure, the reason in err.
XTG_CUDA_API xtg_cuda* xtg_cuda_open(const char* model_path, const char* options, char* err, int err_len);

// No counterpart in xtg_npu.h, whose ABI is one session per handle: many sequences per device over one weight set.
// Open another session over `owner`'s weights on owner's device: its own KV instances, ring table,
// snapshots, activations, stream and step graph; the packed weights are shared, not copied (3.4 GB for the
// Dory-3072 shape). options as for xtg_cuda_open, except that "model" and "device" are the owner's and kv_world
// must be 1. The weights live until the last session over them is closed, whichever is closed first. Sessions are
// independent: each is used by one thread at a time, and several stepping at once from different threads run
// concurrently on the GPU. NULL on failure, the reason in err.
XTG_CUDA_API xtg_cuda* xtg_cuda_open_shared(xtg_cuda* owner, const char* options, char* err, int err_len);

// {"vocab", "context", "max_position", "prefill_ar", "decode_ar", "kv_instances", "ring_instances", "ring_slots",
//  "sliding_window", "kv_bytes", "snapshots", "kvmap", ...} as JSON; the length or -1 (xtg_npu.h:24-26).
XTG_CUDA_API int xtg_cuda_info(xtg_cuda* h, char* out, int out_len);

// Run n tokens at positions pos() .. pos() + n - 1 in steps of up to decode_rows rows. want: 0 no logits, 1 the
// last row, 2 every row. 0 on success; -1 with nothing changed for a token out of range or a full context
// (xtg_npu.h:27-29).
XTG_CUDA_API int xtg_cuda_forward(xtg_cuda* h, const int32_t* tokens, int n, int want, xtg_cuda_logits_fn fn, void* user,
                     char* err, int err_len);

// No counterpart in xtg_npu.h: xtg_cuda_forward for nh sessions at once from one thread (a server's single engine
// thread). Session i runs n[i] tokens from tokens[i]. Each round enqueues every session's next step (up to its
// decode_rows tokens) on that session's own stream before waiting for any of them, so the steps run concurrently on
// the GPU; then each session commits its step and the callback gets its rows, session by session, numbered across
// the call: session i's row j is base_i + j, base_i = n[0] + ... + n[i-1]. want as for xtg_cuda_forward. Every
// token and context check is made before the first step (a refused call changes nothing); a session may appear
// once. If a device wait times out in a session's step, that step is discarded, the round's other steps are
// committed and the call returns -1 after the round. A session given no tokens keeps its snapshots. The caller's
// current CUDA device is the same after the call. 0 on success.
XTG_CUDA_API int xtg_cuda_forward_batch(xtg_cuda* const* hs, int nh, const int32_t* const* tokens, const int* n,
                                       int want, xtg_cuda_logits_fn fn, void* user, char* err, int err_len);

XTG_CUDA_API int64_t xtg_cuda_pos(xtg_cuda* h);   // xtg_npu.h:30

// Back to n positions (n <= pos()). Global caches keep every position; the rings must still hold the window before
// n, else -1 and nothing changes. 0 on success (xtg_npu.h:31-33).
XTG_CUDA_API int xtg_cuda_rewind(xtg_cuda* h, int64_t n);

// Ring snapshots for the prefix cache (xtg_npu.h:34-39): remember the rings at pos() in a slot, go back to them
// later (pos() becomes the snapshot's). A forward below a snapshot's position drops it.
XTG_CUDA_API int xtg_cuda_snapshot_slots(xtg_cuda* h);
XTG_CUDA_API int64_t xtg_cuda_snapshot_pos(xtg_cuda* h, int slot);   // -1: empty
XTG_CUDA_API void xtg_cuda_snapshot(xtg_cuda* h, int slot);
XTG_CUDA_API int xtg_cuda_restore(xtg_cuda* h, int slot);            // 0 on success

// Move the session to another context tier (xtg_npu.h:40-43): tier is a context length ("4096", "8k", "32768",
// "32k"). The global caches' first pos() positions, the rings, the position and the snapshots that fit come along
// by device copies; nothing is computed again. On failure the session keeps its old tier and returns -1.
XTG_CUDA_API int xtg_cuda_grow(xtg_cuda* h, const char* tier, char* err, int err_len);

// Debugging (xtg_npu.h:44-46): a copy of KV instance `instance`'s K codes (value 0, [kv_heads][head_dim][slots],
// the NPU plugin's layout) or V codes (1, [kv_heads][slots][head_dim]), 8-bit; value 2 / 3: the K / V scales
// (f32 [kv_heads][slots]). Returns the size in bytes (out may be NULL), -1 for no such instance or value.
XTG_CUDA_API int64_t xtg_cuda_debug_cache(xtg_cuda* h, int instance, int value, void* out, int64_t len);

XTG_CUDA_API void xtg_cuda_close(xtg_cuda* h);   // xtg_npu.h:47

// ---- extensions (no counterpart in xtg_npu.h) ----

// The argmax of each row of the last step (the device lm_head's fused argmax; ties to the lowest index), n <= rows
// of that step. Returns the number of rows written or -1.
XTG_CUDA_API int xtg_cuda_argmax(xtg_cuda* h, int32_t* out, int n);

// The candidates of the reference's sampler for the rows of the last step, computed on the device from the logits
// still there (engine/src/sampler.cpp: more_likely 26-28, top_logprobs 30-40, the candidate phase of Sampler::sample
// 41-75): idx / logit [rows][k] the k most likely entries of each row, most likely first (ties: lowest index first),
// row_max [rows], total [rows] = sum over the whole row of exp((l - row_max) / temperature) in double (temperature
// <= 0: 1; at 1, log-sum-exp = row_max + log(total), so top_logprobs = logit - that). k in 1..min(1024, vocab).
// A caller reads rows x k candidates back instead of rows x vocab logits. Returns the number of rows or -1.
XTG_CUDA_API int xtg_cuda_topk(xtg_cuda* h, int k, float temperature, int32_t* idx, float* logit, float* row_max,
                               double* total, char* err, int err_len);

// xtg_cuda_topk on caller-owned device memory: logits [rows][vocab] f32 (vocab <= 131072); idx / logit [rows][k],
// row_max [rows], total [rows] on the device; enqueued on stream, not waited for. Returns 0 or -1.
XTG_CUDA_API int xtg_cuda_topk_rows(const float* logits, int rows, int vocab, int k, float temperature, int32_t* idx,
                                    float* logit, float* row_max, double* total, void* stream, char* err,
                                    int err_len);

// Sampler::sample's parameters (engine/include/xtg/sampler.h SamplingParams).
typedef struct {
  float temperature;   // <= 0: greedy
  int top_k;           // 0: off
  float top_p;         // 1: off
  float min_p;         // 0: off
} xtg_cuda_sampling;

// Host only (no device work): Sampler::sample (sampler.cpp:41-94) over one row's candidates from xtg_cuda_topk (k of
// them, fetched at p->temperature) with u, a uniform draw in [0, 1) from the caller's generator standing for the
// reference's uniform_real_distribution(0, total). Returns the token; -2 when the k candidates cannot decide (top_k
// above k, or top_p / min_p with k below min(vocab, 1024), or a top_p mass beyond the sorted 1024-entry head, where
// the reference sorts the whole row): the caller then samples from the full logits row; -1 on bad arguments.
XTG_CUDA_API int xtg_cuda_sample_candidates(const int32_t* idx, const float* logit, int k, float row_max, double total,
                                            int vocab, const xtg_cuda_sampling* p, double u);

// Seeded KV prefill: positions 0 .. n_past - 1 of every instance get the synthetic model's seeded codes and scales
// (the stream map of oracle/xtg_oracle.h); pos() becomes n_past, the ring table and snapshots are reset. -1 when
// n_past does not fit the tier.
XTG_CUDA_API int xtg_cuda_prefill_synthetic(xtg_cuda* h, int64_t n_past, char* err, int err_len);

// Device timing of `steps` verify steps of the m tokens at position pos() (each step re-verifies the same positions:
// the session rewinds between steps), with the step's inputs already on the device: the mean milliseconds per
// step from CUDA events on the session's stream. profile != 0 launches the step's kernels without the graph and
// times each kernel class instead: out_class_ms[c] and out_class_launches[c] for c = 0 GEMV (NVFP4), 1 attention,
// 2 attention combine, 3 residual / embedding / argmax (4 classes; may be NULL). Returns 0 or -1.
XTG_CUDA_API int xtg_cuda_bench(xtg_cuda* h, const int32_t* tokens, int m, int steps, int profile, double* out_ms_per_step,
                   double* out_class_ms, int64_t* out_class_launches, char* err, int err_len);

// Bytes each step streams (weights, KV read at the current position, activations), for the roofline: 0 all,
// 1 the NVFP4 GEMVs (weights + activations), 2 attention (KV read + q / out).
XTG_CUDA_API int64_t xtg_cuda_step_bytes(xtg_cuda* h, int what, int m);

// ---- kernel level: caller-owned device memory; stream is a cudaStream_t (NULL: the default stream) ----

typedef struct xtg_cuda_linear xtg_cuda_linear;

// The weights of one matmul_nvfp4 call (engine/include/xtg/kernels.h:28-31, engine/src/kernels.cpp:84-138): nw NVFP4
// weights in ModelOpt's layout (device pointers: codes [n_out_i][k / 2], scales [n_out_i][k / 16] E4M3, and the
// global scales as host floats), all reading the same x. Packed once into the GEMV's streaming layout.
XTG_CUDA_API xtg_cuda_linear* xtg_cuda_linear_new(int nw, const uint8_t* const* codes, const uint8_t* const* scales,
                                     const float* globals, const int* n_out, int k, char* err, int err_len);
// y_i[m][n_out_i] = x[m][k] W_i^T (x, ys: device f32): m <= 8 rows on the GEMV, more (a prefill chunk, a batch; up to
// 65536) on the tensor-core GEMM. One handle runs on one stream at a time.
XTG_CUDA_API int xtg_cuda_linear_forward(xtg_cuda_linear* w, const float* x, int m, float* const* ys, void* stream, char* err,
                            int err_len);
XTG_CUDA_API int64_t xtg_cuda_linear_bytes(xtg_cuda_linear* w);   // packed weight bytes streamed per call
XTG_CUDA_API void xtg_cuda_linear_free(xtg_cuda_linear* w);

// A checkpoint's BF16 lm_head: matmul_bf16 (engine/src/kernels.cpp:140-155) times the folded logit scale
// (packs/dory/dory.cpp:566-576) for m <= 8 rows, and each row's argmax (ties to the lowest index, sampler.cpp:8-13).
// Device pointers: x [m][hidden] f32, w [vocab][hidden] bf16 (both 16-byte aligned; hidden a multiple of 64, at most
// 5120), logit_scale [vocab], logits [m][vocab] (or NULL), argmax [m] int32 (or NULL). Waits for the result.
XTG_CUDA_API int xtg_cuda_head_bf16(const float* x, int m, const uint16_t* w, int vocab, int hidden,
                                    const float* logit_scale, float* logits, int32_t* argmax, void* stream, char* err,
                                    int err_len);

// The NVFP4 quantizer (device): bf16 [n_out][k] -> codes [n_out][k / 2], scales [n_out][k / 16], global (a device
// float). global = amax / (6 * 448); block scale = E4M3(amax_block / (6 * global)); nearest E2M1, ties to even.
XTG_CUDA_API int xtg_cuda_quantize_nvfp4(const uint16_t* w_bf16, int n_out, int k, uint8_t* codes, uint8_t* scales,
                            float* global, void* stream, char* err, int err_len);

// attention(pool, AttnArgs) (engine/include/xtg/kv.h:64-79, engine/src/kv.cpp:166-286) over a device KV cache in this
// library's layout (slots a multiple of 64; 16-byte aligned buffers):
//   K codes [kv_heads][slots][D]: each 128-dim half of slot s's row as 8 16-byte units, unit u of the half at unit
//     u ^ ((s % 64) ^ (s % 64 >> 3)) & 7;
//   V codes [kv_heads][slots / 64][D][64]: per 64-slot chunk, head dim d's row of 64 slots, its 16-byte unit u at
//     unit u ^ ((d >> 1) & 3);
//   scales f32 [kv_heads][slots].
// ring != 0: slot s holds position ring_pos[s] (int32, -1 empty), else slot = position. head_dim D 128 or 256, at
// most 4 q heads per KV head, n_q <= 8.
typedef struct {
  int n_q;
  int64_t pos0;
  int heads, kv_heads, head_dim, window;
  float scale;
  const float* q;           // [n_q][heads][head_dim]
  const float* k;           // [n_q][kv_heads][head_dim] this call's keys
  const float* v;
  const uint8_t* k_codes;
  const uint8_t* v_codes;
  const float* k_scales;
  const float* v_scales;
  int64_t slots;
  int ring;
  const int32_t* ring_pos;
  int dtype;                // 0 int8, 1 FP8 E4M3
  float* out;               // [n_q][heads][head_dim]
} xtg_cuda_attn_args;
XTG_CUDA_API int xtg_cuda_attention(const xtg_cuda_attn_args* a, int splits, void* stream, char* err, int err_len);

// No counterpart in the reference. xtg_cuda_attention for callers that cannot call cudaMalloc: a host runtime that
// reserved the GPU's memory for its own arena at start-up, or a path on which an allocation may not block or
// synchronise the device. The same kernels and results; the split-KV partials live in a fixed 4,325,376-byte array
// of this library, so kv_heads x splits must be at most 256 (larger requests fail with an error). It allocates
// nothing, enqueues both kernels on `stream` and returns without waiting. The array is held on every GPU that loads
// the library until the process exits; the first call on a device looks up its address there (make that call
// before any stream capture). Every call shares the array and it keeps the last call's contents: calls that
// overlap on the GPU (on different streams, or from several threads at once) race and corrupt each other's results.
XTG_CUDA_API int xtg_cuda_attention_noalloc(const xtg_cuda_attn_args* a, int splits, void* stream, char* err,
                                            int err_len);

// KvCache::store (engine/src/kv.cpp:75-112) into the layout above at head_dim 128: rows k, v [n][kv_heads][128]
// (device f32) at positions pos .. pos + n - 1; a ring keeps the last `slots`. int8: scale amax / 127; FP8: amax / 448
// (the reference's rule).
XTG_CUDA_API int xtg_cuda_kv_store(const float* k, const float* v, int64_t pos, int n, int kv_heads, int64_t slots, int ring,
                      int dtype, uint8_t* k_codes, uint8_t* v_codes, float* k_scales, float* v_scales, void* stream,
                      char* err, int err_len);

// The seeded generators (device; bit-identical with the oracle's xo_gen_*): what 0 normal bf16 (a = stddev),
// 1 uniform f32 in [a, b), 2 int8 in [-127, 127].
XTG_CUDA_API int xtg_cuda_gen(int what, uint64_t seed, uint64_t stream_id, float a, float b, void* out, int64_t n, void* stream,
                 char* err, int err_len);

#ifdef __cplusplus
}
#endif
