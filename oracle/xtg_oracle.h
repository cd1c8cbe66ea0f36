// TEST INFRASTRUCTURE ONLY: a CPU restatement of XTier Go's Dory verify step (the checker for libxtg_cuda, never
// linked into it or called by it). Plain C11 + OpenMP, built by oracle/Makefile into oracle/libxtg_oracle.so.
//
// Pinning: the pieces that exist in the reference are checked against the reference's own compiled kernels
// (oracle/_ref/libxtgref.so, built from its sources) and against the known answers of tests/kernels_test.cpp:
// number formats, nvfp4_row / matmul_nvfp4, justnorm / slerp / rope / swiglu, attention over an FP8 cache. Three
// pieces have no counterpart in the reference and are restated here from its analogous code; their parity is
// UNPINNED (no reference output exists to compare with): the NVFP4 quantizer (ModelOpt's published recipe), the int8
// KV encode (the FP8 rule of engine/src/kv.cpp:94-108 with 127 in place of 448), and the seeded synthetic
// generators. Ring / mask / rewind semantics follow npu/xtg_npu.cpp:236-291,362-369 and are bit-exact targets.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ---- number formats (engine/include/xtg/fp.h:10-41, engine/src/fp.cpp:12-49, engine/src/kv.cpp:20-40) ----
float xo_e4m3_to_f32(uint8_t b);
uint8_t xo_f32_to_e4m3(float f);          // round to nearest even, saturating to +-448, NaN -> 0x7f | sign
uint16_t xo_f32_to_bf16(float f);         // round to nearest even
float xo_bf16_to_f32(uint16_t h);
float xo_e2m1_to_f32(uint8_t nibble);

// ---- seeded synthetic generators (no reference counterpart; shared bit-for-bit with the device generator) ----
uint64_t xo_rand_bits(uint64_t seed, uint64_t stream, uint64_t index);
void xo_gen_normal_bf16(uint64_t seed, uint64_t stream, float stddev, uint16_t* out, int64_t n);
void xo_gen_uniform(uint64_t seed, uint64_t stream, float lo, float hi, float* out, int64_t n);
void xo_gen_int8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n);   // uniform in [-127, 127]

// ---- NVFP4 (engine/include/xtg/kernels.h:13-20; decode engine/src/kernels.cpp:34-60) ----
typedef struct {
  const uint8_t* codes;    // [n_out][k / 2], element 2j in the low nibble
  const uint8_t* scales;   // [n_out][k / 16] E4M3
  float global;
  int n_out, k;
} xo_nvfp4;

// The quantizer (ModelOpt recipe, restated; unpinned): global = amax / (6 * 448); per block of 16 along k the E4M3
// scale of amax_block / (6 * global); codes = nearest E2M1 of w / (scale * global), ties to the even code.
void xo_quantize_nvfp4(const uint16_t* w_bf16, int n_out, int k, uint8_t* codes, uint8_t* scales, float* global);
void xo_nvfp4_row(const xo_nvfp4* w, int row, float* out);
// y_i[m][n_out_i] = x[m][k] W_i^T, the reference's per-output order: per 16-group sum, times the block scale,
// summed over groups, times the global scale.
void xo_matmul_nvfp4(const xo_nvfp4* ws, int nw, const float* x, int m, float* const* ys);

// ---- elementwise (engine/src/kernels.cpp:162-234) ----
void xo_justnorm(float* x, int rows, int width);
void xo_slerp_residual(float* a, const float* b, const float* lr, int rows, int width);
void xo_rope(float* x, int rows, int heads, int head_dim, int64_t pos0, float theta);
void xo_swiglu_scaled(float* g, const float* u, const float* sg, const float* su, int rows, int width);

// ---- KV caches ----
// int8 (restated, unpinned): per (position, KV head) scale = amax / 127 (1 when amax is 0), code = rint(x / scale)
// clamped to +-127; decode = code * scale. fp8: the reference rule of engine/src/kv.cpp:94-108 (amax / 448, E4M3).
enum { XO_KV_I8 = 0, XO_KV_FP8 = 1 };
void xo_kv_encode(int dtype, const float* x, int d, uint8_t* codes, float* scale);
float xo_kv_decode(int dtype, uint8_t code, float scale);

// One attention instance's cache: a global cache (ring = 0, slot = position) or a ring of `slots` slots whose
// positions come from ring_pos (slot -> position, -1 empty; npu/xtg_npu.cpp:121). Rows [slots][kv_heads][d].
typedef struct {
  int dtype;
  int ring;
  int64_t slots;
  uint8_t* k;
  uint8_t* v;
  float* ks;     // [slots][kv_heads]
  float* vs;
} xo_cache;

// Attention of n_q rows at positions pos0 .. over the visible cached keys and this call's own keys (kv.cpp:166-286
// semantics; visibility npu/xtg_npu.cpp:249-256): a cached key at position p is visible to the row at t when
// p < pos0, and for a window when t - p < window; own key j is visible to own row i when j <= i (and i - j < window).
// Online softmax in 64-key tiles, FP32, like the reference.
typedef struct {
  int n_q;
  int64_t pos0;
  int heads, kv_heads, head_dim, window;
  float scale;
  const float* q;      // [n_q][heads][d]
  const float* k;      // [n_q][kv_heads][d] this call's keys
  const float* v;
  const xo_cache* cache;
  const int64_t* ring_pos;
  float* out;          // [n_q][heads][d]
} xo_attn;
void xo_attention(const xo_attn* a);

// The NPU session's masks for `rows` real rows of an `ar`-row step at n_past (npu/xtg_npu.cpp:236-258):
// mask [ar][ctx + ar], wmask [ar][ring + ar], 1 = visible, 0 = hidden.
void xo_fill_masks(int ar, int rows, int64_t n_past, int ctx, int ring, int window, const int64_t* ring_pos,
                   uint8_t* mask, uint8_t* wmask);
// Rewind validity (npu/xtg_npu.cpp:362-369): 1 when every position of the window before `to` is still in the ring.
int xo_rewind_ok(int64_t to, int64_t n_past, int window, int ring, const int64_t* ring_pos);

// ---- the Dory verify step (packs/dory/dory.cpp:467-544 order; loops unrolled with their own weights) ----
typedef struct {
  int kind;            // 0 MLP, 1 sliding attention, 2 global attention
  xo_nvfp4 w[5];       // attention: q, k, v, g, o; MLP: gate, up, down
  const float* lr;     // [hidden]
  const float* qscale; // [heads * d]
  const float* gscale; // [heads * d]
  const float* sg;     // [ffn]
  const float* su;     // [ffn]
  float theta;
  int cache;           // KV instance (attention)
} xo_layer;

typedef struct {
  int hidden, ffn, heads, kv_heads, head_dim, vocab, window;
  int n_in, n_rec, n_out, loops;   // layers[] holds n_in + n_rec * loops + n_out evaluations in order
  const xo_layer* layers;
  xo_nvfp4 head;                   // tied: row t is also token t's embedding
  const float* logit_scale;        // [vocab], folded (dory.cpp:326-327)
  // a checkpoint's (packs/dory/dory.cpp:322-325), or null: the BF16 embedding table [vocab][hidden] (bf16_row,
  // engine/src/kernels.cpp:157-160) and the untied BF16 lm_head [vocab][hidden] (matmul_bf16, kernels.cpp:140-155)
  const uint16_t* embed_bf16;
  const uint16_t* head_bf16;
} xo_model;

typedef struct {
  xo_cache* caches;
  int n_caches;
  int64_t* ring_pos;   // [ring]
  int ring;
  int64_t n_past;
} xo_state;

// One step of m rows at state->n_past: logits [m][vocab]; the new K / V rows go into the caches, ring_pos and
// n_past advance as npu/xtg_npu.cpp:266-291,343 do. work: at least xo_step_work_floats(model, m) floats.
int64_t xo_step_work_floats(const xo_model* model, int m);
void xo_step(const xo_model* model, xo_state* state, const int32_t* tokens, int m, float* logits, float* work);


// ---- the seeded synthetic Dory (no reference counterpart): the model and KV state the tests and benches use ----
// Physical sublayer l is attention when l is even, MLP when odd (the reference's alternation); attention sublayer
// a = l / 2 is global when a % global_every == global_every - 1 (Dory's "every 4th"), else sliding. Evaluations run
// the input sublayers, the recurrent ones `loops` times, then the output ones; every evaluation has its own weights
// (loops unrolled, as tools/npu_et/dory/model.py:287-297 exports them) and every attention evaluation its own KV
// instance (per_loop). Streams: evaluation e, slot s -> 1000 + 16 e + s (attention: q k v g o = 0..4, lr 8,
// qscale 9, gscale 10; MLP: gate up down = 0..2, lr 8, sg 11, su 12); head 1; logit scale 2; KV instance i:
// 500000 + 8 i + {k codes 0, v codes 1, k scales 2, v scales 3}.
typedef struct {
  int hidden, ffn, heads, kv_heads, head_dim, vocab;
  int n_in, n_rec, n_out, loops;
  int window, ring, global_every;
  float theta_sliding, theta_global, weight_std;
  float lr_lo, lr_hi, qs_lo, qs_hi, gs_lo, gs_hi, suv_lo, suv_hi, ls_lo, ls_hi, kvs_lo, kvs_hi;
  uint64_t seed;
} xo_synth_cfg;

int xo_synth_n_evals(const xo_synth_cfg* c);
int xo_synth_kind(const xo_synth_cfg* c, int eval);   // 0 MLP, 1 sliding, 2 global
xo_model* xo_synth_model_new(const xo_synth_cfg* c);
void xo_synth_model_free(xo_model* m);
// KV state with positions 0 .. n_prefill - 1 filled with seeded codes / scales (a ring holds the last `ring`).
xo_state* xo_synth_state_new(const xo_model* m, const xo_synth_cfg* c, int64_t ctx, int kv_dtype, int64_t n_prefill);
void xo_synth_state_free(xo_state* s);


// argmax, the first index of the largest value (engine/src/sampler.cpp:8-13)
int xo_argmax(const float* x, int n);

#ifdef __cplusplus
}
#endif
