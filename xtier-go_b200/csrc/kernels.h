// Internal interface between libxtg_cuda's host code and its sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xtg {

// ---- NVFP4 weights in tensor-core units (weights.cu; layouts in fp4mma.cuh) ----
// A weight [n_out][k] is cut into tiles of 128 rows and K blocks of 64 inputs; unit (t, b) is 4608 contiguous bytes
// (4096 code bytes in the MMA's A layout, 512 bytes of E4M3 scales in the scale-factor atom), units in tile-major
// order. An interleaved pack holds two weights of n_out rows (gate, up): tile t has rows 64 t .. 64 t + 63 of the
// first in tile rows 0-63 and the same rows of the second in tile rows 64-127.
constexpr int kPackTileRows = 128;
constexpr int kPackUnitBytes = 4608;
inline int packed_kblocks(int k) { return (k + 63) / 64; }
inline int packed_tiles(int n_out, bool interleave) { return interleave ? (n_out + 63) / 64 : (n_out + 127) / 128; }
inline int64_t packed_bytes(int n_out, int k, bool interleave) {
  return (int64_t)packed_tiles(n_out, interleave) * packed_kblocks(k) * kPackUnitBytes;
}
// activations as B digits (fp4mma.cuh): 1536 bytes per 64 inputs (4 digits of 8 rows, 1024 bytes, and a 512-byte
// scale atom)
constexpr int kDigitBlockBytes = 1536;
inline int64_t digit_bytes(int k) { return (int64_t)packed_kblocks(k) * kDigitBlockBytes; }
// the prescale of digits of a unit-norm vector (|x| <= 1): every group of the residual stream takes it
constexpr float kUnitPrescale = 2048.f;

void gen_normal_bf16(uint64_t seed, uint64_t stream, float stddev, uint16_t* out, int64_t n, cudaStream_t s);
void gen_uniform(uint64_t seed, uint64_t stream, float lo, float hi, float* out, int64_t n, cudaStream_t s);
void gen_int8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n, cudaStream_t s);
void quantize_nvfp4(const uint16_t* w, int n_out, int k, uint8_t* codes, uint8_t* scales, float* global_out,
                    unsigned int* amax_scratch, cudaStream_t s);
void pack_nvfp4(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b, const uint8_t* scales_b,
                int n_out, int k, bool interleave, uint8_t* dst, cudaStream_t s);

// ---- the GEMV (gemv.cu) ----
// Where a tile's 128 output rows go (STORE epilogue): y[n * ld + r] for activation row n, tile row r < rows; global
// scales of tile rows 0-63 and 64-127.
struct TileOut {
  float* y;
  int ld;
  int rows;
  float global_lo, global_hi;
};

enum GemvEpi { kEpiStore = 0, kEpiSwiglu = 1, kEpiHead = 2, kEpiQkv = 3 };

struct ArgCand {   // the best logit of a tile for one activation row
  float v;
  int i;
};

struct GemvArgs {
  const uint8_t* w;          // units [tiles][kblocks]
  int tiles, kblocks;
  // input: the B digits of the activations ([kblocks][1536], fp4mma.cuh) and the power-of-two prescale of every
  // 16-input group and row ([kblocks * 4][8])
  const uint8_t* xb;
  const float* xb_pre;
  float xb_fixed;            // > 0: every group's prescale is this (xb_pre is not read)
  const int* m_dev;          // activation rows (1..8) read on the device (a replayable graph), or null: m
  int m;
  // kEpiStore
  const TileOut* outs;       // [tiles]
  const float* sumsq;        // optional: y *= 1 / sqrt(sum_p sumsq[n][p] + 1e-6), p < nparts (a justnorm of x)
  int nparts;
  // kEpiSwiglu (interleaved gate / up tiles): v = silu(g * sg) * (u * su) as the next GEMV's digits (K = F)
  float g_gate, g_up;
  const float* sg;
  const float* su;
  int features;              // F
  uint8_t* vb;               // [tiles][1536]
  float* vb_pre;             // [tiles * 4][8]
  float* vsum;               // [8][tiles * split]: sums of v^2 over the features each CTA (part) finishes
  // kEpiQkv: the q | k | v | g projection of an attention sublayer, one 128-row tile per head (head_dim 128): tiles
  // [0, q_tiles) are q heads, then kv_tiles k heads, kv_tiles v heads, and the gate tiles (stored through `outs` as
  // kEpiStore does). q: RoPE, justnorm, times its q scale; k: RoPE, justnorm; k and v rows go into the KV cache and
  // out prepared (the attention's own rows).
  int q_tiles, kv_tiles;
  const float* rope_cos;     // [8][64] of this layer's theta (positions pos0 ..)
  const float* rope_sin;
  const float* qscale;       // [q_tiles * 128]
  float* q_out;              // [8][q_tiles][128]
  float* k_out;              // [8][kv_tiles][128]
  float* v_out;
  uint8_t* kc;
  uint8_t* vc;
  float* ks;
  float* vs;
  int64_t slots;
  int ring;
  int dtype;
  const int64_t* pos0_dev;
  // kEpiHead
  float g_head;
  const float* logit_scale;  // [vocab]
  float* logits;             // [n][vocab]
  int vocab;
  ArgCand* cand;             // [tiles][8]
  // kEpiStore, split tiles (split >= 4), optional: the row sums the nGPT residual update that follows needs, per CTA,
  // so that it reduces a few partials instead of whole rows. For the output dims y this CTA finishes (global index
  // tile * 128 + r) and activation row i: sums of h^2, y^2, (1 - lr)^2 h^2, lr (1 - lr) h y, lr^2 y^2 ->
  // rsum[(k * 8 + i) * grid + cta] (each sum's parts contiguous); h [8][rs_ld] is the residual stream the update
  // starts from
  float* rsum;
  const float* rs_h;
  const float* rs_lr;
  int rs_ld;
  int* err;                  // set to 1 if a bounded wait gave up (never expected); may be null
  int pdl;                   // launched as a programmatic dependent
  int l2_first;              // weight stages with the L2 evict_first policy (read once per step)
};

// How a GEMV is spread over the GPU: `split` CTAs (one cluster) share each tile's K blocks, or (split 1) each CTA
// takes tiles_per_cta whole tiles. ring: shared-memory stages of 4 units.
struct GemvPlan {
  int split = 1, tiles_per_cta = 1, grid = 1, ring = 3;
  int64_t smem = 0;
};
GemvPlan plan_gemv(int tiles, int kblocks, int num_sms, int max_split, int max_tiles_per_cta);
void launch_gemv(int epi, const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl);
// x f32 [m][k] (k a multiple of 16; rows m..7 zero) -> B digits xb [kblocks][1536] and prescales xb_pre [k / 16][8]
void digitize_rows(const float* x, int m, int k, uint8_t* xb, float* xb_pre, cudaStream_t s);

// ---- the BF16 lm_head of a checkpoint (head.cu) ----
constexpr int kMaxHeadBf16Hidden = 5120;   // x's two bf16 planes and the weight stages stay in shared memory
struct HeadBf16Args {
  const float* x;             // [8][hidden] the step's rows (rows >= m unused)
  const int* m_dev;           // rows read on the device (a replayable graph), or null: m
  int m;
  const uint16_t* w;          // [vocab][hidden] bf16
  int vocab, hidden;
  const float* logit_scale;   // [vocab], folded
  float* logits;              // [8][vocab] or null
  ArgCand* cand;              // [ceil(vocab / 128)][8] per-tile argmax candidates
  int* err;                   // set if a bounded wait gave up (never expected); may be null
};
void launch_head_bf16(const HeadBf16Args& h, int num_sms, cudaStream_t s, bool pdl);

// ---- the GEMM (gemm.cu): y[m][n] = x[m][k] W^T for prefill chunks and batches ----
constexpr int kMaxGemmRows = 65536;
// Activation units: [ceil(m / 64)][kblocks] of 9216 bytes (4 digits x 64 rows per unit) and a factor per row
// (1 / its power-of-two prescale, times an optional row scale).
int gemm_padded_rows(int m);   // rows of the activation tiles (a multiple of 64)
int64_t gemm_act_bytes(int m, int k);
// sumsq (optional): the row scale 1 / sqrt(sum_p sumsq[p * ld + row] + 1e-6) (a justnorm of x) goes into act_post
void gemm_digitize(const float* x, int m, int k, uint8_t* act, float* act_post, cudaStream_t s,
                   const float* sumsq = nullptr, int nparts = 0, int ld = 0, bool pdl = false);
// weights: the packed units of wtiles tiles; outs[t] as for the GEMV's STORE epilogue (y[row * ld + r]); ksplit > 1:
// each tile's K blocks in ksplit parts, part ks written split_stride floats further (partial sums)
void launch_gemm(const uint8_t* w, int wtiles, int kblocks, const uint8_t* act, const float* act_post, int m,
                 const TileOut* outs, int num_sms, int* err, cudaStream_t s, int ksplit = 1, int64_t split_stride = 0,
                 bool pdl = false);

}  // namespace xtg
