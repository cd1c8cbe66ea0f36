// Internal interface between libxtg_cuda's host code and its sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xtg {

// ---- the NVFP4 streaming layout (weights.cu) ----
constexpr int kBlockBytes = 576;   // 16 rows x 64 inputs: 512 code bytes + 64 scale bytes
inline int packed_blocks(int k) { return (k + 63) / 64; }
inline int packed_tiles(int n_out, bool interleave) { return interleave ? (n_out + 7) / 8 : (n_out + 15) / 16; }
inline int64_t packed_bytes(int n_out, int k, bool interleave) {
  return (int64_t)packed_tiles(n_out, interleave) * packed_blocks(k) * kBlockBytes;
}

void gen_normal_bf16(uint64_t seed, uint64_t stream, float stddev, uint16_t* out, int64_t n, cudaStream_t s);
void gen_uniform(uint64_t seed, uint64_t stream, float lo, float hi, float* out, int64_t n, cudaStream_t s);
void gen_int8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n, cudaStream_t s);
void quantize_nvfp4(const uint16_t* w, int n_out, int k, uint8_t* codes, uint8_t* scales, float* global_out,
                    unsigned int* amax_scratch, cudaStream_t s);
void pack_nvfp4(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b, const uint8_t* scales_b,
                int n_out, int k, bool interleave, uint8_t* dst, cudaStream_t s);
void unpack_nvfp4(const uint8_t* src, int n_out, int k, uint8_t* codes, uint8_t* scales, cudaStream_t s);

// ---- the GEMV (gemv.cu) ----
// Where a tile's 16 output rows go (STORE epilogue): y[n * ld + r] for activation row n, tile row r < rows.
struct TileOut {
  float* y;
  int ld;
  int rows;
  float global;
  int pad;
};

enum GemvEpi { kEpiStore = 0, kEpiSwiglu = 1, kEpiHead = 2 };

struct ArgCand {   // the best logit of a tile for one activation row
  float v;
  int i;
};

struct GemvArgs {
  const uint8_t* w;          // streaming-layout blocks
  int tiles, blocks;         // tiles of 16 rows, 64-input blocks per tile
  const uint32_t* x16;       // activations, fp16 B fragments: [blocks * 4 steps][32 lanes][2 words]
  const int* m_dev;          // activation rows (1..8) read on the device (a replayable graph), or null: m
  int m;
  float* partial;            // [total warps][2][32 lanes][4] split-K parts
  int* counters;             // [tiles], zero between launches (the finishing warp resets its tile's)
  // kEpiStore
  const TileOut* outs;       // [tiles]
  const float* sumsq;        // optional: y *= 1 / sqrt(sum_p sumsq[p][n] + 1e-6), p < nparts (a justnorm of x)
  int nparts;
  // kEpiSwiglu (interleaved gate / up tiles of 8 features)
  float g_gate, g_up;
  const float* sg;
  const float* su;
  int features;              // F
  uint16_t* v16;             // fragments of v = silu(g * sg) * (u * su) for the next GEMV (K = F)
  float* vsum;               // [tiles][8] sum over the tile's features of v^2
  float* vout;               // optional f32 v [n][F]
  // kEpiHead
  float g_head;
  const float* logit_scale;  // [vocab]
  float* logits;             // [n][vocab]
  int vocab;
  ArgCand* cand;             // [tiles][8]
  int* err;                  // set to 1 if a bounded wait gave up (never expected); may be null
  int pdl;                   // launched as a programmatic dependent
};

int gemv_grid(int num_sms);
int64_t gemv_partial_floats(int grid);
void launch_gemv(int epi, const GemvArgs& a, int max_grid, cudaStream_t s, bool pdl);

// x f32 [m][k] -> fp16 fragments (rows >= m zero); k padded to the blocks of 64.
void pack_activations(const float* x, int m, int k, uint32_t* x16, cudaStream_t s);

}  // namespace xtg
