// Internal interface of the step's small kernels (elementwise.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attention.h"
#include "kernels.h"

namespace xtg {

struct EmbedArgs {
  const StepParams* params;
  const uint8_t* head;      // the tied NVFP4 head in tensor-core units
  int kblocks;              // 64-input blocks per row tile
  float global;
  const uint16_t* table;    // or a BF16 embedding table [vocab][hidden] (a checkpoint's): row t is token t's
  int hidden;
  float* h;                 // [8][hidden]
  uint8_t* xb;              // B digits of h
  float* xb_pre;            // [hidden / 16][8] their prescales
  const float* inv_freq;    // [n_thetas][half]
  int n_thetas;
  int rope_half;            // half the head dim: 64 (0 reads as 64) or 128
  float* rope_cos;          // [n_thetas][8][half]
  float* rope_sin;
  int32_t* ring_pos;        // null without sliding layers
  int64_t ring;
  int pdl;
};

enum ResidMode { kResidSlerp = 0, kResidLoopBegin = 1, kResidLoopNext = 2, kResidLoopEnd = 3 };

struct ResidArgs {
  int mode;
  const StepParams* params;
  int m;
  int hidden;
  float* h;                 // [8][hidden]: the residual stream, updated in place
  const float* o;           // slerp: the sublayer output [8][hidden]
  const float* lr;          // slerp: [hidden]
  float* state;             // loops: [8][hidden]
  float* input;
  uint8_t* xb;              // B digits of the new h
  float* xb_pre;            // [hidden / 16][8] their prescales
  // slerp, optional: the producer's per-CTA row sums (kernels.h GemvArgs::rsum) -- the update then runs over many
  // CTAs with no whole-row reduction
  const float* rsum;
  int nparts;
  int pdl;
  // the batched step (nseq > 0): row r is row r % 8 of sequence r / 8 (its m from params[r / 8]); o is the sum of
  // o_parts partial outputs o_stride floats apart (a K-split GEMM); xb null: no digits
  int nseq;
  int o_parts;
  int64_t o_stride;
  // the batched step: the new h's digits as GEMM activation units (fp4mma.cuh; the unit prescale for every row) and
  // each row's factor (1 / the prescale), or null
  uint8_t* gemm_act;
  float* gemm_post;
};

struct KvStoreArgs {
  const float* k;           // [n][kv_heads][128]
  const float* v;
  int64_t pos;
  int n;
  int kv_heads;
  int64_t slots;
  int ring;
  int dtype;
  uint8_t* kc;
  uint8_t* vc;
  float* ks;
  float* vs;
};

void launch_embed(const EmbedArgs& a, cudaStream_t s, bool pdl);
void launch_resid(const ResidArgs& a, cudaStream_t s, bool pdl);
// epoch (or null): the step counter of the split-KV exchange, advanced once by this, the step's last kernel
void launch_argmax(const ArgCand* cand, int tiles, const StepParams* params, int32_t* out, float* out_val,
                   uint32_t* epoch, cudaStream_t s, bool pdl);
void launch_kv_store(const KvStoreArgs& a, cudaStream_t s);
void kv_prefill(uint64_t seed, uint64_t stream_base, float lo, float hi, int64_t filled, int kv_heads, int hd,
                int64_t slots, uint8_t* kc, uint8_t* vc, float* ks, float* vs, cudaStream_t s);

}  // namespace xtg
