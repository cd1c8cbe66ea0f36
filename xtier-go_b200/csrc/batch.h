// Internal interface of the batched verify step (batch.cu): S sequences over one weight set stepped together, every
// projection one tcgen05 GEMM over their 8 S activation rows (the weights read once per step for all of them), the
// attention per sequence over its own caches. Activation row 8 s + i is row i of sequence s; StepParams params[s]
// gives sequence s's tokens, rows and position.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "attention.h"

namespace xtg {

constexpr int kMaxBatch = 8;   // sequences per batched step: 64 activation rows, one GEMM activation tile

// One sequence's KV instance of one attention sublayer (layout in attention.h) and its ring's slot -> position table.
struct KvSeq {
  uint8_t* kc;
  uint8_t* vc;
  float* ks;
  float* vs;
  const int32_t* ring_pos;   // null for a global cache
  int64_t slots;
};

struct EmbedBatchArgs {
  const StepParams* params;   // [nseq]
  int nseq;
  const uint8_t* head;        // the tied NVFP4 head in tensor-core units
  int kblocks;
  float global;
  const uint16_t* table;      // or a BF16 embedding table [vocab][hidden] (a checkpoint's)
  int hidden;
  float* h;                   // [8 nseq][hidden]
  const float* inv_freq;      // [2][half]
  int rope_half;              // half the head dim: 64 (0 reads as 64) or 128
  float* rope_cos;            // [nseq][2][8][half]
  float* rope_sin;
  int32_t* const* ring_pos;   // [nseq] each sequence's table (null entries: no sliding layers)
  int64_t ring;
  uint8_t* act;               // h's digits as GEMM activation units (a prescale per row from its max)
  float* act_post;            // [64]
  int pdl;
};

// q | k | v | g projection rows (the GEMM's output, K split ksplit ways: parts split_stride floats apart) -> q
// (RoPE, justnorm, q scale), k (RoPE, justnorm), v, each k / v row stored into its sequence's cache (the KvCache::store
// rule) and kept unquantized for the attention's own keys.
struct QkvPrepArgs {
  const StepParams* params;
  int nseq;
  const float* proj;          // [8 nseq][proj_ld]
  int proj_ld, ksplit;
  int64_t split_stride;
  int heads, kv_heads;
  const float* rope_cos;      // [nseq][2][8][D / 2], this layer's theta at [s][theta]
  const float* rope_sin;
  int theta;
  const float* qscale;        // [heads * D]
  float* q_out;               // [8 nseq][heads][D]
  float* k_out;               // [8 nseq][kv_heads][D]
  float* v_out;
  const KvSeq* seqs;          // [nseq]
  int ring, dtype;
  int* err;                   // set (4) for a position outside its cache (nothing is written there)
  int pdl;
  int head_dim;               // D: 128 (0 reads as 128) or 256
};

// gate / up rows (interleaved tiles: columns 128 t + r, r < 64 gate feature 64 t + r, else up feature 64 t + r - 64)
// -> v = silu(g sg) (u su), justnorm'd over the features, as GEMM activation units for the down projection.
struct SwigluBatchArgs {
  const StepParams* params;
  int nseq;
  const float* gu;            // [8 nseq][2 features], K split ksplit ways: parts split_stride floats apart
  int ksplit;
  int64_t split_stride;
  int features;
  const float* sg;
  const float* su;
  uint8_t* act;               // GEMM activation units (one 64-row tile)
  float* act_post;            // [64]
  int pdl;
};

// logits rows [8 nseq][vocab] (x W^T times the head's global) times the per-token logit scale, in place, and each
// row's argmax (ties to the lowest index).
struct ScaleArgmaxArgs {
  const StepParams* params;
  int nseq;
  float* logits;
  int vocab;
  const float* logit_scale;
  int32_t* argmax;            // [8 nseq]
  uint32_t* epoch;            // optional: advanced once (the step's last kernel)
  int pdl;
};

// The nGPT residual update of every live row (slerp_residual, engine/src/kernels.cpp:177-189): h <- justnorm((1 - l)
// justnorm(h) + l justnorm(o)), o the sum of o_parts K-split partial outputs; the new h also as GEMM activation units
// (the unit prescale).
struct SlerpBatchArgs {
  const StepParams* params;
  int nseq;
  int hidden;
  float* h;                   // [8 nseq][hidden], updated in place
  const float* o;
  int o_parts;
  int64_t o_stride;
  const float* lr;            // [hidden]
  uint8_t* act;
  float* act_post;
  int pdl;
};

void launch_embed_batch(const EmbedBatchArgs& a, cudaStream_t s);
void launch_slerp_batch(const SlerpBatchArgs& a, cudaStream_t s);
void launch_qkv_prep(const QkvPrepArgs& a, cudaStream_t s);
void launch_swiglu_batch(const SwigluBatchArgs& a, cudaStream_t s);
void launch_scale_argmax(const ScaleArgmaxArgs& a, cudaStream_t s);

}  // namespace xtg
