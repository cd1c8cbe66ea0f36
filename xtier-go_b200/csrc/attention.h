// Internal interface of the attention kernels (attention.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xtg {

enum KvDtype { kKvInt8 = 0, kKvFp8 = 1 };

// ---- the cache layout of one instance (slots a multiple of 64; head dim D 128 or 256; codes 8-bit, scales f32
// [kv_heads][slots]) ----
// K: [kv_heads][slots][D], each 128-dim half of a row as 8 16-byte units, unit u of slot s's half stored at unit
//    u ^ swz_k(s % 64);
// V: [kv_heads][slots / 64][D][64] (a 64-slot chunk of a head is one contiguous D x 64 block, head dim d its row),
//    the 16-byte unit u (slots 16 u .. 16 u + 15 of the chunk) of row d stored at unit u ^ ((d >> 1) & 3).
// The XORs make the attention kernel's fragment reads from shared memory bank-conflict free; a chunk of K, V and
// its scales are contiguous so that each arrives in one bulk copy.
__host__ __device__ __forceinline__ int swz_k(int s64) { return (s64 ^ (s64 >> 3)) & 7; }

__host__ __device__ __forceinline__ int64_t k_offset(int h, int64_t slot, int d, int64_t slots, int D = 128) {
  return ((int64_t)h * slots + slot) * D + 128 * (d >> 7) + 16 * (((d >> 4) & 7) ^ swz_k((int)(slot & 63))) +
         (d & 15);
}

__host__ __device__ __forceinline__ int64_t v_offset(int h, int d, int64_t slot, int64_t slots, int D = 128) {
  return (((int64_t)h * (slots / 64) + slot / 64) * D + d) * 64 + 16 * ((int)((slot & 63) >> 4) ^ ((d >> 1) & 3)) +
         (slot & 15);
}

// The per-step values a replayable graph reads on the device.
struct StepParams {
  int32_t tokens[8];
  int32_t m;
  // this sequence's rows of the step before these m (a prompt chunk's earlier 8-row groups; 0 in a verify step): the
  // cache is read below pos0 - own_rows, and those rows' keys are this call's own keys, scored unquantized
  int32_t own_rows;
  int64_t pos0;
};

// Batch-1 split-KV across GPUs with the exchange inside the combine kernel (world > 1): each process attends its
// share of the global cache's chunks and merges its own splits; each combine CTA then stores its (row, head)'s merged
// partial (max m, sum l, o[128]) into every peer's exchange slots as 64-bit words that carry the step's sequence
// number beside each value -- a word is complete once its number is right, so no fence or flag is needed -- reads
// the peers' words from its own slots and merges all processes' partials in rank order, so that every process
// computes the same bits. Two slot sets alternate by the running global-layer count: a process one layer ahead never
// writes a slot that a slower one has still to read, since its next write to the same set needs the slower one's
// next layer.
constexpr int kMaxKvWorld = 8;
struct PeerXchg {
  uint64_t* slot[kMaxKvWorld];   // by rank: that process's slots [2][world][8 rows][heads][130]
  const uint32_t* epoch;         // steps completed here (the step's last kernel advances it)
  uint64_t wait_ns;              // bound on waiting for a peer's words
  int world, rank;               // world 0 or 1: off
  int g, n_g;                    // this layer's index among the step's n_g global layers
};

struct KvSeq;   // batch.h

struct AttnArgs {
  // this call's rows, prepared (RoPE, justnorm, q scale): q [m][heads][D], k / v [m][kv_heads][D] (already in the
  // cache at positions pos0 .. pos0 + m - 1; the scores against them use these unquantized rows)
  const float* q;
  const float* k;
  const float* v;
  // the cache (layout in attention.cu)
  uint8_t* kc;
  uint8_t* vc;
  float* ks;
  float* vs;
  int64_t slots;
  int ring;
  const int32_t* ring_pos;  // [slots] for a ring
  int dtype;
  int window;
  float scale;
  const StepParams* params; // m and pos0 on the device, or null: m, pos0
  int m;
  int64_t pos0;
  int heads, kv_heads;
  int splits;               // CTAs per KV head in this launch
  // The chunks of the cache are cut into splits_total parts; this launch computes parts split0 .. split0 + splits - 1
  // (another process may compute the rest: the batch-1 split-KV over GPUs). 0 / 0: split0 0, splits_total = splits.
  int split0, splits_total;
  float* part;              // [splits_total][kv_heads][32][D + 4] (m, l, 2 pads, acc[D]), split-major (a process's
                            // splits are contiguous)
  int part_local;           // partials at index split (this launch's own) instead of split0 + split
  int* err;                 // set if a bounded wait gave up (never expected); may be null
  int pdl;
  // Several sequences in one launch (the batched step, grid z = sequence s): s's caches and ring table from seqs[s]
  // (kc ... ring_pos, slots above unused), its m and pos0 from params[s], its rows of q / k / v 8 s .. 8 s + 7, its
  // partials part_seq_stride floats after sequence s - 1's. null: one sequence.
  const KvSeq* seqs;
  int nseq;
  int64_t part_seq_stride;
  // the cache below pos0 is written by the kernel just before (a prompt chunk's row groups over one cache): its
  // chunks are copied only after the wait for that kernel, not before
  int late_copies;
  // the cache's chunks with the L2 evict_first policy (a global cache, read once per step; a ring stays in L2)
  int l2_first;
  int head_dim;             // D: 128 (0 reads as 128) or 256
};

struct CombineArgs {
  const float* part;
  // this call's rows (as in AttnArgs): the own-key scores are computed here in FP32
  const float* q;
  const float* k;
  const float* v;
  float scale;
  int window;
  int splits, heads, kv_heads;   // splits: every part of the cache's chunks (AttnArgs::splits_total)
  const StepParams* params;
  int m;
  float* out;               // API: [m][heads][D]; null in the step
  const float* gate;        // step: g rows [m][gate_ld] (the projection's g columns)
  int gate_ld;
  const float* gscale;      // [heads * D]
  uint8_t* ab;              // step: the gated output as B digits (the O projection's input, K = heads * D)
  float* ab_pre;            // [heads * D / 16][8] their prescales
  float* asum;              // step: [8][heads] sum of squares per activation row and head
  int pdl;
  PeerXchg x;               // split-KV across GPUs: splits are this process's, merged with the peers' here
  int* err;                 // set if the wait for a peer gave up
  // the batched step (grid z = sequence s, params[s], rows 8 s ..): the gated output in f32 (gated_out [8 S][heads *
  // 128]) and the per-head sums of squares (asum[h * asum_ld + 8 s + i]) instead of digits
  float* gated_out;
  int asum_ld;
  int nseq;
  int64_t part_seq_stride;
  int head_dim;             // D: 128 (0 reads as 128) or 256
  int prompt;               // the batched step of a prompt chunk: the sequences' own_rows may be non-zero
};

// CTAs of the attention kernel that fit on one SM at head dim D (2 at 128, 1 at 256)
int attention_ctas_per_sm(int head_dim);
int64_t attention_part_floats(int kv_heads, int splits, int head_dim = 128);
void launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
void launch_attn_combine(const CombineArgs& a, cudaStream_t s, bool pdl);

}  // namespace xtg
