// K3: GQA decode / verify attention over an int8 (or FP8) KV cache, split-KV with a log-sum-exp combine
// (engine/src/kv.cpp:166-286 semantics; the visibility rule of npu/xtg_npu.cpp:236-258).
//
// Cache layout of one instance: attention.h (k_offset / v_offset). A 64-slot chunk of one KV head is three
// contiguous pieces -- 8 KB of K rows, 8 KB of V (head dim major), 256 B of each scale row -- streamed into shared
// memory by bulk copies (cp.async.bulk, completion on an mbarrier, no multicast) before the kernel waits on the
// previous one: the cached keys and values do not depend on it. Scales: one f32 per (position, KV head), amax / 127
// for int8, amax / 448 for FP8.
// A global instance's slot is the position; a ring's slot s holds position ring_pos[s] (-1 empty). A cached key at
// position p is visible to the row at t when 0 <= p < pos0 (and t - p < window for a sliding layer); this call's
// own key j is visible to own row i when j <= i (and i - j < window).
//
// One CTA per (split of the slots, KV head), 8 warps, two CTAs per SM. Every warp takes part in every 64-slot chunk:
// warp w takes query rows 16 (w & 1) .. +15 -- a query row is (activation row, q head of this KV head), 8 x 4 = 32
// rows, so the 4 q heads sharing a KV head read it once. For the scores it takes the chunk's keys 16 (w >> 1) .. +15;
// the 4 warps of a row half then share the chunk's row maxima and probabilities through shared memory, and for PV
// each takes a quarter of the head dims over all 64 keys, so that a chunk costs each warp a quarter of its products,
// its accumulator holds 16 rows x D / 4 dims, and the online-softmax state (running max, probability sums) is common
// to the row half: its partial needs no merge. The chunks stream through a 4-stage ring.
// QK^T over an int8 cache runs on mma.m16n8k32.s8 straight from the cached codes: Q (after RoPE, justnorm, q scale)
// becomes two signed 8-bit digits per element against its row's max |q| (q = max / 127 * (hi + lo / 254), ~16
// bits), the two integer products are exact and combine as 254 hi + lo before one conversion to FP32. Over an FP8
// cache both digits are fp16 (q = hi + lo, ~22 bits) and the codes become f16 (cvt.rn.f16x2.e4m3x2) for
// mma.m16n8k16. Scores are scaled per key by its K scale in FP32. PV runs on mma.m16n8k16: probabilities times the
// key's V scale are the fp16 A operand, int8 codes become f16 exactly (1152 + b as a half, less 1152). Two
// permutations make every load contiguous: the head dimension inside a k step (lane tq reads 32 contiguous bytes of
// a K row, Q's fragments use the same order) and the keys inside a warp's quarter (lane tq owns keys 4 tq .. 4 tq + 3
// in both products).
#include <algorithm>

#include "attention.h"
#include "batch.h"
#include "common.cuh"
#include "fp4mma.cuh"

namespace xtg {

namespace {

constexpr int kThreads = 256;   // 8 warps: (row half) x (key quarter)
constexpr int kQuarters = 4;    // key quarters of a chunk
constexpr int kStages = 4;      // chunks in flight
constexpr int kQRows = 32;
constexpr int kXchgStride = 128 + 2;   // a split-KV exchange slot: m, l, o[128] as 64-bit words (head dim 128)
constexpr int kMaxSplits = 256;        // parts of a cache's chunks (the combine holds one weight per part)
// a partial's floats at head dim D: m, l, 2 pads, acc[D] (the dims 16-byte aligned)
__host__ __device__ constexpr int part_stride(int D) { return D + 4; }

__device__ __forceinline__ void codes_to_f16(uint32_t word, int dtype, uint32_t& lo, uint32_t& hi) {
  if (dtype == kKvFp8) {
    lo = e4m3x2_to_f16x2(word & 0xffff);
    hi = e4m3x2_to_f16x2(word >> 16);
  } else {
    const uint32_t biased = word ^ 0x80808080u;
    lo = s8x2_to_f16x2(biased, 0x4140);
    hi = s8x2_to_f16x2(biased, 0x4342);
  }
}

template <int D>
struct Stage {                    // one 64-slot chunk of one KV head, as it lies in the cache
  uint8_t k[64 * D];
  uint8_t v[D * 64];
  float ks[64];
  float vs[64];
  int32_t pos[64];
};

template <int D>
struct Smem {
  Stage<D> stage[kStages];        // the chunk ring; after the last chunk, key quarter j's softmax state in stage[j]
  uint64_t full[kStages];
  int released[kStages];          // warps done with the stage's current chunk (the last one refills it)
  // Q A fragments. FP8 cache: [m-tile][hi, lo][k16 step][lane], q = hi + lo, both fp16. Int8 cache: the first half
  // as [m-tile][hi, lo][k32 step][lane] of signed 8-bit digits (qi below).
  uint4 qf[2][2][D / 16][32];
  float qmaxp[kQRows][D / 32];    // int8 cache: a query row's max |q| over the 8-dim pieces of one k32 step
  float qfac[kQRows];             // int8 cache: a query row's digit unit, max |q| / (127 * 254)
  float cmax[kQuarters][kQRows];  // a chunk's row maxima per key quarter
  uint2 pbuf[2][16][16];          // a chunk's P' per row half: [row][unit of 4 keys, swizzled] as fp16
  float lsum[kQuarters][kQRows];  // the probability sums per key quarter, at the end
};

// Head dim 256: the same warp roles over twice the dims (16 k16 steps, 32 n8 tiles of the output); the accumulator
// takes twice the registers and a stage twice the shared memory, so one CTA fits an SM.
template <int D, bool I8>
__global__ void __launch_bounds__(kThreads, D == 128 ? 2 : 1) attention_kernel(const AttnArgs a) {
  static_assert(D == 128 || D == 256, "head dim 128 or 256");
  constexpr int kSteps = D / 16;                          // k16 steps of QK^T
  constexpr int kPartStride = part_stride(D);
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3;
  const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
  const StepParams* prm = a.params ? a.params + seq : nullptr;
  const KvSeq* sq = a.seqs ? a.seqs + seq : nullptr;
  const int m = prm ? prm->m : a.m;
  const int pos0 = (int)(prm ? prm->pos0 : a.pos0);   // positions stay below 2^31
  // the cached keys this call reads lie below kend (a prompt chunk's earlier groups come in as own keys instead)
  const int kend = pos0 - (prm ? prm->own_rows : 0);
  const int64_t slots = sq ? sq->slots : a.slots;
  const int group = a.heads / a.kv_heads;
  const int32_t* ring_pos = sq ? sq->ring_pos : a.ring_pos;
  const float* aq = a.q + (int64_t)seq * kMaxRows * a.heads * D;
  // a sequence with no rows in this step (a batched step's idle group) reads nothing: its position may lie past its
  // cache
  if (m <= 0) return;

  // this CTA's 64-slot chunks: a global cache holds [0, pos0), a ring every slot
  const int64_t span = a.ring ? slots : kend;
  const int64_t nchunks = (span + 63) / 64;
  const int stot = a.splits_total > 0 ? a.splits_total : a.splits, sidx = a.split0 + split;
  const int64_t cb = nchunks * sidx / stot, ce = nchunks * (sidx + 1) / stot;
  const int nc = (int)(ce - cb);
  const uint8_t* kc = (sq ? sq->kc : a.kc) + (int64_t)kvh * slots * D;
  const uint8_t* vc = (sq ? sq->vc : a.vc) + (int64_t)kvh * D * slots;
  const float* ks = (sq ? sq->ks : a.ks) + (int64_t)kvh * slots;
  const float* vs = (sq ? sq->vs : a.vs) + (int64_t)kvh * slots;
  const uint32_t stage_bytes = 2 * 64 * D + 2 * 64 * 4 + (a.ring ? 64 * 4 : 0);
  // chunk i of this CTA into stage i % kStages, by lanes 0-4 of warp 0: one bulk copy per lane (the copies of one
  // thread complete one after another)
  auto issue = [&](int i) {
    Stage<D>& st = sm.stage[i % kStages];
    uint64_t* bar = &sm.full[i % kStages];
    const int64_t c = cb + i;
    if (c < 0 || (c + 1) * 64 > slots) {   // never: a chunk outside the cache is recorded, not read
      if (lane == 0 && a.err) atomicExch(a.err, 5);
      return;
    }
    if (lane == 0) mbar_expect_tx(bar, stage_bytes);
    __syncwarp();
    if (a.l2_first) {
      const uint64_t pol = l2_evict_first();
      if (lane == 0) bulk_g2s_hint(st.k, kc + c * 64 * D, 64 * D, bar, pol);
      if (lane == 1) bulk_g2s_hint(st.v, vc + c * 64 * D, 64 * D, bar, pol);
      if (lane == 2) bulk_g2s_hint(st.ks, ks + c * 64, 64 * 4, bar, pol);
      if (lane == 3) bulk_g2s_hint(st.vs, vs + c * 64, 64 * 4, bar, pol);
    } else {
      if (lane == 0) bulk_g2s(st.k, kc + c * 64 * D, 64 * D, bar);
      if (lane == 1) bulk_g2s(st.v, vc + c * 64 * D, 64 * D, bar);
      if (lane == 2) bulk_g2s(st.ks, ks + c * 64, 64 * 4, bar);
      if (lane == 3) bulk_g2s(st.vs, vs + c * 64, 64 * 4, bar);
    }
    if (lane == 4 && a.ring) bulk_g2s(st.pos, ring_pos + c * 64, 64 * 4, bar);
  };
  // the cached keys and values below pos0 do not depend on the previous kernel (this step writes positions pos0 ..
  // only): the first chunks go out now -- unless that kernel wrote some of them (late_copies)
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      sm.released[s] = 0;
    }
    mbar_init_fence();
  }
  __syncthreads();
  if (warp == 0 && !a.late_copies)
    for (int i = 0; i < kStages && i < nc; ++i) issue(i);
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  if (warp == 0 && a.late_copies)
    for (int i = 0; i < kStages && i < nc; ++i) issue(i);

  // ---- A fragments of the queries of this KV head (prepared: RoPE, justnorm, q scale), straight from memory, split
  // q = hi + lo (both fp16) so that the scores keep ~22 bits: step st, lane tq reads head dims
  // 128 (st >> 3) + 32 tq + 4 (st & 7) + {0, 1} (a0, a1) and + {2, 3} (a2, a3) of its rows gg and gg + 8 ----
  auto qrow = [&](int r, int d0) {   // 4 head dims of query row r (zeros for rows past m)
    const int i = r / group, hg = r % group;
    return i < m ? *reinterpret_cast<const float4*>(aq + ((int64_t)i * a.heads + kvh * group + hg) * D + d0)
                 : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  // int8 cache: the digit fragments of k32 step st (4 per 128-dim half), m-tile t2, lane (gg, t): rows gg and gg + 8
  // of the tile, head dims d0 .. d0 + 3 (registers x: row gg, y: row gg + 8) and d0 + 4 .. d0 + 7 (z, w), where
  // d0 = 128 (st >> 2) + 32 t + 8 (st & 3) -- the MMA's k index 4 t + i is head dim d0 + i, 16 + 4 t + i is d0 + 4 + i
  uint4 (*qi)[2][D / 32][32] = reinterpret_cast<uint4 (*)[2][D / 32][32]>(&sm.qf[0][0][0][0]);
  if constexpr (I8) {
    constexpr int kSt = D / 32;
    constexpr int kFrag = 2 * kSt * 32 / kThreads;   // (m-tile, k32 step, lane) fragments per thread
    float4 qv[kFrag][4];
#pragma unroll
    for (int u = 0; u < kFrag; ++u) {   // every load first
      const int idx = (int)threadIdx.x + u * kThreads;
      const int l = idx & 31, st = (idx >> 5) % kSt, t2 = idx / (32 * kSt), gg = l >> 2;
      const int d0 = 128 * (st >> 2) + 32 * (l & 3) + 8 * (st & 3);
      qv[u][0] = qrow(16 * t2 + gg, d0);
      qv[u][1] = qrow(16 * t2 + gg + 8, d0);
      qv[u][2] = qrow(16 * t2 + gg, d0 + 4);
      qv[u][3] = qrow(16 * t2 + gg + 8, d0 + 4);
    }
    // each row's max |q|: over the 4 lanes of a row within a fragment, then over the k32 steps through shared memory
#pragma unroll
    for (int u = 0; u < kFrag; ++u) {
      const int idx = (int)threadIdx.x + u * kThreads;
      const int l = idx & 31, st = (idx >> 5) % kSt, t2 = idx / (32 * kSt), gg = l >> 2;
      float mx[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float4 p = qv[u][h], r = qv[u][2 + h];
        mx[h] = fmaxf(fmaxf(fmaxf(fabsf(p.x), fabsf(p.y)), fmaxf(fabsf(p.z), fabsf(p.w))),
                      fmaxf(fmaxf(fabsf(r.x), fabsf(r.y)), fmaxf(fabsf(r.z), fabsf(r.w))));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
        mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      }
      if ((l & 3) == 0) {
        sm.qmaxp[16 * t2 + gg][st] = mx[0];
        sm.qmaxp[16 * t2 + gg + 8][st] = mx[1];
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kFrag; ++u) {
      const int idx = (int)threadIdx.x + u * kThreads;
      const int l = idx & 31, st = (idx >> 5) % kSt, t2 = idx / (32 * kSt), gg = l >> 2;
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {   // h: row gg (registers x, z) or gg + 8 (y, w)
        const int r = 16 * t2 + gg + 8 * h;
        float M = 0.f;
#pragma unroll
        for (int s2 = 0; s2 < kSt; ++s2) M = fmaxf(M, sm.qmaxp[r][s2]);
        const float inv = M > 0.f ? 127.f / M : 0.f;
        if (st == 0 && (l & 3) == 0) sm.qfac[r] = M * (1.f / (127.f * 254.f));
#pragma unroll
        for (int half = 0; half < 2; ++half) {   // dims d0 .. + 3 (x / y) and d0 + 4 .. + 7 (z / w)
          const float4 p = qv[u][h + 2 * half];
          const float v[4] = {p.x, p.y, p.z, p.w};
          uint32_t wh = 0, wl = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = v[e] * inv, xh = rintf(x);
            const int dh = (int)xh, dl = (int)rintf((x - xh) * 254.f);   // |dh|, |dl| <= 127
            wh |= (uint32_t)(dh & 0xff) << (8 * e);
            wl |= (uint32_t)(dl & 0xff) << (8 * e);
          }
          hi[h + 2 * half] = wh;
          lo[h + 2 * half] = wl;
        }
      }
      qi[t2][0][st][l] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      qi[t2][1][st][l] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
  } else {
    constexpr int kFragLoads = 2 * kSteps * 32 / kThreads;   // (m-tile, step, lane) fragments per thread
    float4 qv[kFragLoads][2];
#pragma unroll
    for (int u = 0; u < kFragLoads; ++u) {   // every load first
      const int idx = (int)threadIdx.x + u * kThreads;
      const int l = idx & 31, st = (idx >> 5) % kSteps, t2 = idx / (32 * kSteps), gg = l >> 2;
      const int d0 = 128 * (st >> 3) + 32 * (l & 3) + 4 * (st & 7);
      qv[u][0] = qrow(16 * t2 + gg, d0);
      qv[u][1] = qrow(16 * t2 + gg + 8, d0);
    }
#pragma unroll
    for (int u = 0; u < kFragLoads; ++u) {
      const int idx = (int)threadIdx.x + u * kThreads;
      const int l = idx & 31, st = (idx >> 5) % kSteps, t2 = idx / (32 * kSteps);
      const float4 r0 = qv[u][0], r1 = qv[u][1];
      const float v[8] = {r0.x, r0.y, r1.x, r1.y, r0.z, r0.w, r1.z, r1.w};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half h0 = __float2half_rn(v[2 * j]), h1 = __float2half_rn(v[2 * j + 1]);
        hi[j] = pack_f16x2(__half2float(h0), __half2float(h1));
        lo[j] = pack_f16x2(v[2 * j] - __half2float(h0), v[2 * j + 1] - __half2float(h1));
      }
      sm.qf[t2][0][st][l] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      sm.qf[t2][1][st][l] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
  }
  __syncthreads();
  const int mt = warp & 1, kq = warp >> 1;   // this warp's query rows 16 mt .. + 15 and chunk keys 16 kq .. + 15
  // per-row factor of a raw score: the int8 path's digit unit times the softmax scale (the FP8 path's scale alone),
  // times log2(e): the running max and the probabilities are kept in base 2, p = 2^(s - max) = e^(s ln 2 - max ln 2)
  constexpr float kLog2e = 1.4426950408889634f;
  const float rf0 = (I8 ? sm.qfac[16 * mt + g] * a.scale : a.scale) * kLog2e;
  const float rf1 = (I8 ? sm.qfac[16 * mt + g + 8] * a.scale : a.scale) * kLog2e;
  const bool active = (16 * mt) / group < m;   // its query rows hold at least one activation row
  // the activation rows of this lane's two query rows and their positions
  const int arow0 = (16 * mt + g) / group, arow1 = (16 * mt + g + 8) / group;
  const int t0 = pos0 + arow0, t1 = pos0 + arow1;
  const bool live0 = arow0 < m, live1 = arow1 < m;

  // PV role of this warp: query rows 16 mt .. + 15, head dims kDq dq .. + kDq - 1 (a quarter of the head)
  constexpr int kDq = D / 4, kDt = kDq / 8;
  const int dq = kq;
  float acc[kDt][4];
#pragma unroll
  for (int dt = 0; dt < kDt; ++dt) acc[dt][0] = acc[dt][1] = acc[dt][2] = acc[dt][3] = 0.f;
  // the running max of rows g and g + 8 (base 2; the same in the 4 warps of a row half, which see the same chunk
  // maxima) and this lane's part of their probability sums (its 4 keys of every chunk)
  float run_m0 = -INFINITY, run_m1 = -INFINITY, run_l0 = 0.f, run_l1 = 0.f;
  // the named barrier of the row half's 4 warps (1 or 2; constant ids let the CTA reserve only those)
  auto half_bar = [&]() {
    if (mt == 0)
      named_bar_sync(1, 128);
    else
      named_bar_sync(2, 128);
  };

  // One chunk (slot base c0) from its stage. Scores and probabilities: this warp's 16 keys 16 kq .. + 15; the MMA k
  // index and the keys are permuted so that lane tq owns the 4 consecutive keys 4 tq .. + 3 of a 16-key group:
  // k = 2 tq + {0, 1} are keys 4 tq + {0, 1}, k = 2 tq + 8 + {0, 1} keys 4 tq + {2, 3}. The score tile T (n8)
  // column 2 tq + c is then key 4 tq + 2 T + c, and the K row that lane g supplies to tile T is key
  // 4 ((g >> 1) & 3) + 2 T + (g & 1). The row half's 4 warps meet twice: for the chunk's row maxima, and once every
  // probability times V scale (P', fp16) is in shared memory, after which each warp multiplies all 64 keys' P' by V
  // for its quarter of the head dims.
  auto chunk = [&](const Stage<D>& stg, int64_t c0) {
    float s[2][4];   // raw scores of 2 n8 tiles: x rf (row) x the key's K scale below
    if constexpr (I8) {
      // ---- S = Q K^T on the int8 codes: 2 n8 tiles x D / 32 k32 steps x (hi, lo) digits, exact in int32 ----
      int ch[2][4], cl[2][4];
#pragma unroll
      for (int T = 0; T < 2; ++T) ch[T][0] = ch[T][1] = ch[T][2] = ch[T][3] = cl[T][0] = cl[T][1] = cl[T][2] = cl[T][3] = 0;
#pragma unroll
      for (int hs = 0; hs < D / 128; ++hs) {   // a 128-dim half: lane tq's 32 bytes of a K row, units 2 tq, 2 tq + 1
        uint4 kw[2][2];
#pragma unroll
        for (int T = 0; T < 2; ++T) {
          const int key = 16 * kq + 4 * ((g >> 1) & 3) + 2 * T + (g & 1);
          const uint8_t* row = stg.k + key * D + 128 * hs;
          kw[T][0] = *reinterpret_cast<const uint4*>(row + 16 * ((2 * tq) ^ swz_k(key)));
          kw[T][1] = *reinterpret_cast<const uint4*>(row + 16 * ((2 * tq + 1) ^ swz_k(key)));
        }
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {   // k32 step 4 hs + sub: bytes 8 sub .. + 7 of the lane's 32
          const uint4 qh = qi[mt][0][4 * hs + sub][lane], ql = qi[mt][1][4 * hs + sub][lane];
#pragma unroll
          for (int T = 0; T < 2; ++T) {
            const uint4& w = kw[T][sub >> 1];
            const uint32_t b0 = (sub & 1) ? w.z : w.x, b1 = (sub & 1) ? w.w : w.y;
            mma_s8(ch[T], qh, b0, b1);
            mma_s8(cl[T], ql, b0, b1);
          }
        }
      }
#pragma unroll
      for (int T = 0; T < 2; ++T)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[T][c] = __int2float_rn(254 * ch[T][c] + cl[T][c]);   // |.| < 2^31
    } else {
      // ---- S = Q K^T over 2 n8 tiles x kSteps k16 steps, q = hi + lo ----
      float sl[2][4];   // the hi and lo products accumulate apart (shorter dependency chains)
#pragma unroll
      for (int T = 0; T < 2; ++T) s[T][0] = s[T][1] = s[T][2] = s[T][3] = sl[T][0] = sl[T][1] = sl[T][2] = sl[T][3] = 0.f;
#pragma unroll
      for (int hs = 0; hs < D / 64; ++hs) {   // dims 128 (hs >> 1) + 32 tq + 16 (hs & 1) .. + 15: steps 4 hs .. + 3
        uint4 kw[2];
#pragma unroll
        for (int T = 0; T < 2; ++T) {
          const int key = 16 * kq + 4 * ((g >> 1) & 3) + 2 * T + (g & 1);
          kw[T] = *reinterpret_cast<const uint4*>(stg.k + key * D + 128 * (hs >> 1) +
                                                  16 * ((2 * tq + (hs & 1)) ^ swz_k(key)));
        }
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int st = 4 * hs + sub;
          const uint4 qh = sm.qf[mt][0][st][lane], ql = sm.qf[mt][1][st][lane];
#pragma unroll
          for (int T = 0; T < 2; ++T) {
            const uint32_t word = sub == 0 ? kw[T].x : sub == 1 ? kw[T].y : sub == 2 ? kw[T].z : kw[T].w;
            uint32_t b0, b1;
            codes_to_f16(word, (int)kKvFp8, b0, b1);
            mma_f16(s[T], qh.x, qh.y, qh.z, qh.w, b0, b1);
            mma_f16(sl[T], ql.x, ql.y, ql.z, ql.w, b0, b1);
          }
        }
      }
#pragma unroll
      for (int T = 0; T < 2; ++T)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[T][c] += sl[T][c];
    }
    // ---- scale, mask, online softmax: s[T][c] (row g) and s[T][2 + c] (row g + 8) are key 16 kq + 4 tq + 2 T + c ----
    const float4 kq4 = *reinterpret_cast<const float4*>(stg.ks + 16 * kq + 4 * tq);
    const float4 vq4 = *reinterpret_cast<const float4*>(stg.vs + 16 * kq + 4 * tq);
    const float ksc[4] = {kq4.x, kq4.y, kq4.z, kq4.w}, vsc[4] = {vq4.x, vq4.y, vq4.z, vq4.w};
    float mx0 = -INFINITY, mx1 = -INFINITY;
    if (!a.ring && a.window == 0 && c0 + 64 <= kend) {
      // every key of the chunk lies below kend and no window applies: visible to every row (rows past m hold zero
      // queries and are never written out)
#pragma unroll
      for (int T = 0; T < 2; ++T)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          s[T][c] *= ksc[2 * T + c] * rf0;
          s[T][2 + c] *= ksc[2 * T + c] * rf1;
          mx0 = fmaxf(mx0, s[T][c]);
          mx1 = fmaxf(mx1, s[T][2 + c]);
        }
    } else {
      int kpos[4];
      if (a.ring) {
        const int4 pq = *reinterpret_cast<const int4*>(stg.pos + 16 * kq + 4 * tq);
        kpos[0] = pq.x; kpos[1] = pq.y; kpos[2] = pq.z; kpos[3] = pq.w;
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) kpos[r] = (int)c0 + 16 * kq + 4 * tq + r;
      }
#pragma unroll
      for (int T = 0; T < 2; ++T) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int kk = 2 * T + c;
          const int p = kpos[kk];
          const bool ok = p >= 0 && p < kend;
          const bool vis0 = live0 && ok && (a.window == 0 || t0 - p < a.window);
          const bool vis1 = live1 && ok && (a.window == 0 || t1 - p < a.window);
          s[T][c] = vis0 ? s[T][c] * (ksc[kk] * rf0) : -INFINITY;
          s[T][2 + c] = vis1 ? s[T][2 + c] * (ksc[kk] * rf1) : -INFINITY;
          mx0 = fmaxf(mx0, s[T][c]);
          mx1 = fmaxf(mx1, s[T][2 + c]);
        }
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    if (tq == 0) {
      sm.cmax[kq][16 * mt + g] = mx0;
      sm.cmax[kq][16 * mt + g + 8] = mx1;
    }
    half_bar();
#pragma unroll
    for (int q = 0; q < kQuarters; ++q) {   // the chunk's row maxima over the 4 key quarters
      mx0 = fmaxf(mx0, sm.cmax[q][16 * mt + g]);
      mx1 = fmaxf(mx1, sm.cmax[q][16 * mt + g + 8]);
    }
    // scores are in base-2 units: p = 2^(s - max); a row with nothing visible yet keeps max -inf, corr 1 and p 0
    const float new_m0 = fmaxf(run_m0, mx0), new_m1 = fmaxf(run_m1, mx1);
    const float base0 = new_m0 == -INFINITY ? 0.f : new_m0, base1 = new_m1 == -INFINITY ? 0.f : new_m1;
    const float corr0 = new_m0 == -INFINITY ? 1.f : ex2_approx(run_m0 - new_m0);
    const float corr1 = new_m1 == -INFINITY ? 1.f : ex2_approx(run_m1 - new_m1);
    run_m0 = new_m0;
    run_m1 = new_m1;
    run_l0 *= corr0;
    run_l1 *= corr1;
    // P' (probability times V scale) of this lane's keys 16 kq + 4 tq .. + 3 for rows g, g + 8: 8 bytes each, unit
    // 4 kq + tq of the row stored at unit (4 kq + tq) ^ 4 (g & 3) (conflict-free stores and loads)
    uint32_t pa[4];
#pragma unroll
    for (int T = 0; T < 2; ++T) {
      float p[4];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int kk = 2 * T + c;
        p[c] = ex2_approx(s[T][c] - base0);   // 2^-inf = 0 for a masked key
        p[2 + c] = ex2_approx(s[T][2 + c] - base1);
        run_l0 += p[c];
        run_l1 += p[2 + c];
        p[c] *= vsc[kk];
        p[2 + c] *= vsc[kk];
      }
      pa[2 * T] = pack_f16x2(p[0], p[1]);
      pa[2 * T + 1] = pack_f16x2(p[2], p[3]);
    }
    const int pu = (4 * kq + tq) ^ (4 * (g & 3));
    sm.pbuf[mt][g][pu] = make_uint2(pa[0], pa[2]);
    sm.pbuf[mt][g + 8][pu] = make_uint2(pa[1], pa[3]);
    if (corr0 != 1.f || corr1 != 1.f) {
#pragma unroll
      for (int dt = 0; dt < kDt; ++dt) {
        acc[dt][0] *= corr0;
        acc[dt][1] *= corr0;
        acc[dt][2] *= corr1;
        acc[dt][3] *= corr1;
      }
    }
    half_bar();
    // ---- O += P' V over the chunk's 64 keys (4 k16 steps) for head dims d = kDq dq + 8 dt + g: lane tq supplies
    // keys 16 ks + 4 tq .. + 3 (one 32-bit word of V, 8 bytes of P' per row) ----
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int u = (4 * ks + tq) ^ (4 * (g & 3));
      const uint2 pg = sm.pbuf[mt][g][u], pg8 = sm.pbuf[mt][g + 8][u];
#pragma unroll
      for (int dt = 0; dt < kDt; ++dt) {
        const int d = kDq * dq + 8 * dt + g;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(stg.v + d * 64 + 16 * (ks ^ ((d >> 1) & 3)) + 4 * tq);
        uint32_t b0, b1;
        codes_to_f16(w, I8 ? (int)kKvInt8 : (int)kKvFp8, b0, b1);
        mma_f16(acc[dt], pg.x, pg8.x, pg.y, pg8.y, b0, b1);
      }
    }
  };

  // every warp takes its part of every chunk; the last warp done with a stage refills it (nobody waits for it)
  for (int i = 0; i < nc; ++i) {
    const int s = i % kStages;
    mbar_wait_bounded(&sm.full[s], (uint32_t)(i / kStages) & 1u, lane == 0 ? a.err : nullptr);
    if (active) chunk(sm.stage[s], (cb + i) * 64);
    if (i + kStages < nc) {
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();   // this warp's reads of the stage are ordered before its release
        last = atomicAdd(&sm.released[s], 1) == kThreads / 32 - 1;
        if (last) {
          sm.released[s] = 0;
          __threadfence_block();
          fence_proxy_async_smem();   // the other warps' reads before the bulk copies that overwrite the stage
        }
      }
      if (__shfl_sync(0xffffffffu, last, 0)) issue(i + kStages);
    }
  }
  // ---- the CTA's partial: the row sums over the quad and the 4 key-quarter warps; each warp stores its dims ----
  run_l0 += __shfl_xor_sync(0xffffffffu, run_l0, 1);
  run_l0 += __shfl_xor_sync(0xffffffffu, run_l0, 2);
  run_l1 += __shfl_xor_sync(0xffffffffu, run_l1, 1);
  run_l1 += __shfl_xor_sync(0xffffffffu, run_l1, 2);
  if (active && tq == 0) {
    sm.lsum[kq][16 * mt + g] = run_l0;
    sm.lsum[kq][16 * mt + g + 8] = run_l1;
  }
  __syncthreads();
  if (active) {
    const int pidx = a.part_local ? split : sidx;
#pragma unroll
    for (int h = 0; h < 2; ++h) {   // rows g and g + 8 of the row half
      const int r = 16 * mt + g + 8 * h;
      if (r / group >= m) continue;
      float L = 0.f;
#pragma unroll
      for (int q = 0; q < kQuarters; ++q) L += sm.lsum[q][r];
      float* out = a.part + (int64_t)seq * a.part_seq_stride + (((int64_t)pidx * a.kv_heads + kvh) * kQRows + r) * kPartStride;
      if (dq == 0 && tq == 0) {
        out[0] = (h ? run_m1 : run_m0) * 0.6931471805599453f;   // natural-log units for the combine
        out[1] = L;
      }
#pragma unroll
      for (int dt = 0; dt < kDt; ++dt)
        *reinterpret_cast<float2*>(out + 4 + kDq * dq + 8 * dt + 2 * tq) =
            h ? make_float2(acc[dt][2], acc[dt][3]) : make_float2(acc[dt][0], acc[dt][1]);
    }
  }
}

// Combine the splits of (activation row, q head) by log-sum-exp; then either the plain output (API) or the Dory
// output gate, fp16 fragments for the O projection and the per-head sum of squares (the step). One CTA per (row,
// head), one thread per head dimension; the split weights are computed once, every partial is loaded in one wave.
template <int D>
__global__ void __launch_bounds__(D) attn_combine_kernel(const CombineArgs a) {
  constexpr int kRegSplits = 64;   // partials held in registers (the rest are read in a second pass)
  constexpr int kPartStride = part_stride(D);
  __shared__ float wgt[kMaxSplits];
  __shared__ float cached[2];      // the splits' max m and their sum of l relative to it
  __shared__ float part_s[D / 32][kMaxRows];
  __shared__ float ml[2][kMaxSplits];   // every split's m and l
  const int i = blockIdx.x, h = blockIdx.y, seq = blockIdx.z, d = threadIdx.x;
  const int col = h * D + d;
  // the gate's scale is a parameter: loaded before the dependency wait
  const float gsc = a.out ? 0.f : a.gscale[col];
  const int m = a.params ? a.params[seq].m : a.m;
  const int own0 = a.params ? a.params[seq].own_rows : 0;   // the sequence's earlier rows of this step
  const int64_t rows0 = (int64_t)seq * kMaxRows;   // this sequence's first activation row
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  if (i >= m) return;
  const int group = a.heads / a.kv_heads, kvh = h / group, qr = i * group + h % group;
  const float* base = a.part + (int64_t)seq * a.part_seq_stride + ((int64_t)kvh * kQRows + qr) * kPartStride;
  const int64_t sstride = (int64_t)a.kv_heads * kQRows * kPartStride;   // split s at s * sstride
  const float qd = a.q[((rows0 + i) * a.heads + h) * D + d];
  float kj[kMaxRows], vj[kMaxRows];
#pragma unroll
  for (int j = 0; j < kMaxRows; ++j) {
    kj[j] = j < m ? a.k[((rows0 + j) * a.kv_heads + kvh) * D + d] : 0.f;
    vj[j] = j < m ? a.v[((rows0 + j) * a.kv_heads + kvh) * D + d] : 0.f;
  }
  const float gt = a.out ? 0.f : a.gate[(rows0 + i) * a.gate_ld + col];
  // every independent load in one wave: this thread's dim of every split's partial, the m and l of splits d,
  // d + D, ...
  const int ns = a.splits < kRegSplits ? a.splits : kRegSplits;
  float acc_s[kRegSplits];
#pragma unroll
  for (int s = 0; s < kRegSplits; ++s) acc_s[s] = s < ns ? base[s * sstride + 4 + d] : 0.f;
  constexpr int kMlLoads = kMaxSplits / D;
  float mls[kMlLoads][2];
#pragma unroll
  for (int u = 0; u < kMlLoads; ++u) {
    const int sp = d + u * D;
    mls[u][0] = sp < a.splits ? base[sp * sstride] : -INFINITY;
    mls[u][1] = sp < a.splits ? base[sp * sstride + 1] : 0.f;
  }
#pragma unroll
  for (int u = 0; u < kMlLoads; ++u) {
    const int sp = d + u * D;
    if (sp < a.splits) {
      ml[0][sp] = mls[u][0];
      ml[1][sp] = mls[u][1];
    }
  }
  __syncthreads();
  // split weights exp(m_s - M) and sum_s l_s exp(m_s - M), by the first warp in a fixed order
  if (threadIdx.x < 32) {
    float mx = -INFINITY;
    for (int s = threadIdx.x; s < a.splits; s += 32) mx = fmaxf(mx, ml[0][s]);
    mx = warp_max(mx);
    float l = 0.f;
    for (int s = threadIdx.x; s < a.splits; s += 32) {
      const float ms = ml[0][s];
      const float w = ms == -INFINITY ? 0.f : expf(ms - mx);
      wgt[s] = w;
      l += w == 0.f ? 0.f : ml[1][s] * w;
    }
    l = warp_sum(l);
    if (threadIdx.x == 0) {
      cached[0] = mx;
      cached[1] = l;
    }
  }
  // this call's own keys j <= i, scored in FP32 from the prepared rows (the reference attends to them unquantized)
  {
    float prod[kMaxRows];
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) prod[j] = warp_sum(qd * kj[j]);
    if ((d & 31) == 0)
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) part_s[d >> 5][j] = prod[j];
  }
  __syncthreads();
  float own_s[kMaxRows], own_m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxRows; ++j) {
    const bool vis = j < m && j <= i && (a.window == 0 || i - j < a.window);
    float pr = (part_s[0][j] + part_s[1][j]) + (part_s[2][j] + part_s[3][j]);
    if constexpr (D == 256) pr += (part_s[4][j] + part_s[5][j]) + (part_s[6][j] + part_s[7][j]);
    own_s[j] = vis ? pr * a.scale : -INFINITY;
    own_m = fmaxf(own_m, own_s[j]);
  }
  float wgt_max = cached[0], lcached = cached[1];
  float o = 0.f;
#pragma unroll
  for (int s = 0; s < kRegSplits; ++s)
    if (s < ns) o += acc_s[s] * wgt[s];
  for (int s = kRegSplits; s < a.splits; ++s)
    if (wgt[s] != 0.f) o += base[s * sstride + 4 + d] * wgt[s];
  if (D == 128 && a.x.world > 1) {   // head dim 128 only: the exchange slots hold 128 dims
    // split-KV across GPUs: this process's cached part (m, l, o relative to m) to every peer, theirs from this
    // process's slots, all merged in rank order (the same bits on every process)
    const uint32_t run = *a.x.epoch * (uint32_t)a.x.n_g + (uint32_t)a.x.g, seq = run + 1;
    const int64_t set = (int64_t)(run & 1) * a.x.world;
    auto slot_of = [&](uint64_t* sl, int src) { return sl + (((set + src) * kMaxRows + i) * a.heads + h) * kXchgStride; };
    uint64_t* mine = a.x.slot[0];
#pragma unroll
    for (int t = 0; t < kMaxKvWorld; ++t) {
      if (t < a.x.world && t == a.x.rank) mine = a.x.slot[t];
      if (t < a.x.world && t != a.x.rank) {
        uint64_t* w = slot_of(a.x.slot[t], a.x.rank);
        put_seq_word(w + 2 + d, o, seq);
        if (d == 0) {
          put_seq_word(w, wgt_max, seq);
          put_seq_word(w + 1, lcached, seq);
        }
      }
    }
    float mt[kMaxKvWorld], lt[kMaxKvWorld], ot[kMaxKvWorld];
    float mx = -INFINITY;
#pragma unroll
    for (int t = 0; t < kMaxKvWorld; ++t) {
      mt[t] = -INFINITY;
      lt[t] = ot[t] = 0.f;
      if (t < a.x.world) {
        if (t == a.x.rank) {
          mt[t] = wgt_max;
          lt[t] = lcached;
          ot[t] = o;
        } else {
          const uint64_t* w = slot_of(mine, t);
          mt[t] = take_seq_word(w, seq, a.x.wait_ns, a.err);
          lt[t] = take_seq_word(w + 1, seq, a.x.wait_ns, a.err);
          ot[t] = take_seq_word(w + 2 + d, seq, a.x.wait_ns, a.err);
        }
      }
      mx = fmaxf(mx, mt[t]);
    }
    float l = 0.f, oo = 0.f;
#pragma unroll
    for (int t = 0; t < kMaxKvWorld; ++t) {
      const float wt = mt[t] == -INFINITY ? 0.f : expf(mt[t] - mx);
      l += wt == 0.f ? 0.f : lt[t] * wt;
      oo += wt == 0.f ? 0.f : ot[t] * wt;
    }
    wgt_max = mx;
    lcached = l;
    o = oo;
  }
  // a prompt chunk's earlier groups (every row before this one, within the window), scored in FP32 like the own
  // keys: blocks of 8 keys folded into the cached part (max wgt_max, sum lcached, output o) before this group's keys
  for (int jb = 0; jb < own0; jb += kMaxRows) {
    float kb[kMaxRows], vb[kMaxRows], prod[kMaxRows];
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      const int64_t r = rows0 - own0 + jb + j;
      kb[j] = a.k[(r * a.kv_heads + kvh) * D + d];
      vb[j] = a.v[(r * a.kv_heads + kvh) * D + d];
    }
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) prod[j] = qd * kb[j];
    warp_sum8(prod);
    __syncthreads();   // every thread has read part_s's previous sums
    if ((d & 31) == 0)
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) part_s[d >> 5][j] = prod[j];
    __syncthreads();
    float sj[kMaxRows], bm = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      float pr = (part_s[0][j] + part_s[1][j]) + (part_s[2][j] + part_s[3][j]);
      if constexpr (D == 256) pr += (part_s[4][j] + part_s[5][j]) + (part_s[6][j] + part_s[7][j]);
      const bool vis = a.window == 0 || own0 + i - (jb + j) < a.window;
      sj[j] = vis ? pr * a.scale : -INFINITY;
      bm = fmaxf(bm, sj[j]);
    }
    const float nm = fmaxf(wgt_max, bm);
    const float cw = wgt_max == -INFINITY ? 0.f : expf(wgt_max - nm);
    lcached *= cw;
    o *= cw;
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      const float pj = sj[j] == -INFINITY ? 0.f : expf(sj[j] - nm);
      lcached += pj;
      o += pj * vb[j];
    }
    wgt_max = nm;
  }
  const float mall = fmaxf(own_m, wgt_max);
  const float cs = wgt_max == -INFINITY ? 0.f : expf(wgt_max - mall);   // the cached part's weight
  // merge the cached part (relative to wgt_max) and the own keys (relative to mall)
  float lsum = lcached * cs;
  o *= cs;
#pragma unroll
  for (int j = 0; j < kMaxRows; ++j) {
    const float pj = own_s[j] == -INFINITY ? 0.f : expf(own_s[j] - mall);
    lsum += pj;
    o += pj * vj[j];
  }
  o *= lsum > 0.f ? 1.f / lsum : 0.f;
  if (a.out) {
    a.out[((int64_t)i * a.heads + h) * D + d] = o;
    return;
  }
  o *= 1.f / (1.f + expf(-gt * gsc));
  __shared__ float red[32];
  const float ss = block_sum(o * o, red);
  if (a.gated_out) {   // the batched step: f32 rows for the GEMM's digitizer
    a.gated_out[(rows0 + i) * a.heads * D + col] = o;
    if (d == 0) a.asum[h * a.asum_ld + rows0 + i] = ss;
    return;
  }
  if (d == 0) a.asum[(int64_t)i * a.heads + h] = ss;   // [row][head]: the O projection's parts of row i together
  // the O projection's input: this head's D / 16 groups of 16 as B digits (a quad per group)
  __shared__ float ov[D];
  ov[d] = o;
  __syncthreads();
  if (d < D / 4) {
    const int gl = d >> 2, t = d & 3, G = h * (D / 16) + gl;
    const float v[4] = {ov[16 * gl + 4 * t], ov[16 * gl + 4 * t + 1], ov[16 * gl + 4 * t + 2], ov[16 * gl + 4 * t + 3]};
    uint32_t code[kDigits], sf[kDigits];
    const float p = digitize16_quad(v, code, sf);
    store_digits_quad(a.ab + (int64_t)(G >> 2) * kBBlockBytes, i, G & 3, t, code, sf);
    if (t == 0) a.ab_pre[(int64_t)G * 8 + i] = p;
  }
}

// The batched step's combine (up to kWarpSplits splits): one warp per (sequence, activation row, q head), lane l
// holding head dims 4 l .. 4 l + 3 and split l's m and l. The merge, the own keys' dot products and the norm need only
// shuffles, no block barrier; every load goes out in one wave after the dependency wait. (For the 8-row step the
// CTA per pair above measured faster: 2.538 against 2.614-2.647 ms per config-3 step, its loads spread over 4
// warps.)
constexpr int kWarpSplits = 24;
constexpr int kCombineWarps = 8;

__device__ __forceinline__ float4 ld4g(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float dot4(float4 a, float4 b) { return (a.x * b.x + a.y * b.y) + (a.z * b.z + a.w * b.w); }

template <bool kPrompt>
__global__ void __launch_bounds__(kCombineWarps * 32) attn_combine_warp_kernel(const CombineArgs a) {
  constexpr int kD = 128, kPartStride = part_stride(kD);   // head dim 128
  const int lane = threadIdx.x & 31;
  const int pair = (int)blockIdx.x * (int)(blockDim.x >> 5) + (int)(threadIdx.x >> 5);
  const int per_seq = kMaxRows * a.heads;
  const int seq = pair / per_seq, i = (pair % per_seq) / a.heads, h = pair % a.heads;
  const bool exists = seq < a.nseq;
  const int d0 = 4 * lane, col = h * kD + d0;
  // the gate's scale is a parameter: loaded before the dependency wait
  const float4 gsc = exists ? ld4g(a.gscale + col) : make_float4(0.f, 0.f, 0.f, 0.f);
  const int m = exists ? (a.params ? a.params[seq].m : a.m) : 0;
  // the sequence's earlier rows of this step (a prompt chunk only: the verify path keeps its registers)
  const int own0 = kPrompt && exists && a.params ? a.params[seq].own_rows : 0;
  const int64_t rows0 = (int64_t)seq * kMaxRows;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  if (i >= m) return;   // the whole warp
  const int group = a.heads / a.kv_heads, kvh = h / group, qr = i * group + h % group;
  const float* base = a.part + (int64_t)seq * a.part_seq_stride + ((int64_t)kvh * kQRows + qr) * kPartStride;
  const int64_t sstride = (int64_t)a.kv_heads * kQRows * kPartStride;
  const float ms = lane < a.splits ? base[lane * sstride] : -INFINITY;
  const float ls = lane < a.splits ? base[lane * sstride + 1] : 0.f;
  // verify rows: every load in one wave up front; a prompt chunk (which also folds the earlier groups' keys) loads
  // the split partials and its own rows where it uses them, to keep its registers down
  float4 acc[kWarpSplits];
  if constexpr (!kPrompt) {
#pragma unroll
    for (int s = 0; s < kWarpSplits; ++s)
      acc[s] = s < a.splits ? ld4g(base + s * sstride + 4 + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float4 q4 = ld4g(a.q + ((rows0 + i) * a.heads + h) * kD + d0);
  float4 kj[kMaxRows], vj[kMaxRows];
  auto load_own = [&]() {
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      kj[j] = j < m ? ld4g(a.k + ((rows0 + j) * a.kv_heads + kvh) * kD + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
      vj[j] = j < m ? ld4g(a.v + ((rows0 + j) * a.kv_heads + kvh) * kD + d0) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if constexpr (!kPrompt) load_own();
  const float4 gt = ld4g(a.gate + (rows0 + i) * a.gate_ld + col);
  // split weights exp(m_s - M) and sum_s l_s exp(m_s - M); the dims' sum in split order
  const float M = warp_max(ms);
  const float w = ms == -INFINITY ? 0.f : expf(ms - M);
  const float lcached = warp_sum(w == 0.f ? 0.f : ls * w);
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int s = 0; s < kWarpSplits; ++s) {
    const float ws = __shfl_sync(0xffffffffu, w, s);
    if (s < a.splits) {
      const float4 as = kPrompt ? ld4g(base + s * sstride + 4 + d0) : acc[s];
      o.x += as.x * ws;
      o.y += as.y * ws;
      o.z += as.z * ws;
      o.w += as.w * ws;
    }
  }
  float mall = M, lsum = lcached;
  if constexpr (kPrompt) {
    // this call's own keys, scored in FP32 from the prepared rows (the reference attends to them unquantized): a
    // prompt chunk's earlier groups (every row before this one, within the window), then this group's rows j <= i;
    // each block of 8 keys is folded into the running (max, sum, output), starting from the cached part's
    auto fold = [&](const float4 (&kb)[kMaxRows], const float4 (&vb)[kMaxRows], int jb, int nvis) {
      // keys jb .. jb + 7 of the sequence's step rows; the first nvis are candidates; this row is own0 + i
      float sj[kMaxRows], bm = -INFINITY;
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) sj[j] = dot4(q4, kb[j]);
      warp_sum8(sj);
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) {
        const bool vis = j < nvis && jb + j <= own0 + i && (a.window == 0 || own0 + i - (jb + j) < a.window);
        sj[j] = vis ? sj[j] * a.scale : -INFINITY;
        bm = fmaxf(bm, sj[j]);
      }
      const float nm = fmaxf(mall, bm);
      const float cs = mall == -INFINITY ? 0.f : expf(mall - nm);   // the part folded so far
      lsum *= cs;
      o.x *= cs;
      o.y *= cs;
      o.z *= cs;
      o.w *= cs;
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) {
        const float pj = sj[j] == -INFINITY ? 0.f : expf(sj[j] - nm);
        lsum += pj;
        o.x += pj * vb[j].x;
        o.y += pj * vb[j].y;
        o.z += pj * vb[j].z;
        o.w += pj * vb[j].w;
      }
      mall = nm;
    };
    for (int jb = 0; jb < own0; jb += kMaxRows) {   // the earlier groups: whole blocks of 8 rows
      float4 kb[kMaxRows], vb[kMaxRows];
#pragma unroll
      for (int j = 0; j < kMaxRows; ++j) {
        const int64_t r = rows0 - own0 + jb + j;
        kb[j] = ld4g(a.k + (r * a.kv_heads + kvh) * kD + d0);
        vb[j] = ld4g(a.v + (r * a.kv_heads + kvh) * kD + d0);
      }
      fold(kb, vb, jb, kMaxRows);
    }
    load_own();
    fold(kj, vj, own0, m);
  } else {
    // this call's own keys j <= i, scored in FP32 from the prepared rows (the reference attends to them unquantized)
    float own_s[kMaxRows], own_m = -INFINITY;
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      const float pr = warp_sum(dot4(q4, kj[j]));
      const bool vis = j < m && j <= i && (a.window == 0 || i - j < a.window);
      own_s[j] = vis ? pr * a.scale : -INFINITY;
      own_m = fmaxf(own_m, own_s[j]);
    }
    mall = fmaxf(own_m, M);
    const float cs = M == -INFINITY ? 0.f : expf(M - mall);   // the cached part's weight
    lsum = lcached * cs;
    o.x *= cs;
    o.y *= cs;
    o.z *= cs;
    o.w *= cs;
#pragma unroll
    for (int j = 0; j < kMaxRows; ++j) {
      const float pj = own_s[j] == -INFINITY ? 0.f : expf(own_s[j] - mall);
      lsum += pj;
      o.x += pj * vj[j].x;
      o.y += pj * vj[j].y;
      o.z += pj * vj[j].z;
      o.w += pj * vj[j].w;
    }
  }
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  float v[4] = {o.x * inv, o.y * inv, o.z * inv, o.w * inv};
  const float gtv[4] = {gt.x, gt.y, gt.z, gt.w}, gsv[4] = {gsc.x, gsc.y, gsc.z, gsc.w};
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] *= 1.f / (1.f + expf(-gtv[c] * gsv[c]));
  const float ss = warp_sum((v[0] * v[0] + v[1] * v[1]) + (v[2] * v[2] + v[3] * v[3]));
  // f32 rows for the GEMM's digitizer and the per-head sums of squares
  *reinterpret_cast<float4*>(a.gated_out + (rows0 + i) * a.heads * kD + col) = make_float4(v[0], v[1], v[2], v[3]);
  if (lane == 0) a.asum[h * a.asum_ld + rows0 + i] = ss;
}

}  // namespace

int attention_ctas_per_sm(int head_dim) { return head_dim == 256 ? 1 : 2; }

int64_t attention_part_floats(int kv_heads, int splits, int head_dim) {
  return (int64_t)kv_heads * splits * kQRows * part_stride(head_dim);
}

void launch_attention(const AttnArgs& a_in, cudaStream_t s, bool pdl) {
  AttnArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  XTG_REQUIRE(a.kv_heads >= 1 && a.heads >= 1, "attention: at least one q head and one KV head");
  XTG_REQUIRE(a.heads % a.kv_heads == 0 && a.heads / a.kv_heads <= 4, "attention: at most 4 q heads per KV head");
  XTG_REQUIRE(a.slots % 64 == 0, "attention: cache slots must be a multiple of 64");
  XTG_REQUIRE(a.splits >= 1 && a.splits <= kMaxSplits, "attention: 1..256 splits");
  XTG_REQUIRE(a.splits_total == 0 || (a.split0 >= 0 && a.split0 + a.splits <= a.splits_total &&
                                       a.splits_total <= kMaxSplits),
              "attention: split range outside 0..splits_total (at most 256)");
  if (a.head_dim == 0) a.head_dim = 128;
  XTG_REQUIRE(a.head_dim == 128 || a.head_dim == 256, "attention: head_dim 128 or 256");
  XTG_REQUIRE(a.dtype == kKvInt8 || a.dtype == kKvFp8, "attention: KV dtype int8 (0) or fp8 (1)");
  const bool d256 = a.head_dim == 256, i8 = a.dtype == kKvInt8;
  // one kernel per (head dim, KV dtype): the int8 cache's QK^T runs on integer MMAs
  void (*const fn)(const AttnArgs) = d256 ? (i8 ? attention_kernel<256, true> : attention_kernel<256, false>)
                                          : (i8 ? attention_kernel<128, true> : attention_kernel<128, false>);
  const int smem = d256 ? (int)sizeof(Smem<256>) : (int)sizeof(Smem<128>);
  static std::atomic<uint64_t> optin[4];
  ensure_smem_optin((const void*)fn, smem, optin[(d256 ? 2 : 0) + (i8 ? 1 : 0)]);
  cudaLaunchConfig_t cfg = {};
  XTG_REQUIRE(!a.seqs || (a.nseq >= 1 && a.nseq <= kMaxBatch && a.params), "attention: 1..8 sequences with params");
  cfg.gridDim = dim3(a.splits, a.kv_heads, a.seqs ? a.nseq : 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, fn, a));
}

void launch_attn_combine(const CombineArgs& a_in, cudaStream_t s, bool pdl) {
  CombineArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  if (a.head_dim == 0) a.head_dim = 128;
  XTG_REQUIRE(a.head_dim == 128 || a.head_dim == 256, "combine: head_dim 128 or 256");
  XTG_REQUIRE(a.head_dim == 128 || a.x.world <= 1, "combine: head_dim 256 in one process (no split-KV exchange)");
  XTG_REQUIRE(a.splits >= 1 && a.splits <= kMaxSplits, "combine: 1..256 splits");
  XTG_REQUIRE(a.kv_heads >= 1 && a.heads >= 1 && a.heads % a.kv_heads == 0, "combine: q heads a multiple of KV heads");
  XTG_REQUIRE(a.x.world <= 1 || (a.x.world <= kMaxKvWorld && a.x.rank >= 0 && a.x.rank < a.x.world && a.x.epoch &&
                                 a.err && a.out == nullptr),
              "combine: split-KV exchange needs 2..8 processes, the epoch and an error word (the step only)");
  for (int t = 0; t < a.x.world && a.x.world > 1; ++t)
    XTG_REQUIRE(a.x.slot[t], "combine: split-KV exchange without the slots of every process");
  XTG_REQUIRE(!a.gated_out || (a.nseq >= 1 && a.nseq <= kMaxBatch && a.params && a.asum && a.gate && a.gscale),
              "combine: the batched step needs 1..8 sequences, params, the gate and the sums");
  cudaLaunchConfig_t cfg = {};
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (a.gated_out && a.splits <= kWarpSplits && a.x.world <= 1 && a.head_dim == 128) {   // batched: a warp per pair
    // as many warps per CTA as keep one CTA per SM or more
    const int pairs = a.nseq * kMaxRows * a.heads;
    int dev = 0, sms = 0;
    XTG_CUDA(cudaGetDevice(&dev));
    XTG_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int wpc = std::max(1, std::min(kCombineWarps, pairs / std::max(1, sms)));
    cfg.gridDim = dim3((unsigned)((pairs + wpc - 1) / wpc));
    cfg.blockDim = dim3(wpc * 32);
    if (a.prompt)
      XTG_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_warp_kernel<true>, a));
    else
      XTG_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_warp_kernel<false>, a));
    return;
  }
  cfg.gridDim = dim3(kMaxRows, a.heads, a.gated_out ? a.nseq : 1);
  cfg.blockDim = dim3(a.head_dim);
  if (a.head_dim == 256)
    XTG_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_kernel<256>, a));
  else
    XTG_CUDA(cudaLaunchKernelEx(&cfg, attn_combine_kernel<128>, a));
}

}  // namespace xtg
