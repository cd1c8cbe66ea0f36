// K1: NVFP4 weight x activation GEMV for the 1..8-row decode / verify step (matmul_nvfp4's hot loop,
// engine/src/kernels.cpp:84-138, m <= 8) on the block-scaled FP4 tensor cores of sm_100a.
//
// Why tensor cores, and why this form: at 8 rows the weights are read once and used 8 times, far below any
// tensor-core ridge, so the kernel must stream NVFP4 at HBM speed. Converting the E2M1 codes and E4M3 scales on the
// CUDA cores costs ~95 instructions per 576 weight bytes, which alone fills the SM's issue slots at HBM rate.
// tcgen05.mma kind::mxf4nvf4 takes the codes and the per-16 E4M3 scales as they are stored, so the weights go from
// HBM to shared memory (bulk copies) to the tensor core untouched. The activations become the FP4 B operand as
// 4 scaled E2M1 digits per value (fp4mma.cuh): N = 32 digit rows, the epilogue adds each row's 4 digit columns.
// One MMA is 128 weight rows x 64 inputs; its accumulator lives in TMEM.
//
// Work split: tiles of 128 rows. A GEMV with fewer tiles than CTA slots splits each tile's K blocks over a cluster
// of `split` CTAs, whose partial sums meet in distributed shared memory (summed in cluster-rank order, no atomics);
// otherwise each CTA takes whole tiles. In every CTA one thread streams weight units through a ring of shared-memory
// stages (cp.async.bulk, completion on mbarriers; the first stages are issued before griddepcontrol.wait, since the
// weights do not depend on the previous kernel), one thread issues the MMAs, and four warps drain the TMEM
// accumulator (double-buffered across tiles) into the epilogue: a plain store (with an optional justnorm row scale),
// SwiGLU, or the lm_head with its per-tile argmax candidates. Every sum has a fixed order: results are the same on
// every launch.
#include <algorithm>

#include "attention.h"
#include "common.cuh"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kThreads = 256;
constexpr int kStageUnits = 4;
constexpr int kMaxRing = 6;
// shared memory of an SM, the part the system keeps per CTA, the most one CTA may have
constexpr int64_t kSmPerSm = 233472, kPerCtaReserve = 1024, kMaxSmem = 232448;
constexpr int kAccCols = 64;   // TMEM columns per accumulator (32 used)
static_assert(kBBlockBytes == kDigitBlockBytes, "the host's digit buffer size");
constexpr int kSumsqLoads = 10;   // the producer's row-sum parts a lane loads: at most 320 parts

struct Params {
  GemvArgs a;
  int split, tpc, ring, slice_max, rpr;
  uint32_t tmem_cols;
  uint32_t off_b, off_pre, off_red, off_vsq, off_cand, off_bar, off_misc;
};

struct SmemPlan {
  uint32_t off_b, off_pre, off_red, off_vsq, off_cand, off_bar, off_misc, total;
  int rpr;   // partial-row slots per source CTA in the cluster reduction
};

SmemPlan smem_plan(int ring, int slice, int split) {
  SmemPlan s;
  // STORE: ceil(128 / split) rows per rank; SwiGLU: 2 x 16 x ceil(4 / split) (gate and up of its feature groups)
  s.rpr = std::max((kTileRows + split - 1) / split, 32 * ((4 + split - 1) / split));
  uint32_t o = (uint32_t)(ring * kStageUnits * kUnitBytes);
  s.off_b = o;
  o += (uint32_t)slice * kBBlockBytes;
  s.off_pre = o;
  o += (uint32_t)slice * 4 * 8 * 4;
  s.off_red = o;
  o += (uint32_t)(split * s.rpr * 8 * 4);
  s.off_vsq = o;
  o += 8 * 64 * 4;
  s.off_cand = o;
  o += 4 * 8 * 8;
  s.off_bar = o;
  o += (2 * kMaxRing + 8) * 8;
  s.off_misc = o;
  o += 128;
  s.total = o;
  return s;
}

// TMEM: the accumulator (two when a CTA takes several tiles), the slice's activation scales, the ring's weight scales
int tmem_columns(int tiles_per_cta, int slice, int ring) {
  return (tiles_per_cta > 1 ? 2 : 1) * kAccCols + 4 * slice + 4 * ring * kStageUnits;
}

__device__ __forceinline__ void wait_bar(uint64_t* bar, uint32_t parity, int* err) {
  mbar_wait_bounded(bar, parity, err);
}

// first row (STORE) or 16-feature group (SwiGLU) a cluster rank finishes: ceil(n * rank / split)
__device__ __forceinline__ int share_begin(int n, int rank, int split) { return (n * rank + split - 1) / split; }

// Block-wide (two halves of 128 threads) sum / max of v over the threads of each half; scratch: 8 floats.
__device__ __forceinline__ float half_reduce(float v, bool is_max, float* scratch, int tid) {
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if ((tid & 31) == 0) scratch[tid >> 5] = v;
  __syncthreads();
  const float* w = scratch + 4 * (tid >> 7);
  return is_max ? fmaxf(fmaxf(w[0], w[1]), fmaxf(w[2], w[3])) : ((w[0] + w[1]) + (w[2] + w[3]));
}

// What the q|k|v finish of one thread reads from memory other than the cluster's partials, loaded long before the
// partials meet: the position, the q scale of its head dim, the gate tile's output, and the RoPE factors of its rows
// (at most 4: rows i0 + hf, i0 + hf + 2, ...).
struct QkvPre {
  int64_t pos0;
  float qscale;
  TileOut out;
  float cs[4], sn[4];
};

// kEpiQkv, after the cluster's partials met: this rank's activation rows of tile t (one head), two rows at a time
// (threads 0-127 and 128-255, thread = head dim)
__device__ __forceinline__ void qkv_finish(const GemvArgs& a, const QkvPre& pre, const float* red, float* scratch,
                                           int t, int srank, int S, int m, int tid) {
  const int i0 = share_begin(8, srank, S), i1 = share_begin(8, srank + 1, S), nil = (8 + S - 1) / S;
  const int type = t < a.q_tiles ? 0 : t < a.q_tiles + a.kv_tiles ? 1 : t < a.q_tiles + 2 * a.kv_tiles ? 2 : 3;
  const int d = tid & 127, hf = tid >> 7;
  float* xs = scratch + 8;   // [2][128]
  const int64_t pos0 = pre.pos0;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int ib = i0 + 2 * it;
    if (ib >= i1) break;
    const int i = ib + hf;
    const bool row = i < i1, live = row && i < m;
    float x = 0.f;
    if (row)
      for (int c = 0; c < S; ++c) x += red[(c * nil + (i - i0)) * kTileRows + d];
    if (type == 3) {   // the gate: stored as kEpiStore does
      const TileOut& o = pre.out;
      if (live && d < o.rows) o.y[(int64_t)i * o.ld + d] = x;
      continue;
    }
    float r = x;
    if (type <= 1) {   // NeoX RoPE on (d, d + 64), then justnorm over the head
      xs[hf * 128 + d] = x;
      __syncthreads();
      const float c = pre.cs[it], sn = pre.sn[it];
      const float other = xs[hf * 128 + (d ^ 64)];
      r = d < 64 ? x * c - other * sn : x * c + other * sn;
      const float f = 1.f / sqrtf(half_reduce(r * r, false, scratch, tid) + 1e-6f);
      r *= f;
    }
    if (type == 0) {
      if (live) a.q_out[((int64_t)i * a.q_tiles + t) * 128 + d] = r * pre.qscale;
      continue;
    }
    // k / v: the prepared row, and its codes and scale in the cache (the KvCache::store rule)
    const int h = t - a.q_tiles - (type == 2 ? a.kv_tiles : 0);
    const float amax = half_reduce(fabsf(r), true, scratch, tid);
    if (!live) continue;
    (type == 1 ? a.k_out : a.v_out)[((int64_t)i * a.kv_tiles + h) * 128 + d] = r;
    const float top = a.dtype == kKvFp8 ? 448.f : 127.f;
    const float sc = amax > 0.f ? __fdiv_rn(amax, top) : 1.f;
    const float tq = __fmul_rn(r, __fdiv_rn(1.f, sc));
    uint8_t code;
    if (a.dtype == kKvFp8) {
      code = f32_to_e4m3(tq);
    } else {
      const float q = fminf(fmaxf(rintf(tq), -127.f), 127.f);
      code = (uint8_t)(int8_t)(int)q;
    }
    const int64_t p = pos0 + i, slot = a.ring ? p % a.slots : p;
    if (type == 1)
      a.kc[k_offset(h, slot, d, a.slots)] = code;
    else
      a.vc[v_offset(h, d, slot, a.slots)] = code;
    if (d == 0) (type == 1 ? a.ks : a.vs)[(int64_t)h * a.slots + slot] = sc;
  }
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ Params P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const GemvArgs& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = a.kblocks, S = P.split, ring = P.ring;
  // this CTA's job: tiles [t0, t0 + nt) x K blocks [k0, k0 + nkb)
  int t0, nt, k0, nkb, srank;
  if (S > 1) {
    t0 = blockIdx.x / S;
    nt = 1;
    srank = (int)(blockIdx.x % S);
    k0 = KB * srank / S;
    nkb = KB * (srank + 1) / S - k0;
  } else {
    t0 = blockIdx.x * P.tpc;
    nt = min(P.tpc, a.tiles - t0);
    srank = 0;
    k0 = 0;
    nkb = KB;
  }
  const int nunits = nt * nkb, nstages = (nunits + kStageUnits - 1) / kStageUnits;
  uint8_t* ringbuf = smem;
  uint8_t* bbuf = smem + P.off_b;
  float* pre_s = reinterpret_cast<float*>(smem + P.off_pre);   // [nkb * 4][8]
  float* red = reinterpret_cast<float*>(smem + P.off_red);     // [S][rpr][8]
  float* vsq = reinterpret_cast<float*>(smem + P.off_vsq);
  ArgCand* cand_s = reinterpret_cast<ArgCand*>(smem + P.off_cand);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P.off_bar);
  uint64_t* full = bars;
  uint64_t* empty = bars + ring;
  uint64_t* bfull = bars + 2 * ring;
  uint64_t* accfull = bars + 2 * ring + 1;    // [2]
  uint64_t* accempty = bars + 2 * ring + 3;   // [2]
  uint64_t* done = bars + 2 * ring + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + P.off_misc);
  float* pslice = reinterpret_cast<float*>(smem + P.off_misc + 16);   // [8] the rows' common prescale
  float* rowscale = reinterpret_cast<float*>(smem + P.off_misc + 48);   // [8]

  // ---- set-up: TMEM before the dependent launch (a dependent CTA on this SM may wait for our columns) ----
  if (S > 1) cluster_arrive_relaxed();   // every CTA of the cluster is running before the first remote store
  if (warp == 2) tmem_alloc(tmem_slot, P.tmem_cols);
  if (tid == 0) {
    for (int i = 0; i < ring; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(bfull, 1);
    mbar_init(&accfull[0], 1);
    mbar_init(&accfull[1], 1);
    mbar_init(&accempty[0], kTileRows);
    mbar_init(&accempty[1], kTileRows);
    mbar_init(done, 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  // A stage's units are contiguous in the weight (consecutive K blocks of one tile, or whole tiles when the K blocks
  // are not split), so a stage is one bulk copy: the bulk copies of one thread complete one after another, and a
  // few large copies stream far faster than many small ones.
  auto unit_src = [&](int u) {
    const int t = t0 + u / nkb, kb = k0 + u % nkb;
    return a.w + ((int64_t)t * KB + kb) * kUnitBytes;
  };
  const uint64_t wpol = l2_evict_first();
  auto issue_stage = [&](int st) {
    const int slot = st % ring, first = st * kStageUnits;
    const int cnt = min(kStageUnits, nunits - first);
    mbar_expect_tx(&full[slot], (uint32_t)cnt * kUnitBytes);
    if (a.l2_first)
      bulk_g2s_hint(ringbuf + slot * kStageUnits * kUnitBytes, unit_src(first), (uint32_t)cnt * kUnitBytes,
                    &full[slot], wpol);
    else
      bulk_g2s(ringbuf + slot * kStageUnits * kUnitBytes, unit_src(first), (uint32_t)cnt * kUnitBytes, &full[slot]);
  };
  if (tid == 0)
    for (int st = 0; st < ring && st < nstages; ++st) issue_stage(st);
  __syncwarp();

  // Loads that do not depend on the previous kernel (parameters no kernel of the step writes) go out before the
  // dependency wait, so that the finish after the MMAs does not wait for memory.
  const int m = a.m_dev ? *a.m_dev : a.m;
  float sgv[4] = {0.f, 0.f, 0.f, 0.f}, suv[4] = {0.f, 0.f, 0.f, 0.f};   // kEpiSwiglu: this thread's features
  TileOut ofin = {};                                                    // kEpiStore: the tile's output
  float rs_lr = 0.f, rs_h = 0.f;   // kEpiStore with row sums: the rate and h of this thread's finished element
  QkvPre qpre = {};
  if constexpr (EPI == kEpiSwiglu) {
    const int g0 = share_begin(4, srank, S), g1 = share_begin(4, srank + 1, S);
    const int quad = tid >> 2, qt = tid & 3, gl = quad >> 3;
    if (quad < (g1 - g0) * 8) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int f = t0 * 64 + 16 * (g0 + gl) + 4 * qt + c;
        if (f < a.features) {
          sgv[c] = a.sg[f];
          suv[c] = a.su[f];
        }
      }
    }
  } else if constexpr (EPI == kEpiStore) {
    if (a.outs) ofin = a.outs[t0];
    if (a.rsum && S > 1) {
      const int r0 = share_begin(kTileRows, srank, S), nr = share_begin(kTileRows, srank + 1, S) - r0;
      if (tid < nr * 8) rs_lr = a.rs_lr[t0 * kTileRows + r0 + tid % nr];
    }
  } else if constexpr (EPI == kEpiQkv) {
    qpre.pos0 = *a.pos0_dev;
    if (t0 < a.q_tiles) qpre.qscale = a.qscale[t0 * 128 + (tid & 127)];
    if (t0 >= a.q_tiles + 2 * a.kv_tiles && a.outs) qpre.out = a.outs[t0];
  }
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  if constexpr (EPI == kEpiStore) {   // h (the previous residual update's output): loaded long before the finish
    if (a.rsum && S > 1) {
      const int r0 = share_begin(kTileRows, srank, S), nr = share_begin(kTileRows, srank + 1, S) - r0;
      if (tid < nr * 8 && tid / nr < m) rs_h = a.rs_h[(int64_t)(tid / nr) * a.rs_ld + t0 * kTileRows + r0 + tid % nr];
    }
  }
  if constexpr (EPI == kEpiQkv) {
    // RoPE factors (written by the step's first kernel): q and k heads, this thread's rows
    if (t0 < a.q_tiles + a.kv_tiles) {
      const int i0 = share_begin(8, srank, S), i1 = share_begin(8, srank + 1, S), e = tid & 63;
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int i = i0 + 2 * it + (tid >> 7);
        if (i < i1) {
          qpre.cs[it] = a.rope_cos[i * 64 + e];
          qpre.sn[it] = a.rope_sin[i * 64 + e];
        }
      }
    }
  }

  // ---- the B operand of this CTA's K slice: the producer's digits, brought to one prescale per row ----
  // (a thread other than the weight producer issues the copy, so that it does not queue behind the weight stages)
  if (tid == 96) {
    mbar_expect_tx(bfull, (uint32_t)nkb * kBBlockBytes);
    bulk_g2s(bbuf, a.xb + (int64_t)k0 * kBBlockBytes, (uint32_t)nkb * kBBlockBytes, bfull);
  }
  __syncwarp();
  {
    const int i = warp;   // warp i: activation row i
    // the row's sum of squares over the producer's parts ([row][part]): lane l takes parts l, l + 32, ... (one wave
    // of coalesced loads, issued with the prescale loads below so that the two take one round trip)
    float pv[kSumsqLoads];
    if (EPI == kEpiStore && a.sumsq) {
#pragma unroll
      for (int u = 0; u < kSumsqLoads; ++u) {
        const int q = lane + 32 * u;
        pv[u] = q < a.nparts ? a.sumsq[(int64_t)i * a.nparts + q] : 0.f;
      }
    }
    float pmin = a.xb_fixed;
    if (!(a.xb_fixed > 0.f)) {
      // the slice's prescales ([group][row]) are one contiguous range: every thread loads a share (whole cache
      // lines per warp), then warp i takes row i's smallest from shared memory
      const float* src = a.xb_pre + (int64_t)k0 * 4 * 8;
      for (int e = tid; e < nkb * 4 * 8; e += kThreads) pre_s[e] = src[e];
      __syncthreads();
      pmin = 3.0e38f;
      for (int b = lane; b < nkb * 4; b += 32) pmin = fminf(pmin, pre_s[b * 8 + i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pmin = fminf(pmin, __shfl_xor_sync(0xffffffffu, pmin, o));
    }
    if (lane == 0) pslice[i] = pmin;
    if (EPI == kEpiStore) {
      // the parts summed in lane order, then a butterfly over the warp (a fixed order)
      float t = 1.f;
      if (a.sumsq) {
        t = pv[0];
#pragma unroll
        for (int u = 1; u < kSumsqLoads; ++u) t += pv[u];
        t = warp_sum(t);
        t = 1.f / sqrtf(t + 1e-6f);
      }
      if (lane == 0) rowscale[i] = t;
    }
  }
  wait_bar(bfull, 0, a.err);
  __syncthreads();
  if (!(a.xb_fixed > 0.f)) {
    // the scale words of the slice: word (K block kb, digit row r = 8 d + i) holds the scales of groups 4 kb .. 4 kb + 3,
    // each brought from its group's prescale to the row's smallest
    for (int e = tid; e < nkb * kDigitRows; e += kThreads) {
      const int kb = e / kDigitRows, r = e - kb * kDigitRows, i = r & 7;
      uint32_t* w = reinterpret_cast<uint32_t*>(bbuf + kb * kBBlockBytes + kBCodeBytes + sf_offset(r, 0));
      const uint32_t v = *w;
      const int ps = __float_as_int(pslice[i]);
      uint32_t o = 0u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = (__float_as_int(pre_s[(4 * kb + j) * 8 + i]) - ps) >> 23;
        o |= ue4m3_scale_down((v >> (8 * j)) & 0xffu, k) << (8 * j);
      }
      if (o != v) *w = o;
    }
    fence_proxy_async_smem();
  }
  __syncthreads();
  if (S > 1) cluster_wait();   // every thread: the cluster phase opened at the start

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      for (int st = ring; st < nstages; ++st) {
        const int slot = st % ring;
        wait_bar(&empty[slot], (uint32_t)((st / ring) - 1) & 1u, a.err);
        issue_stage(st);
      }
      // every issued copy has landed before the CTA may exit (normally long since)
      for (int slot = 0; slot < ring && slot < nstages; ++slot) {
        const int last = slot + ((nstages - 1 - slot) / ring) * ring;
        wait_bar(&full[slot], (uint32_t)(last / ring) & 1u, a.err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: the slice's activation scales go to TMEM once; per unit the weight scales, then the MMA.
    // One thread issues everything, so the per-unit work is kept to a few instructions: indices advance
    // incrementally and the descriptors by their start-address field (16-byte units, no carry out of 14 bits). ----
    if (lane == 0 && nt == 1) {
      // One tile (every split CTA): unit u is K block u, each B block's scales are used once and go to TMEM just
      // before its MMA, and a full stage is straight-line code (no per-unit branch: the issue loop stays short).
      tc_fence_after();
      const uint32_t ring_addr = smem_u32(ringbuf), b_addr = smem_u32(bbuf);
      const uint32_t sfb0 = tbase + kAccCols, sfa0 = sfb0 + 4 * (uint32_t)nkb;
      const uint64_t da0 = a_desc(ring_addr), dsfa0 = sf_desc(ring_addr + kUnitCodeBytes), db0 = a_desc(b_addr);
      const uint64_t dsfb0 = sf_desc(b_addr + kBCodeBytes);
      auto unit = [&](uint32_t ui, uint32_t kbi) {
        tc_cp_sf(sfb0 + 4 * kbi, dsfb0 + kbi * (kBBlockBytes >> 4));
        tc_cp_sf(sfa0 + 4 * ui, dsfa0 + ui * (kUnitBytes >> 4));
        tc_mma_fp4(tbase, da0 + ui * (kUnitBytes >> 4), db0 + kbi * (kBBlockBytes >> 4), sfa0 + 4 * ui,
                   sfb0 + 4 * kbi, kbi > 0 ? 1u : 0u);
      };
      int slot = 0;
      uint32_t phase = 0;
      for (int st = 0; st < nstages; ++st) {
        wait_bar(&full[slot], phase, a.err);
        tc_fence_after();
        const uint32_t u0 = (uint32_t)(slot * kStageUnits), kb0 = (uint32_t)(st * kStageUnits);
        const int cnt = nunits - st * kStageUnits;
        if (cnt >= kStageUnits) {
#pragma unroll
          for (int idx = 0; idx < kStageUnits; ++idx) unit(u0 + idx, kb0 + idx);
        } else {
          for (int idx = 0; idx < cnt; ++idx) unit(u0 + idx, kb0 + idx);
        }
        tc_commit(&empty[slot]);
        if (++slot == ring) {
          slot = 0;
          phase ^= 1u;
        }
      }
      tc_commit(&accfull[0]);
      tc_commit(done);
    } else if (lane == 0 && nkb % kStageUnits == 0) {
      // Several whole tiles whose K blocks fill whole stages (the head): the slice's activation scales go to TMEM
      // once; a stage is straight-line code; the accumulator switches (and waits for the epilogue) only at the
      // first stage of a tile and completes at its last.
      tc_fence_after();
      const uint32_t ring_addr = smem_u32(ringbuf), b_addr = smem_u32(bbuf);
      const uint32_t sfb0 = tbase + 2 * kAccCols, sfa0 = sfb0 + 4 * (uint32_t)nkb;
      for (int kb = 0; kb < nkb; ++kb) tc_cp_sf(sfb0 + 4 * kb, sf_desc(b_addr + (uint32_t)(kb * kBBlockBytes + kBCodeBytes)));
      const uint64_t da0 = a_desc(ring_addr), dsfa0 = sf_desc(ring_addr + kUnitCodeBytes), db0 = a_desc(b_addr);
      const int spt = nkb / kStageUnits;   // stages per tile
      int slot = 0, j = 0, sj = 0;
      uint32_t phase = 0;
      for (int st = 0; st < nstages; ++st) {
        if (sj == 0 && j >= 2) {
          wait_bar(&accempty[j & 1], (uint32_t)((j >> 1) - 1) & 1u, a.err);
        }
        wait_bar(&full[slot], phase, a.err);
        tc_fence_after();
        const uint32_t u0 = (uint32_t)(slot * kStageUnits), kb0 = (uint32_t)(sj * kStageUnits);
        const uint32_t tacc = tbase + (uint32_t)((j & 1) * kAccCols);
#pragma unroll
        for (int idx = 0; idx < kStageUnits; ++idx) {
          const uint32_t ui = u0 + idx, kbi = kb0 + idx;
          tc_cp_sf(sfa0 + 4 * ui, dsfa0 + ui * (kUnitBytes >> 4));
          tc_mma_fp4(tacc, da0 + ui * (kUnitBytes >> 4), db0 + kbi * (kBBlockBytes >> 4), sfa0 + 4 * ui,
                     sfb0 + 4 * kbi, kbi > 0 ? 1u : 0u);
        }
        tc_commit(&empty[slot]);
        if (++sj == spt) {
          tc_commit(&accfull[j & 1]);
          sj = 0;
          ++j;
        }
        if (++slot == ring) {
          slot = 0;
          phase ^= 1u;
        }
      }
      tc_commit(done);
    } else if (lane == 0) {
      tc_fence_after();
      const uint32_t ring_addr = smem_u32(ringbuf), b_addr = smem_u32(bbuf);
      const uint32_t acc_cols = nt > 1 ? 2 * kAccCols : kAccCols;
      const uint32_t sfb0 = tbase + acc_cols, sfa0 = sfb0 + 4 * (uint32_t)nkb;
      for (int kb = 0; kb < nkb; ++kb) tc_cp_sf(sfb0 + 4 * kb, sf_desc(b_addr + (uint32_t)(kb * kBBlockBytes + kBCodeBytes)));
      const uint64_t da0 = a_desc(ring_addr), dsfa0 = sf_desc(ring_addr + kUnitCodeBytes), db0 = a_desc(b_addr);
      int j = 0, kb = 0;
      for (int st = 0; st < nstages; ++st) {
        const int slot = st % ring, cnt = min(kStageUnits, nunits - st * kStageUnits);
        wait_bar(&full[slot], (uint32_t)(st / ring) & 1u, a.err);
        tc_fence_after();
        const uint32_t u0 = (uint32_t)(slot * kStageUnits);
        for (int idx = 0; idx < cnt; ++idx) {
          if (kb == 0 && j >= 2) {
            wait_bar(&accempty[j & 1], (uint32_t)((j >> 1) - 1) & 1u, a.err);
            tc_fence_after();
          }
          const uint32_t ui = u0 + (uint32_t)idx;
          const uint32_t sfa = sfa0 + 4 * ui;
          tc_cp_sf(sfa, dsfa0 + ui * (kUnitBytes >> 4));
          tc_mma_fp4(tbase + (uint32_t)((j & 1) * kAccCols), da0 + ui * (kUnitBytes >> 4),
                     db0 + (uint32_t)kb * (kBBlockBytes >> 4), sfa, sfb0 + 4 * (uint32_t)kb, kb > 0 ? 1u : 0u);
          if (++kb == nkb) {
            tc_commit(&accfull[j & 1]);
            kb = 0;
            ++j;
          }
        }
        tc_commit(&empty[slot]);
      }
      tc_commit(done);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---- epilogue: TMEM lane quarter q = warp - 4 holds tile rows 32 q .. 32 q + 31 ----
    const int q = warp - 4, r = 32 * q + lane;
    float inv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) inv[i] = 1.f / pslice[i];
    for (int j = 0; j < nt; ++j) {
      const int acc = j & 1, t = t0 + j;
      // the tile's output description (or logit scale) is loaded before the wait, off the MMAs' critical path
      TileOut o = {};
      float ls = 0.f;
      if constexpr (EPI == kEpiHead) {
        const int row = t * kTileRows + r;
        ls = row < a.vocab ? a.logit_scale[row] * a.g_head : 0.f;
      } else if constexpr (EPI != kEpiSwiglu) {
        if (a.outs) o = a.outs[t];
      }
      wait_bar(&accfull[acc], (uint32_t)(j >> 1) & 1u, a.err);
      tc_fence_after();
      float d[kDigitRows];
      const uint32_t taddr = tbase + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * kAccCols);
      tmem_ld16(taddr, *reinterpret_cast<float(*)[16]>(&d[0]));
      tmem_ld16(taddr + 16, *reinterpret_cast<float(*)[16]>(&d[16]));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&accempty[acc]);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        y[i] = ((d[i] + d[8 + i]) + (d[16 + i] + d[24 + i])) * inv[i];
      if constexpr (EPI == kEpiHead) {
        const int row = t * kTileRows + r;
        const bool ok = row < a.vocab;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float l = ok ? y[i] * ls : -INFINITY;
          if (ok && i < m) a.logits[(int64_t)i * a.vocab + row] = l;
          int li = row;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, l, o);
            const int oi = __shfl_xor_sync(0xffffffffu, li, o);
            if (ov > l || (ov == l && oi < li)) {
              l = ov;
              li = oi;
            }
          }
          if (lane == 0) cand_s[q * 8 + i] = ArgCand{l, li};
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (q == 0 && lane < 8) {
          ArgCand best = cand_s[lane];
          for (int qq = 1; qq < 4; ++qq) {
            const ArgCand c = cand_s[qq * 8 + lane];
            if (c.v > best.v || (c.v == best.v && c.i < best.i)) best = c;
          }
          a.cand[t * 8 + lane] = best;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      } else {
        float g;
        if constexpr (EPI == kEpiSwiglu)
          g = r < 64 ? a.g_gate : a.g_up;
        else
          g = r < 64 ? o.global_lo : o.global_hi;
#pragma unroll
        for (int i = 0; i < 8; ++i) y[i] *= g;
        if (EPI == kEpiStore && S == 1 && EPI != kEpiQkv) {
          if (r < o.rows)
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (i < m) o.y[(int64_t)i * o.ld + r] = y[i] * rowscale[i];
        } else {
          // push this CTA's part of row r to the cluster rank that finishes it
          int owner, slot;
          if constexpr (EPI == kEpiQkv) {   // ranks finish activation rows (whole heads)
            const int nil = (8 + S - 1) / S;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int ow = (i * S) / 8;
              float* dst = red + ((srank * nil) + (i - share_begin(8, ow, S))) * kTileRows + r;
              if (S == 1)
                *dst = y[i];
              else
                st_cluster_f32(dst, (uint32_t)ow, y[i]);
            }
            owner = -1;
            slot = 0;
          } else if constexpr (EPI == kEpiStore) {
            owner = (r * S) / kTileRows;
            slot = r - share_begin(kTileRows, owner, S);
          } else {
            const int f = r & 63;
            owner = ((f >> 4) * S) / 4;
            const int g0 = share_begin(4, owner, S), g1 = share_begin(4, owner + 1, S);
            slot = (r >= 64 ? 16 * (g1 - g0) : 0) + f - 16 * g0;
          }
          float* dst = red + (srank * P.rpr + slot) * 8;
          if (owner < 0) {
          } else if (S == 1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = y[i];
          } else {
            st_cluster_f32x8(dst, (uint32_t)owner, y);
          }
        }
      }
    }
  }
  // ---- split tiles meet in the cluster; SwiGLU pairs gate and up rows ----
  __syncthreads();
  if (EPI != kEpiHead && (S > 1 || EPI == kEpiSwiglu || EPI == kEpiQkv)) {
    if (S > 1) cluster_sync();
    const int t = t0;
    auto total = [&](int slot, int i) {
      float v = 0.f;
      for (int c = 0; c < S; ++c) v += red[(c * P.rpr + slot) * 8 + i];
      return v;
    };
    if constexpr (EPI == kEpiQkv) {
      qkv_finish(a, qpre, red, vsq, t, srank, S, m, tid);
    } else if constexpr (EPI == kEpiStore) {
      const TileOut& o = ofin;
      const int r0 = share_begin(kTileRows, srank, S), nr = share_begin(kTileRows, srank + 1, S) - r0;
      if (a.rsum) {
        // one element per thread (nr * 8 <= 256); the row sums over the nr lanes of a row (nr divides 32: aligned
        // groups of lanes), in a fixed butterfly order
        const int i = tid / nr, rl = tid % nr, r = r0 + rl;
        float y = 0.f;
        if (tid < nr * 8 && i < m && r < o.rows) {
          y = total(rl, i) * rowscale[i];
          o.y[(int64_t)i * o.ld + r] = y;
        }
        const float h = rs_h, lr = rs_lr, w = 1.f - lr;
        float v[5] = {h * h, y * y, w * w * h * h, lr * w * h * y, lr * lr * y * y};
        for (int off = nr >> 1; off > 0; off >>= 1)
#pragma unroll
          for (int k = 0; k < 5; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
        if (tid < nr * 8 && rl == 0) {
#pragma unroll
          for (int k = 0; k < 5; ++k) a.rsum[((int64_t)k * 8 + i) * gridDim.x + blockIdx.x] = v[k];
        }
      } else {
        for (int p = tid; p < nr * 8; p += kThreads) {
          const int i = p / nr, rl = p % nr, r = r0 + rl;
          if (i < m && r < o.rows) o.y[(int64_t)i * o.ld + r] = total(rl, i) * rowscale[i];
        }
      }
    } else {
      // quad (group g, row i): lane t holds features 16 g + 4 t .. + 3 of the tile; v -> digits of the next GEMV
      const int g0 = share_begin(4, srank, S), g1 = share_begin(4, srank + 1, S), nf = 16 * (g1 - g0);
      const int quad = tid >> 2, qt = tid & 3;
      const bool active = quad < (g1 - g0) * 8;
      const int gl = quad >> 3, i = quad & 7, g = g0 + gl;
      float v[4] = {0.f, 0.f, 0.f, 0.f}, sq = 0.f;
      if (active) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int fl = 16 * gl + 4 * qt + c, f = t * 64 + 16 * g + 4 * qt + c;
          if (f < a.features && i < m) {
            const float z = total(fl, i) * sgv[c];
            const float u = total(nf + fl, i) * suv[c];
            v[c] = z / (1.f + expf(-z)) * u;
          }
          sq += v[c] * v[c];
        }
      }
      if (tid < 8 * 64 / 4) vsq[i * 16 + ((gl * 4 + qt) & 15)] = active ? sq : 0.f;
      uint32_t code[kDigits], sf[kDigits];
      const float pb = digitize16_quad(v, code, sf);   // every lane of the warp takes part
      if (active) {
        store_digits_quad(a.vb + (int64_t)t * kBBlockBytes, i, g, qt, code, sf);
        if (qt == 0) a.vb_pre[((int64_t)t * 4 + g) * 8 + i] = pb;
      }
      __syncthreads();
      if (tid < 8) {
        float s2 = 0.f;
        for (int e = 0; e < 4 * (g1 - g0); ++e) s2 += vsq[tid * 16 + e];
        a.vsum[(int64_t)tid * gridDim.x + blockIdx.x] = s2;   // [row][part], part = t * S + srank
      }
    }
  }
  // ---- teardown: every tcgen05 operation has completed before the columns go back ----
  if (warp == 2) {
    if (lane == 0) wait_bar(done, 0, a.err);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, P.tmem_cols);
  }
}

// x f32 [m][k] -> digits: one quad per (16-input group, row)
__global__ void digitize_rows_kernel(const float* x, int m, int k, uint8_t* xb, float* xb_pre) {
  const int64_t quad = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 2;
  const int qt = threadIdx.x & 3;
  const int groups = (k + 63) / 64 * 4;   // every group of the padded K blocks
  const bool active = quad < (int64_t)groups * 8;
  const int g = active ? (int)(quad / 8) : 0, i = (int)(quad % 8);
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  if (active && i < m && 16 * g < k) {
    const float4 q = *reinterpret_cast<const float4*>(x + (int64_t)i * k + 16 * g + 4 * qt);
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    v[3] = q.w;
  }
  uint32_t code[kDigits], sf[kDigits];
  const float pb = digitize16_quad(v, code, sf);
  if (active) {
    store_digits_quad(xb + (int64_t)(g >> 2) * kBBlockBytes, i, g & 3, qt, code, sf);
    if (qt == 0) xb_pre[(int64_t)g * 8 + i] = pb;
  }
}

}  // namespace

GemvPlan plan_gemv(int tiles, int kblocks, int num_sms, int max_split, int max_tiles_per_cta) {
  GemvPlan p;
  for (int cps = 2; cps >= 1; --cps) {
    const int slots = num_sms * cps;
    if (tiles >= slots || max_split <= 1) {
      p.split = 1;
      p.tiles_per_cta = std::max(1, std::min(max_tiles_per_cta, (tiles + slots - 1) / slots));
      p.grid = (tiles + p.tiles_per_cta - 1) / p.tiles_per_cta;
    } else {
      p.split = std::max(1, std::min(std::min(max_split, kblocks), slots / tiles));
      p.tiles_per_cta = 1;
      p.grid = tiles * p.split;
    }
    const int slice = (kblocks + p.split - 1) / p.split;
    p.ring = cps == 2 ? 3 : kMaxRing;
    p.smem = smem_plan(p.ring, slice, p.split).total;
    if (cps == 2 && 2 * (p.smem + kPerCtaReserve) > kSmPerSm) continue;
    if (cps == 2 && tmem_columns(p.tiles_per_cta, slice, p.ring) > 256) continue;
    XTG_REQUIRE(p.smem <= kMaxSmem, "gemv: the K slice does not fit in shared memory");
    return p;
  }
  return p;
}

void launch_gemv(int epi, const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
  XTG_REQUIRE(epi != kEpiHead || p.split == 1, "gemv: the head epilogue takes whole tiles");
  XTG_REQUIRE(!a.sumsq || a.nparts <= 32 * kSumsqLoads, "gemv: at most 320 row-sum parts");
  XTG_REQUIRE(!a.rsum || (epi == kEpiStore && p.split >= 4 && p.split <= 8 && (p.split & (p.split - 1)) == 0),
              "gemv: row sums need a STORE GEMV split 4 or 8 ways");
  XTG_REQUIRE((epi != kEpiSwiglu && epi != kEpiQkv) || p.tiles_per_cta == 1,
              "gemv: the SwiGLU and q|k|v epilogues take one tile per CTA");
  XTG_REQUIRE(p.split >= 1 && p.split <= 8 && p.ring >= 1 && p.ring <= kMaxRing, "gemv: bad plan");
  Params P = {};
  P.a = a;
  P.a.pdl = pdl ? 1 : 0;
  P.split = p.split;
  P.tpc = p.tiles_per_cta;
  P.ring = p.ring;
  P.slice_max = (a.kblocks + p.split - 1) / p.split;
  const SmemPlan sp = smem_plan(p.ring, P.slice_max, p.split);
  P.rpr = sp.rpr;
  P.off_b = sp.off_b;
  P.off_pre = sp.off_pre;
  P.off_red = sp.off_red;
  P.off_vsq = sp.off_vsq;
  P.off_cand = sp.off_cand;
  P.off_bar = sp.off_bar;
  P.off_misc = sp.off_misc;
  const int cols = tmem_columns(p.tiles_per_cta, P.slice_max, p.ring);
  XTG_REQUIRE(cols <= 512, "gemv: the K slice's scales do not fit in TMEM");
  P.tmem_cols = cols <= 256 ? 256 : 512;
  // No more CTAs on an SM than its 512 TMEM columns hold: a CTA beyond that would wait in tcgen05.alloc until a
  // neighbour exits (measured: a third 76 KB O-projection CTA on an SM started ~7 us late). The dynamic shared memory
  // is raised, where needed, until one more CTA no longer fits.
  const int per_sm = 512 / (int)P.tmem_cols;
  const uint32_t smem_floor = (uint32_t)(kSmPerSm / (per_sm + 1) - kPerCtaReserve + 128);
  const uint32_t smem_bytes = std::max(sp.total, smem_floor);
  static std::atomic<uint64_t> optin[4];
  auto* k = epi == kEpiStore    ? gemv_kernel<kEpiStore>
            : epi == kEpiSwiglu ? gemv_kernel<kEpiSwiglu>
            : epi == kEpiQkv    ? gemv_kernel<kEpiQkv>
                                : gemv_kernel<kEpiHead>;
  ensure_smem_optin((const void*)k, (int)kMaxSmem, optin[epi]);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (p.split > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = p.split;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, k, P));
}

void digitize_rows(const float* x, int m, int k, uint8_t* xb, float* xb_pre, cudaStream_t s) {
  XTG_REQUIRE(k % 16 == 0 && m >= 0 && m <= 8, "digitize: k a multiple of 16, at most 8 rows");
  const int64_t threads = (int64_t)((k + 63) / 64 * 4) * 8 * 4;
  digitize_rows_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(x, m, k, xb, xb_pre);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg
