// K1: NVFP4 weight x fp16 activation GEMV for the 1..8-row decode / verify step (the hot loop of
// engine/src/kernels.cpp:84-138 matmul_nvfp4, m <= 8).
//
// Why tensor cores at m = 8: streaming NVFP4 at HBM speed is ~23 weight bytes per clock per SM, and each code byte
// holds 2 weights used by 8 rows: 32 FMAs per byte, ~340 FP32 FMAs per clock per SM against the 128 the CUDA cores
// issue. So every E2M1 code pair is converted to f16x2 (cvt.rn.f16x2.e2m1x2) and multiplied by its E4M3 block
// scale (cvt.rn.f16x2.e4m3x2, hmul2) -- e2m1 x e4m3 has at most 6 significant bits and lies in [2^-10, 2688], so
// this product is EXACT in fp16 -- and fed to mma.m16n8k16 (f32 accumulation) as the A operand, 16 weight rows x 16
// inputs; the activations (<= 8 rows, zero padded) are the B operand. The per-tensor global scale is applied in
// the epilogue. Compared with the reference's order (per-16 group sum in FP32, times the scale) only the FP32
// rounding of the sums differs, and the activations are rounded once to fp16.
//
// Work split: the weight is a stream of 576-byte blocks (weights.cu). Every warp of the grid takes an equal
// contiguous run of blocks (split-K inside a tile when a run starts or ends mid-tile), so the warps of a CTA cover
// one contiguous run and the grid covers the weight exactly once. Each warp streams its run through its own ring
// of shared-memory stages with bulk copies (cp.async.bulk global -> shared, completion on an mbarrier; no
// multicast); the first stages are issued before griddepcontrol.wait, since the weights do not depend on the
// previous kernel, and the kernel lets its dependent launch at once, so the next kernel's copies start while this
// one finishes. A tile split between warps of one CTA is summed in shared memory in warp order; a tile split
// between CTAs goes through a global scratch slot per CTA, and the CTA whose atomic increment completes the tile
// sums the CTA parts in CTA order. Every sum has a fixed order, so results are the same every launch.
#include "common.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kWarps = 8;
constexpr int kStageBlocks = 4;                           // blocks per bulk copy
constexpr int kStages = 3;                                // copies in flight per warp
constexpr int kStageBytes = kStageBlocks * kBlockBytes;   // 2304

struct GemvSmem {
  unsigned char ring[kWarps][kStages][kStageBytes];
  uint64_t bar[kWarps][kStages];
  float4 part[kWarps][2][32];   // split-tile parts of each warp: [0] its first tile, [1] its last
  float rowscale[kMaxRows];
  float red[32][kMaxRows];
};

__device__ __forceinline__ int64_t owner_of(int64_t u, int64_t units, int64_t total_warps) {
  return ((u + 1) * total_warps - 1) / units;
}

template <int EPI>
__device__ __forceinline__ void epilogue(const GemvArgs& a, int t, const float (&acc)[4], int m, const float* rowscale,
                                         int lane) {
  const int g = lane >> 2, tq = lane & 3;
  const int n0 = 2 * tq, n1 = 2 * tq + 1;
  if constexpr (EPI == kEpiStore) {
    const TileOut o = a.outs[t];
    const float s0 = o.global * rowscale[n0], s1 = o.global * rowscale[n1];
    if (g < o.rows) {
      if (n0 < m) o.y[(int64_t)n0 * o.ld + g] = acc[0] * s0;
      if (n1 < m) o.y[(int64_t)n1 * o.ld + g] = acc[1] * s1;
    }
    if (g + 8 < o.rows) {
      if (n0 < m) o.y[(int64_t)n0 * o.ld + g + 8] = acc[2] * s0;
      if (n1 < m) o.y[(int64_t)n1 * o.ld + g + 8] = acc[3] * s1;
    }
  } else if constexpr (EPI == kEpiSwiglu) {
    const int f = t * 8 + g;
    float v0 = 0.f, v1 = 0.f;
    if (f < a.features) {
      const float sg = a.sg[f], su = a.su[f];
      const float z0 = acc[0] * a.g_gate * sg, z1 = acc[1] * a.g_gate * sg;
      v0 = z0 / (1.f + expf(-z0)) * (acc[2] * a.g_up * su);
      v1 = z1 / (1.f + expf(-z1)) * (acc[3] * a.g_up * su);
      if (n0 >= m) v0 = 0.f;
      if (n1 >= m) v1 = 0.f;
      a.v16[frag_offset_halves(f, n0)] = __half_as_ushort(__float2half_rn(v0));
      a.v16[frag_offset_halves(f, n1)] = __half_as_ushort(__float2half_rn(v1));
      if (a.vout) {
        if (n0 < m) a.vout[(int64_t)n0 * a.features + f] = v0;
        if (n1 < m) a.vout[(int64_t)n1 * a.features + f] = v1;
      }
    }
    // sum of squares over the tile's 8 features, per activation row (fixed shuffle order)
    float q0 = v0 * v0, q1 = v1 * v1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      q0 += __shfl_xor_sync(0xffffffffu, q0, o);
      q1 += __shfl_xor_sync(0xffffffffu, q1, o);
    }
    if (g == 0) {
      a.vsum[t * 8 + n0] = q0;
      a.vsum[t * 8 + n1] = q1;
    }
  } else {   // kEpiHead
    const int r0 = t * 16 + g, r1 = r0 + 8;
    float l[4];
    l[0] = r0 < a.vocab ? acc[0] * a.g_head * a.logit_scale[r0] : -INFINITY;
    l[1] = r0 < a.vocab ? acc[1] * a.g_head * a.logit_scale[r0] : -INFINITY;
    l[2] = r1 < a.vocab ? acc[2] * a.g_head * a.logit_scale[r1] : -INFINITY;
    l[3] = r1 < a.vocab ? acc[3] * a.g_head * a.logit_scale[r1] : -INFINITY;
    if (r0 < a.vocab) {
      if (n0 < m) a.logits[(int64_t)n0 * a.vocab + r0] = l[0];
      if (n1 < m) a.logits[(int64_t)n1 * a.vocab + r0] = l[1];
    }
    if (r1 < a.vocab) {
      if (n0 < m) a.logits[(int64_t)n0 * a.vocab + r1] = l[2];
      if (n1 < m) a.logits[(int64_t)n1 * a.vocab + r1] = l[3];
    }
    // the tile's best row per activation row; ties go to the lower vocabulary index
    float bv0 = l[0], bv1 = l[1];
    int bi0 = r0, bi1 = r0;
    if (l[2] > bv0) { bv0 = l[2]; bi0 = r1; }
    if (l[3] > bv1) { bv1 = l[3]; bi1 = r1; }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      const float ov0 = __shfl_xor_sync(0xffffffffu, bv0, o), ov1 = __shfl_xor_sync(0xffffffffu, bv1, o);
      const int oi0 = __shfl_xor_sync(0xffffffffu, bi0, o), oi1 = __shfl_xor_sync(0xffffffffu, bi1, o);
      if (ov0 > bv0 || (ov0 == bv0 && oi0 < bi0)) { bv0 = ov0; bi0 = oi0; }
      if (ov1 > bv1 || (ov1 == bv1 && oi1 < bi1)) { bv1 = ov1; bi1 = oi1; }
    }
    if (g == 0) {
      a.cand[t * 8 + n0] = ArgCand{bv0, bi0};
      a.cand[t * 8 + n1] = ArgCand{bv1, bi1};
    }
  }
}

// One block: 4 k16 steps, each an MMA of 16 rows x 16 inputs x 8 activation rows; even steps accumulate into acc,
// odd steps into acc2 (two independent MMA chains). xb: this block's activation fragments (two uint4, a pair of
// steps each).
__device__ __forceinline__ void block_mma2(float (&acc)[4], float (&acc2)[4], const uint4 w, const uint2 s,
                                           const uint4* xb) {
  const uint4 b01 = xb[0], b23 = xb[32];
  const uint32_t bx[4] = {b01.x, b01.z, b23.x, b23.z}, by[4] = {b01.y, b01.w, b23.y, b23.w};
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sc = e4m3x2_to_f16x2(j < 2 ? (s.x >> (16 * j)) : (s.y >> (16 * (j - 2))));
    const __half2 sh = *reinterpret_cast<const __half2*>(&sc);
    const __half2 s_lo = __low2half2(sh), s_hi = __high2half2(sh);
    uint32_t c[4];
    e2m1x8_to_f16x2x4(wr[j], c);
    const __half2 h0 = __hmul2(*reinterpret_cast<const __half2*>(&c[0]), s_lo);
    const __half2 h1 = __hmul2(*reinterpret_cast<const __half2*>(&c[1]), s_hi);
    const __half2 h2 = __hmul2(*reinterpret_cast<const __half2*>(&c[2]), s_lo);
    const __half2 h3 = __hmul2(*reinterpret_cast<const __half2*>(&c[3]), s_hi);
    const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&h0), a1 = *reinterpret_cast<const uint32_t*>(&h1);
    const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&h2), a3 = *reinterpret_cast<const uint32_t*>(&h3);
    if (j & 1)
      mma_f16(acc2, a0, a1, a2, a3, bx[j], by[j]);
    else
      mma_f16(acc, a0, a1, a2, a3, bx[j], by[j]);
  }
}

// The parts of tile t held by CTA warps wa..wb (warp indices within the CTA), summed in warp order. A warp's part
// of t sits in slot 0 when t is the first tile of its run, else in slot 1.
__device__ __forceinline__ float4 cta_sum(const GemvSmem& sm, int t, int wa, int wb, int64_t cta_warp0,
                                          int64_t units, int64_t total_warps, int blocks, int lane) {
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int v = wa; v <= wb; ++v) {
    const int64_t g = cta_warp0 + v;
    const int64_t v0 = g * units / total_warps, v1 = (g + 1) * units / total_warps;
    if (v1 <= v0) continue;
    const float4 p = sm.part[v][(t == (int)(v0 / blocks)) ? 0 : 1][lane];
    s.x += p.x;
    s.y += p.y;
    s.z += p.z;
    s.w += p.w;
  }
  return s;
}

template <int EPI>
__global__ void __launch_bounds__(kWarps * 32, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  GemvSmem& sm = *reinterpret_cast<GemvSmem*>(smem_raw);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t total_warps = (int64_t)gridDim.x * kWarps;
  const int64_t cta_warp0 = (int64_t)blockIdx.x * kWarps;
  const int64_t gw = cta_warp0 + warp;
  const int64_t units = (int64_t)a.tiles * a.blocks;
  const int64_t u0 = gw * units / total_warps, u1 = (gw + 1) * units / total_warps;
  const int64_t cta_u0 = cta_warp0 * units / total_warps, cta_u1 = (cta_warp0 + kWarps) * units / total_warps;
  const int n = (int)(u1 - u0);   // this warp's blocks
  const int nst = (n + kStageBlocks - 1) / kStageBlocks;
  const uint8_t* src = a.w + u0 * kBlockBytes;
  uint64_t* bars = sm.bar[warp];
  auto issue = [&](int st) {   // lane 0: stage st of the run into its ring slot
    const int slot = st % kStages;
    const int cnt = n - st * kStageBlocks < kStageBlocks ? n - st * kStageBlocks : kStageBlocks;
    const uint32_t bytes = (uint32_t)cnt * kBlockBytes;
    mbar_expect_tx(&bars[slot], bytes);
    bulk_g2s(sm.ring[warp][slot], src + (int64_t)st * kStageBytes, bytes, &bars[slot]);
  };
  // the weights do not depend on the previous kernel: start streaming before waiting on it
  if (lane == 0 && n > 0) {
#pragma unroll
    for (int j = 0; j < kStages; ++j) mbar_init(&bars[j], 1);
    mbar_init_fence();
    for (int st = 0; st < kStages && st < nst; ++st) issue(st);
  }
  __syncwarp();
  if (a.pdl) {
    pdl_launch_next();
    pdl_wait();
  }
  const int m = a.m_dev ? *a.m_dev : a.m;
  if constexpr (EPI == kEpiStore) {
    if (a.sumsq) {
      const int r = threadIdx.x & 7, j0 = threadIdx.x >> 3;
      float acc = 0.f;
      for (int p = j0; p < a.nparts; p += 32) acc += a.sumsq[p * kMaxRows + r];
      sm.red[j0][r] = acc;
      __syncthreads();
      if (threadIdx.x < kMaxRows) {
        float t = 0.f;
        for (int j = 0; j < 32; ++j) t += sm.red[j][threadIdx.x];
        sm.rowscale[threadIdx.x] = 1.f / sqrtf(t + 1e-6f);
      }
    } else if (threadIdx.x < kMaxRows) {
      sm.rowscale[threadIdx.x] = 1.f;
    }
    __syncthreads();
  }
  const float* rowscale = sm.rowscale;
  const uint4* x16 = reinterpret_cast<const uint4*>(a.x16);
  const int first_tile = n > 0 ? (int)(u0 / a.blocks) : -1;
  if (n > 0) {
    int t = first_tile;
    int kb = (int)(u0 - (int64_t)t * a.blocks);   // block index inside tile t
    int part_kb0 = kb;
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t parity = 0;
    // the end of tile t's part: the epilogue for a whole tile, else a shared-memory slot
    auto tile_done = [&]() {
      float f[4] = {acc[0] + acc2[0], acc[1] + acc2[1], acc[2] + acc2[2], acc[3] + acc2[3]};
      if (part_kb0 == 0)
        epilogue<EPI>(a, t, f, m, rowscale, lane);
      else
        sm.part[warp][t == first_tile ? 0 : 1][lane] = make_float4(f[0], f[1], f[2], f[3]);
      ++t;
      kb = 0;
      part_kb0 = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = acc2[q] = 0.f;
    };
    for (int st = 0; st < nst; ++st) {
      const int slot = st % kStages;
      mbar_wait_bounded(&bars[slot], (parity >> slot) & 1u, lane == 0 ? a.err : nullptr);
      parity ^= 1u << slot;
      const unsigned char* buf = sm.ring[warp][slot] + lane * 16;
      const unsigned char* sbuf = sm.ring[warp][slot] + 512 + (lane >> 2) * 8;
      const int cnt = n - st * kStageBlocks < kStageBlocks ? n - st * kStageBlocks : kStageBlocks;
      if (cnt == kStageBlocks && kb + kStageBlocks <= a.blocks) {   // the common case: no boundary inside
        const uint4* xb = x16 + kb * 64 + lane;
#pragma unroll
        for (int i = 0; i < kStageBlocks; ++i)
          block_mma2(acc, acc2, *reinterpret_cast<const uint4*>(buf + i * kBlockBytes),
                     *reinterpret_cast<const uint2*>(sbuf + i * kBlockBytes), xb + i * 64);
        kb += kStageBlocks;
        if (kb == a.blocks) tile_done();
      } else {
        for (int i = 0; i < cnt; ++i) {
          block_mma2(acc, acc2, *reinterpret_cast<const uint4*>(buf + i * kBlockBytes),
                     *reinterpret_cast<const uint2*>(sbuf + i * kBlockBytes), x16 + kb * 64 + lane);
          if (++kb == a.blocks) tile_done();
        }
      }
      __syncwarp();
      if (lane == 0 && st + kStages < nst) {   // the slot was read: refill it with the run's next stage
        fence_proxy_async_smem();
        issue(st + kStages);
      }
    }
    if (kb > 0)   // the run ends inside tile t
      sm.part[warp][t == first_tile ? 0 : 1][lane] =
          make_float4(acc[0] + acc2[0], acc[1] + acc2[1], acc[2] + acc2[2], acc[3] + acc2[3]);
  }
  __syncthreads();
  if (n <= 0) return;
  // ---- split tiles: the last warp of the CTA that covers a tile sums the CTA's parts of it ----
  const int last_tile = (int)((u1 - 1) / a.blocks);
  for (int which = 0; which < 2; ++which) {
    const int t = which == 0 ? first_tile : last_tile;
    if (which == 1 && last_tile == first_tile) break;
    const int64_t tb = (int64_t)t * a.blocks, te = tb + a.blocks;
    const int64_t pb = u0 > tb ? u0 : tb, pe = u1 < te ? u1 : te;   // this warp's part of t
    if (pb == tb && pe == te) continue;                              // whole tile: done in the loop
    if (!(pe == te || u1 == cta_u1)) continue;                        // a later warp of the CTA continues t
    const int64_t owner_first = ((tb + 1) * total_warps - 1) / units;
    const int wa = (int)((owner_first > cta_warp0 ? owner_first : cta_warp0) - cta_warp0);
    const float4 s4 = cta_sum(sm, t, wa, warp, cta_warp0, units, total_warps, a.blocks, lane);
    float f[4] = {s4.x, s4.y, s4.z, s4.w};
    if (tb >= cta_u0 && te <= cta_u1) {   // every part of t is in this CTA
      epilogue<EPI>(a, t, f, m, rowscale, lane);
      continue;
    }
    // t continues in another CTA: park this CTA's sum; the CTA completing t sums the CTA parts in CTA order
    const int cta_first_tile = (int)(cta_u0 / a.blocks);
    const int cslot = t == cta_first_tile ? 0 : 1;
    reinterpret_cast<float4*>(a.partial)[((int64_t)blockIdx.x * 2 + cslot) * 32 + lane] = s4;
    __threadfence();
    const int covered = (int)((te < cta_u1 ? te : cta_u1) - (tb > cta_u0 ? tb : cta_u0));
    int old = 0;
    if (lane == 0) old = atomicAdd(&a.counters[t], covered);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + covered != a.blocks) continue;
    __threadfence();
    const int64_t ca = (((tb + 1) * total_warps - 1) / units) / kWarps;
    const int64_t cb = (((te) * total_warps - 1) / units) / kWarps;
    float sum[4] = {0.f, 0.f, 0.f, 0.f};
    for (int64_t c = ca; c <= cb; ++c) {
      const int64_t c0 = c * kWarps * units / total_warps, c1 = (c + 1) * kWarps * units / total_warps;
      if (c1 <= c0) continue;
      const int cs2 = t == (int)(c0 / a.blocks) ? 0 : 1;
      const float4 p = __ldcg(reinterpret_cast<const float4*>(a.partial) + (c * 2 + cs2) * 32 + lane);
      sum[0] += p.x;
      sum[1] += p.y;
      sum[2] += p.z;
      sum[3] += p.w;
    }
    if (lane == 0) a.counters[t] = 0;
    epilogue<EPI>(a, t, sum, m, rowscale, lane);
  }
}

// x f32 [m][k] -> fragments; one thread per (k pair, row).
__global__ void pack_activations_kernel(const float* x, int m, int k, int kp, uint32_t* x16) {
  const int64_t total = (int64_t)(kp / 2) * kMaxRows;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % kMaxRows), kk = (int)(i / kMaxRows) * 2;
    float v0 = 0.f, v1 = 0.f;
    if (n < m && kk < k) {
      v0 = x[(int64_t)n * k + kk];
      v1 = kk + 1 < k ? x[(int64_t)n * k + kk + 1] : 0.f;
    }
    x16[frag_offset_halves(kk, n) >> 1] = pack_f16x2(v0, v1);
  }
}

}  // namespace

int gemv_grid(int num_sms) { return num_sms * 2; }

int64_t gemv_partial_floats(int grid) { return (int64_t)grid * 2 * 32 * 4; }

void launch_gemv(int epi, const GemvArgs& a_in, int max_grid, cudaStream_t s, bool pdl) {
  GemvArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  // at least 8 blocks per warp where the weight is small; never more CTAs than the scratch was sized for
  const int64_t units = (int64_t)a.tiles * a.blocks;
  const int64_t want = (units + kWarps * 8 - 1) / (kWarps * 8);
  const int grid = (int)(want < max_grid ? (want > 0 ? want : 1) : max_grid);
  static bool attr_set[3] = {false, false, false};
  if (!attr_set[epi]) {
    auto* k = epi == kEpiStore ? gemv_kernel<kEpiStore> : epi == kEpiSwiglu ? gemv_kernel<kEpiSwiglu> : gemv_kernel<kEpiHead>;
    XTG_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(GemvSmem)));
    attr_set[epi] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = sizeof(GemvSmem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (epi == kEpiStore)
    XTG_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<kEpiStore>, a));
  else if (epi == kEpiSwiglu)
    XTG_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<kEpiSwiglu>, a));
  else
    XTG_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<kEpiHead>, a));
}

void pack_activations(const float* x, int m, int k, uint32_t* x16, cudaStream_t s) {
  const int kp = packed_blocks(k) * 64;
  const int64_t total = (int64_t)(kp / 2) * kMaxRows;
  const int grid = (int)((total + 255) / 256);
  pack_activations_kernel<<<grid, 256, 0, s>>>(x, m, k, kp, x16);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg
