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
// contiguous run of blocks (split-K inside a tile when a run starts or ends mid-tile). A tile's parts land in a
// scratch slot each; the warp whose atomic increment completes the tile sums the parts in warp order (the same
// order every launch: deterministic) and runs the epilogue. Weight loads of a warp's first batch and an L2
// prefetch of its whole run are issued before griddepcontrol.wait, so they overlap the previous kernel.
#include "common.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kWarps = 8;
constexpr int kBatch = 4;   // blocks in flight per warp

__device__ __forceinline__ int64_t owner_of(int64_t u, int64_t units, int64_t total_warps) {
  return ((u + 1) * total_warps - 1) / units;
}

struct Frag {
  float c[4];
};

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

// One block: 4 k16 steps, each an MMA of 16 rows x 16 inputs x 8 activation rows.
__device__ __forceinline__ void block_mma(float (&acc)[4], const uint4 w, const uint2 s, const uint2* xb) {
  const uint32_t wr[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t sc = e4m3x2_to_f16x2(j < 2 ? (s.x >> (16 * j)) : (s.y >> (16 * (j - 2))));
    const uint32_t s_lo = __byte_perm(sc, 0, 0x1010), s_hi = __byte_perm(sc, 0, 0x3232);
    const uint32_t q = wr[j];
    const uint32_t a0 = hmul2_u32(e2m1x2_to_f16x2(q & 0xff), s_lo);
    const uint32_t a1 = hmul2_u32(e2m1x2_to_f16x2((q >> 8) & 0xff), s_hi);
    const uint32_t a2 = hmul2_u32(e2m1x2_to_f16x2((q >> 16) & 0xff), s_lo);
    const uint32_t a3 = hmul2_u32(e2m1x2_to_f16x2(q >> 24), s_hi);
    const uint2 b = xb[j * 32];
    mma_f16(acc, a0, a1, a2, a3, b.x, b.y);
  }
}


// The end of a warp's part of tile t (nb blocks): the epilogue when the part is the whole tile, else park it and,
// if this part completes the tile, sum all parts in warp order and run the epilogue.
template <int EPI>
__device__ __noinline__ void finish_part(const GemvArgs& a, int t, const float (&acc)[4], int nb, int64_t u0,
                                         int64_t gw, int64_t units, int64_t total_warps, int m,
                                         const float* rowscale, int lane) {
  if (nb == a.blocks) {
    epilogue<EPI>(a, t, acc, m, rowscale, lane);
    return;
  }
  const int64_t tile_begin = (int64_t)t * a.blocks, tile_end = tile_begin + a.blocks;
  const int slot = (t == (int)(u0 / a.blocks)) ? 0 : 1;
  reinterpret_cast<float4*>(a.partial)[(gw * 2 + slot) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  __threadfence();
  int old = 0;
  if (lane == 0) old = atomicAdd(&a.counters[t], nb);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old + nb != a.blocks) return;
  __threadfence();
  const int64_t wa = owner_of(tile_begin, units, total_warps), wb = owner_of(tile_end - 1, units, total_warps);
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t w = wa; w <= wb; ++w) {
    const int64_t wu0 = w * units / total_warps, wu1 = (w + 1) * units / total_warps;
    if (wu1 <= wu0) continue;   // a warp without blocks parked nothing
    const int64_t w_first_tile = wu0 / a.blocks;
    const int s2 = (t == w_first_tile) ? 0 : 1;
    const float4 p = __ldcg(reinterpret_cast<const float4*>(a.partial) + (w * 2 + s2) * 32 + lane);
    sum[0] += p.x;
    sum[1] += p.y;
    sum[2] += p.z;
    sum[3] += p.w;
  }
  if (lane == 0) a.counters[t] = 0;
  epilogue<EPI>(a, t, sum, m, rowscale, lane);
}

template <int EPI>
__global__ void __launch_bounds__(kWarps * 32, 2) gemv_kernel(const __grid_constant__ GemvArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t total_warps = (int64_t)gridDim.x * kWarps;
  const int64_t gw = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t units = (int64_t)a.tiles * a.blocks;
  const int64_t u0 = gw * units / total_warps, u1 = (gw + 1) * units / total_warps;
  __shared__ float rowscale[kMaxRows];
  __shared__ float red[32][kMaxRows];

  // issue the first batch of weight loads and an L2 prefetch of the whole run before waiting on the producer
  if (u1 > u0 && lane == 0) prefetch_l2(a.w + u0 * kBlockBytes, (uint32_t)((u1 - u0) * kBlockBytes));
  uint4 cw[kBatch];
  uint2 cs[kBatch];
  {
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int64_t u = u0 + i;
      if (u < u1) {
        const uint8_t* blk = a.w + u * kBlockBytes;
        cw[i] = __ldg(reinterpret_cast<const uint4*>(blk) + lane);
        cs[i] = __ldg(reinterpret_cast<const uint2*>(blk + 512) + (lane >> 2));
      }
    }
  }
  if (a.pdl) pdl_wait();
  const int m = a.m_dev ? *a.m_dev : a.m;
  if constexpr (EPI == kEpiStore) {
    if (a.sumsq) {
      const int n = threadIdx.x & 7, j0 = threadIdx.x >> 3;
      float s = 0.f;
      for (int p = j0; p < a.nparts; p += 32) s += a.sumsq[p * kMaxRows + n];
      red[j0][n] = s;
      __syncthreads();
      if (threadIdx.x < kMaxRows) {
        float t = 0.f;
        for (int j = 0; j < 32; ++j) t += red[j][threadIdx.x];
        rowscale[threadIdx.x] = 1.f / sqrtf(t + 1e-6f);
      }
    } else if (threadIdx.x < kMaxRows) {
      rowscale[threadIdx.x] = 1.f;
    }
    __syncthreads();
  }
  if (a.pdl) pdl_launch_next();

  const uint2* x16 = reinterpret_cast<const uint2*>(a.x16);
  if (u1 <= u0) return;
  int t = (int)(u0 / a.blocks);             // the tile of the current part
  int64_t tile_begin = (int64_t)t * a.blocks, first = u0;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t base = u0; base < u1; base += kBatch) {
    uint4 nw[kBatch];
    uint2 ns[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {   // the next batch, in flight while this one is multiplied
      const int64_t v = base + kBatch + i;
      if (v < u1) {
        const uint8_t* blk = a.w + v * kBlockBytes;
        nw[i] = __ldg(reinterpret_cast<const uint4*>(blk) + lane);
        ns[i] = __ldg(reinterpret_cast<const uint2*>(blk + 512) + (lane >> 2));
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int64_t v = base + i;
      if (v < u1) {
        if (v == tile_begin + a.blocks) {   // a tile ends inside the batch: finish its part, start the next
          finish_part<EPI>(a, t, acc, (int)(v - first), u0, gw, units, total_warps, m, rowscale, lane);
          ++t;
          tile_begin = v;
          first = v;
          acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        }
        block_mma(acc, cw[i], cs[i], x16 + (v - tile_begin) * 4 * 32 + lane);
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      cw[i] = nw[i];
      cs[i] = ns[i];
    }
  }
  finish_part<EPI>(a, t, acc, (int)(u1 - first), u0, gw, units, total_warps, m, rowscale, lane);
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

int64_t gemv_partial_floats(int grid) { return (int64_t)grid * kWarps * 2 * 32 * 4; }

void launch_gemv(int epi, const GemvArgs& a_in, int max_grid, cudaStream_t s, bool pdl) {
  GemvArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  // at least 8 blocks per warp where the weight is small; never more CTAs than the scratch was sized for
  const int64_t units = (int64_t)a.tiles * a.blocks;
  const int64_t want = (units + kWarps * 8 - 1) / (kWarps * 8);
  const int grid = (int)(want < max_grid ? (want > 0 ? want : 1) : max_grid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWarps * 32);
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
