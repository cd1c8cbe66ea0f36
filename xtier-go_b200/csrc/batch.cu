// The batched verify step's own kernels (batch.h): what the GEMV's fused epilogues do for one sequence, done here for
// the 8 S rows of S sequences between the tcgen05 GEMMs: the embedding rows and RoPE tables (packs/dory/dory.cpp's
// head row decode, nvfp4_row at engine/src/kernels.cpp:34-45; rope at kernels.cpp:191-223), the q / k / v
// preparation and the KvCache::store of the new rows (dory.cpp:482-490, engine/src/kv.cpp:75-112), the scaled SwiGLU
// and its justnorm (kernels.cpp:225-234, dory.cpp:474-475) with the digits of the down projection's input, and the
// logit scale (dory.cpp:566-576) with the argmax (engine/src/sampler.cpp:8-13). Every sum has a fixed order.
#include "attention.h"
#include "batch.h"
#include "common.cuh"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kMaxClusterRanks = 8;

template <class Args>
void launch_with_pdl(void (*kernel)(Args), dim3 grid, dim3 block, size_t smem, const Args& args, cudaStream_t s,
                     bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, kernel, args));
}

__device__ __forceinline__ float head_weight(const uint8_t* w, int kblocks, float global, int row, int k) {
  const int t = row / kTileRows, r = row % kTileRows, b = k / kKBlock, kk = k % kKBlock;
  const uint8_t* unit = w + ((int64_t)t * kblocks + b) * kUnitBytes;
  const uint8_t byte = unit[a_code_offset(r, kk & ~1)];
  const uint8_t sc = unit[kUnitCodeBytes + sf_offset(r, kk >> 4)];
  const float s = __fmul_rn(e4m3_to_f32(sc), global);
  return __fmul_rn(e2m1_to_f32((kk & 1) ? byte >> 4 : byte & 15), s);
}

// grid (8, nseq): row i of sequence s; the row is digitized for the first GEMM too (its max sets its prescale)
__global__ void embed_batch_kernel(const EmbedBatchArgs a) {
  extern __shared__ float hrow[];   // [hidden]
  __shared__ float red[8];
  const int i = blockIdx.x, s = blockIdx.y, r = kMaxRows * s + i;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const StepParams& p = a.params[s];
  const int m = p.m;
  const int64_t pos0 = p.pos0;
  float* h = a.h + (int64_t)r * a.hidden;
  const int tok = i < m ? p.tokens[i] : 0;
  float mx = 0.f;
  for (int k = threadIdx.x; k < a.hidden; k += blockDim.x) {
    const float v = i >= m    ? 0.f
                    : a.table ? bf16_bits_to_f32(a.table[(int64_t)tok * a.hidden + k])
                              : head_weight(a.head, a.kblocks, a.global, tok, k);
    h[k] = v;
    hrow[k] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  const float pre = block_prescale(mx);
  if (threadIdx.x == 0) a.act_post[r] = 1.f / pre;
  const int groups = a.hidden / 16;
  for (int g0 = 0; g0 < groups; g0 += (int)blockDim.x / 4) {   // a quad per group; every lane takes part
    const int g = g0 + (int)(threadIdx.x >> 2), t = threadIdx.x & 3;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (g < groups)
#pragma unroll
      for (int c = 0; c < 4; ++c) v[c] = hrow[16 * g + 4 * t + c];
    uint32_t code[kGemmDigits], sf[kGemmDigits];
    digitize16_quad_n<kGemmDigits>(v, code, sf, pre);
    if (g < groups) store_gemm_digits_quad(a.act, r, g, t, code, sf);
  }
  // this row's RoPE factors for both thetas (FP32(pos) * inv_freq, then cos / sin)
  const int half = a.rope_half > 0 ? a.rope_half : 64;
  for (int e = threadIdx.x; e < 2 * half; e += blockDim.x) {
    const int th = e / half, f = e % half;
    const float ang = __fmul_rn((float)(pos0 + i), a.inv_freq[th * half + f]);
    float sn, c;
    sincosf(ang, &sn, &c);
    const int64_t at = (((int64_t)s * 2 + th) * kMaxRows + i) * half + f;
    a.rope_cos[at] = c;
    a.rope_sin[at] = sn;
  }
  // the ring's slot -> position table gains this step's rows (the attention masks positions >= pos0 anyway)
  if (threadIdx.x == 0 && i < m && a.ring_pos[s]) {
    const int64_t q = pos0 + i;
    a.ring_pos[s][q % a.ring] = (int32_t)q;
  }
}

// Sum (max) of v over the D threads of the block (D / 32 warps), every thread gets it; red: D / 32 floats, fixed
// order.
template <int D>
__device__ __forceinline__ float sum_heads(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = (red[0] + red[1]) + (red[2] + red[3]);
  if constexpr (D == 256) t += (red[4] + red[5]) + (red[6] + red[7]);
  return t;
}
template <int D>
__device__ __forceinline__ float max_heads(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  if constexpr (D == 256) t = fmaxf(t, fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])));
  return t;
}

// grid (2 heads + 2 kv_heads, 8 nseq), D threads: thread d of head column block h, activation row r = 8 s + i.
// The gate's blocks only sum the K parts (into part 0, which the combine reads). Also the 8-row step's q|k|v
// preparation at head dim 256 (nseq 1, one K part), where a head spans two of the GEMV's 128-row tiles.
template <int D>
__global__ void __launch_bounds__(D) qkv_prep_kernel(const QkvPrepArgs a) {
  constexpr int kHalf = D / 2;
  __shared__ float red[D / 32];
  __shared__ float xs[D];
  const int hb = blockIdx.x, r = blockIdx.y, s = r / kMaxRows, i = r % kMaxRows, d = threadIdx.x;
  const int nq = a.heads, nk = a.kv_heads;
  const int type = hb < nq ? 0 : hb < nq + nk ? 1 : hb < nq + 2 * nk ? 2 : 3;   // q, k, v, gate
  const int h = type == 0 ? hb : type == 1 ? hb - nq : type == 2 ? hb - nq - nk : hb - nq - 2 * nk;
  const int col = (type == 0 ? 0 : type == 1 ? nq * D : type == 2 ? (nq + nk) * D : (nq + 2 * nk) * D) + h * D + d;
  const float qs = type == 0 ? a.qscale[h * D + d] : 0.f;   // a parameter: before the wait
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const StepParams& p = a.params[s];
  if (i >= p.m) return;
  float x = 0.f;
  for (int k = 0; k < a.ksplit; ++k) x += a.proj[(int64_t)k * a.split_stride + (int64_t)r * a.proj_ld + col];
  if (type == 3) {
    if (a.ksplit > 1) const_cast<float*>(a.proj)[(int64_t)r * a.proj_ld + col] = x;
    return;
  }
  float v = x;
  if (type <= 1) {   // NeoX RoPE on (d, d + D / 2), then justnorm over the head
    xs[d] = x;
    __syncthreads();
    const int64_t at = (((int64_t)s * 2 + a.theta) * kMaxRows + i) * kHalf + (d & (kHalf - 1));
    const float c = a.rope_cos[at], sn = a.rope_sin[at];
    const float other = xs[d ^ kHalf];
    v = d < kHalf ? x * c - other * sn : x * c + other * sn;
    v *= 1.f / sqrtf(sum_heads<D>(v * v, red) + 1e-6f);
  }
  if (type == 0) {
    a.q_out[((int64_t)r * a.heads + h) * D + d] = v * qs;
    return;
  }
  // k / v: the prepared row, and its codes and scale in the sequence's cache (the KvCache::store rule)
  (type == 1 ? a.k_out : a.v_out)[((int64_t)r * a.kv_heads + h) * D + d] = v;
  const float amax = max_heads<D>(fabsf(v), red);
  const float top = a.dtype == kKvFp8 ? 448.f : 127.f;
  const float sc = amax > 0.f ? __fdiv_rn(amax, top) : 1.f;
  const float tq = __fmul_rn(v, __fdiv_rn(1.f, sc));
  uint8_t code;
  if (a.dtype == kKvFp8) {
    code = f32_to_e4m3(tq);
  } else {
    const float q = fminf(fmaxf(rintf(tq), -127.f), 127.f);
    code = (uint8_t)(int8_t)(int)q;
  }
  const KvSeq& kv = a.seqs[s];
  const int64_t pos = p.pos0 + i, slot = a.ring ? pos % kv.slots : pos;
  if (slot < 0 || slot >= kv.slots) {   // a position outside the cache: recorded, nothing written
    if (d == 0 && a.err) atomicExch(a.err, 4);
    return;
  }
  if (type == 1)
    kv.kc[k_offset(h, slot, d, kv.slots, D)] = code;
  else
    kv.vc[v_offset(h, d, slot, kv.slots, D)] = code;
  if (d == 0) (type == 1 ? kv.ks : kv.vs)[(int64_t)h * kv.slots + slot] = sc;
}

// One cluster of `C` CTAs per activation row (the 64 rows of the GEMM's activation tile; rows past a sequence's m,
// and past 8 nseq, get zero digits), CTA c the features F c / C .., a thread 4 consecutive features (a quad one
// 16-feature group). The row's sum of squares and max |v| meet over distributed shared memory (added in rank order).
__global__ void swiglu_batch_kernel(const SwigluBatchArgs a) {
  __shared__ float part[2][kMaxClusterRanks];
  __shared__ float red[2][32];
  const int tid = threadIdx.x, r = blockIdx.y, s = r / kMaxRows, i = r % kMaxRows, F = a.features;
  const int C = (int)gridDim.x, rank = (int)cluster_rank();
  const int f0 = rank * (F / C) + 4 * tid;
  cluster_arrive_relaxed();   // every CTA of the cluster is running before the first remote store (below)
  float sgv[4], suv[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {   // parameters: before the wait
    sgv[c] = a.sg[f0 + c];
    suv[c] = a.su[f0 + c];
  }
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = s < a.nseq && i < a.params[s].m;
  const float* gu = a.gu + (int64_t)r * 2 * F;
  float v[4] = {0.f, 0.f, 0.f, 0.f}, ss = 0.f, mx = 0.f;
  if (live) {
    const int base = 128 * (f0 >> 6) + (f0 & 63);   // 4 consecutive features share their 64-feature tile
    float4 g4 = *reinterpret_cast<const float4*>(gu + base), u4 = *reinterpret_cast<const float4*>(gu + base + 64);
    for (int k = 1; k < a.ksplit; ++k) {   // the K parts, in order
      const float4 gk = *reinterpret_cast<const float4*>(gu + k * a.split_stride + base);
      const float4 uk = *reinterpret_cast<const float4*>(gu + k * a.split_stride + base + 64);
      g4.x += gk.x; g4.y += gk.y; g4.z += gk.z; g4.w += gk.w;
      u4.x += uk.x; u4.y += uk.y; u4.z += uk.z; u4.w += uk.w;
    }
    const float gz[4] = {g4.x, g4.y, g4.z, g4.w}, gv[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float z = gz[c] * sgv[c];
      const float u = gv[c] * suv[c];
      v[c] = z / (1.f + expf(-z)) * u;
      ss += v[c] * v[c];
      mx = fmaxf(mx, fabsf(v[c]));
    }
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = ss;
    red[1][tid >> 5] = mx;
  }
  __syncthreads();
  cluster_wait();
  if (tid == 0) {
    float t = 0.f, m = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      t += red[0][w];
      m = fmaxf(m, red[1][w]);
    }
    for (int q = 0; q < C; ++q) {   // this CTA's part into every rank's table
      st_cluster_f32(&part[0][rank], (uint32_t)q, t);
      st_cluster_f32(&part[1][rank], (uint32_t)q, m);
    }
  }
  cluster_sync();
  float tot = 0.f, amax = 0.f;
  for (int q = 0; q < C; ++q) {
    tot += part[0][q];
    amax = fmaxf(amax, part[1][q]);
  }
  const float p = block_prescale(amax);
  if (rank == 0 && tid == 0) a.act_post[r] = (1.f / sqrtf(tot + 1e-6f)) * (1.f / p);
  uint32_t code[kGemmDigits], sf[kGemmDigits];
  digitize16_quad_n<kGemmDigits>(v, code, sf, p);   // whole warps: blockDim a multiple of 32
  store_gemm_digits_quad(a.act, r, f0 >> 4, tid & 3, code, sf);
}

// One cluster of C CTAs per activation row, a thread 4 consecutive dims (a quad one 16-dim group): the five sums that
// give |h|, |o| and |(1 - l) fa h + l fb o| (fa = 1 / |h|, fb = 1 / |o|) meet over distributed shared memory (added
// in rank order), then every CTA updates and digitizes its own dims.
__global__ void slerp_batch_kernel(const SlerpBatchArgs a) {
  __shared__ float part[5][kMaxClusterRanks];
  __shared__ float red[5][32];
  const int tid = threadIdx.x, r = blockIdx.y, s = r / kMaxRows, i = r % kMaxRows, H = a.hidden;
  const int C = (int)gridDim.x, rank = (int)cluster_rank();
  const int d0 = rank * (H / C) + 4 * tid;
  cluster_arrive_relaxed();   // every CTA of the cluster is running before the first remote store (below)
  const float4 l4 = *reinterpret_cast<const float4*>(a.lr + d0);   // a parameter: before the wait
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = i < a.params[s].m;
  float* hr = a.h + (int64_t)r * H;
  float4 h4 = make_float4(0.f, 0.f, 0.f, 0.f), o4 = h4;
  if (live) {
    h4 = *reinterpret_cast<const float4*>(hr + d0);
    const float* orow = a.o + (int64_t)r * H;
    o4 = *reinterpret_cast<const float4*>(orow + d0);
    for (int q = 1; q < a.o_parts; ++q) {   // the K parts, in order
      const float4 p4 = *reinterpret_cast<const float4*>(orow + q * a.o_stride + d0);
      o4.x += p4.x; o4.y += p4.y; o4.z += p4.z; o4.w += p4.w;
    }
  }
  const float hv[4] = {h4.x, h4.y, h4.z, h4.w}, ov[4] = {o4.x, o4.y, o4.z, o4.w}, lv[4] = {l4.x, l4.y, l4.z, l4.w};
  float v5[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float w = 1.f - lv[c];
    v5[0] += hv[c] * hv[c];
    v5[1] += ov[c] * ov[c];
    v5[2] += w * w * hv[c] * hv[c];
    v5[3] += lv[c] * w * hv[c] * ov[c];
    v5[4] += lv[c] * lv[c] * ov[c] * ov[c];
  }
#pragma unroll
  for (int k = 0; k < 5; ++k) v5[k] = warp_sum(v5[k]);
  if ((tid & 31) == 0)
#pragma unroll
    for (int k = 0; k < 5; ++k) red[k][tid >> 5] = v5[k];
  __syncthreads();
  cluster_wait();
  if (tid < 5) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[tid][w];
    for (int q = 0; q < C; ++q) st_cluster_f32(&part[tid][rank], (uint32_t)q, t);
  }
  cluster_sync();
  float tot[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    tot[k] = 0.f;
    for (int q = 0; q < C; ++q) tot[k] += part[k][q];
  }
  const float fa = 1.f / sqrtf(tot[0] + 1e-6f), fb = 1.f / sqrtf(tot[1] + 1e-6f);
  const float f = 1.f / sqrtf(fa * fa * tot[2] + 2.f * fa * fb * tot[3] + fb * fb * tot[4] + 1e-6f);
  float v[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) v[c] = live ? ((1.f - lv[c]) * fa * hv[c] + lv[c] * fb * ov[c]) * f : 0.f;
  if (live) *reinterpret_cast<float4*>(hr + d0) = make_float4(v[0], v[1], v[2], v[3]);
  uint32_t code[kGemmDigits], sf[kGemmDigits];
  digitize16_quad_n<kGemmDigits>(v, code, sf, kUnitPrescale);   // whole warps: blockDim a multiple of 32
  store_gemm_digits_quad(a.act, r, d0 >> 4, tid & 3, code, sf);
  if (rank == 0 && tid == 0) a.act_post[r] = 1.f / kUnitPrescale;
}

// one CTA per activation row
__global__ void __launch_bounds__(1024) scale_argmax_kernel(const ScaleArgmaxArgs a) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int r = blockIdx.x, s = r / kMaxRows, i = r % kMaxRows;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  if (a.epoch && r == 0 && threadIdx.x == 0) *a.epoch += 1u;
  if (i >= a.params[s].m) return;
  float* row = a.logits + (int64_t)r * a.vocab;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int k = threadIdx.x; k < a.vocab; k += blockDim.x) {
    const float l = row[k] * a.logit_scale[k];
    row[k] = l;
    if (l > v) {   // k rises: the first maximum of this thread's entries
      v = l;
      idx = k;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    bv[warp] = v;
    bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? bv[lane] : -INFINITY;
    idx = lane < nw ? bi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (lane == 0) a.argmax[r] = idx;
  }
}

}  // namespace

void launch_embed_batch(const EmbedBatchArgs& a, cudaStream_t s) {
  XTG_REQUIRE(a.nseq >= 1 && a.nseq <= kMaxBatch, "embed_batch: 1..8 sequences");
  XTG_REQUIRE(a.hidden % 64 == 0 && a.hidden <= 12288, "embed_batch: hidden a multiple of 64, at most 12288");
  launch_with_pdl(embed_batch_kernel, dim3(kMaxRows, a.nseq), dim3(256), (size_t)a.hidden * 4, a, s, a.pdl != 0);
}

void launch_qkv_prep(const QkvPrepArgs& a, cudaStream_t s) {
  XTG_REQUIRE(a.nseq >= 1 && a.nseq <= kMaxBatch && a.ksplit >= 1, "qkv_prep: 1..8 sequences");
  const int D = a.head_dim > 0 ? a.head_dim : 128;
  XTG_REQUIRE(D == 128 || D == 256, "qkv_prep: head_dim 128 or 256");
  if (D == 256)
    launch_with_pdl(qkv_prep_kernel<256>, dim3(2 * a.heads + 2 * a.kv_heads, kMaxRows * a.nseq), dim3(256), 0, a, s,
                    a.pdl != 0);
  else
    launch_with_pdl(qkv_prep_kernel<128>, dim3(2 * a.heads + 2 * a.kv_heads, kMaxRows * a.nseq), dim3(128), 0, a, s,
                    a.pdl != 0);
}

void launch_swiglu_batch(const SwigluBatchArgs& a, cudaStream_t s) {
  // the cluster size: the most CTAs per row (up to 8) whose threads (4 features each) fill whole warps
  int C = 0;
  for (int c = kMaxClusterRanks; c >= 1 && !C; c >>= 1)
    if (a.features % (128 * c) == 0 && a.features / c / 4 <= 1024) C = c;
  XTG_REQUIRE(C >= 1, "swiglu_batch: features a multiple of 128, at most 4096 per CTA");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, kGemmRows);
  cfg.blockDim = dim3(a.features / C / 4);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 2 : 1;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, swiglu_batch_kernel, a));
}

void launch_slerp_batch(const SlerpBatchArgs& a, cudaStream_t s) {
  int C = 0;   // the most CTAs per row (up to 8) whose threads (4 dims each) fill whole warps
  for (int c = kMaxClusterRanks; c >= 1 && !C; c >>= 1)
    if (a.hidden % (128 * c) == 0 && a.hidden / c / 4 <= 1024) C = c;
  XTG_REQUIRE(C >= 1 && a.nseq >= 1 && a.nseq <= kMaxBatch && a.o_parts >= 1, "slerp_batch: hidden a multiple of 128");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, kMaxRows * a.nseq);
  cfg.blockDim = dim3(a.hidden / C / 4);
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.pdl ? 2 : 1;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, slerp_batch_kernel, a));
}

void launch_scale_argmax(const ScaleArgmaxArgs& a, cudaStream_t s) {
  launch_with_pdl(scale_argmax_kernel, dim3(kMaxRows * a.nseq), dim3(1024), 0, a, s, a.pdl != 0);
}

}  // namespace xtg
