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

// grid (8, nseq): row i of sequence s
__global__ void embed_batch_kernel(const EmbedBatchArgs a) {
  const int i = blockIdx.x, s = blockIdx.y;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const StepParams& p = a.params[s];
  const int m = p.m;
  const int64_t pos0 = p.pos0;
  float* h = a.h + (int64_t)(8 * s + i) * a.hidden;
  const int tok = i < m ? p.tokens[i] : 0;
  for (int k = threadIdx.x; k < a.hidden; k += blockDim.x)
    h[k] = i < m ? head_weight(a.head, a.kblocks, a.global, tok, k) : 0.f;
  // this row's RoPE factors for both thetas (FP32(pos) * inv_freq, then cos / sin)
  for (int e = threadIdx.x; e < 2 * 64; e += blockDim.x) {
    const int th = e >> 6, f = e & 63;
    const float ang = __fmul_rn((float)(pos0 + i), a.inv_freq[th * 64 + f]);
    float sn, c;
    sincosf(ang, &sn, &c);
    const int64_t at = (((int64_t)s * 2 + th) * kMaxRows + i) * 64 + f;
    a.rope_cos[at] = c;
    a.rope_sin[at] = sn;
  }
  // the ring's slot -> position table gains this step's rows (the attention masks positions >= pos0 anyway)
  if (threadIdx.x == 0 && i < m && a.ring_pos[s]) {
    const int64_t q = pos0 + i;
    a.ring_pos[s][q % a.ring] = (int32_t)q;
  }
}

// Sum of v over the 128 threads of the block (4 warps), every thread gets it; red: 4 floats, fixed order.
__device__ __forceinline__ float sum128(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return (red[0] + red[1]) + (red[2] + red[3]);
}
__device__ __forceinline__ float max128(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

// grid (2 heads + 2 kv_heads, 8 nseq), 128 threads: thread d of head column block h, activation row r = 8 s + i.
// The gate's blocks only sum the K parts (into part 0, which the combine reads).
__global__ void __launch_bounds__(128) qkv_prep_kernel(const QkvPrepArgs a) {
  __shared__ float red[4];
  __shared__ float xs[128];
  const int hb = blockIdx.x, r = blockIdx.y, s = r / kMaxRows, i = r % kMaxRows, d = threadIdx.x;
  const int nq = a.heads, nk = a.kv_heads;
  const int type = hb < nq ? 0 : hb < nq + nk ? 1 : hb < nq + 2 * nk ? 2 : 3;   // q, k, v, gate
  const int h = type == 0 ? hb : type == 1 ? hb - nq : type == 2 ? hb - nq - nk : hb - nq - 2 * nk;
  const int col = (type == 0 ? 0 : type == 1 ? nq * 128 : type == 2 ? (nq + nk) * 128 : (nq + 2 * nk) * 128) +
                  h * 128 + d;
  const float qs = type == 0 ? a.qscale[h * 128 + d] : 0.f;   // a parameter: before the wait
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
  if (type <= 1) {   // NeoX RoPE on (d, d + 64), then justnorm over the head
    xs[d] = x;
    __syncthreads();
    const int64_t at = (((int64_t)s * 2 + a.theta) * kMaxRows + i) * 64 + (d & 63);
    const float c = a.rope_cos[at], sn = a.rope_sin[at];
    const float other = xs[d ^ 64];
    v = d < 64 ? x * c - other * sn : x * c + other * sn;
    v *= 1.f / sqrtf(sum128(v * v, red) + 1e-6f);
  }
  if (type == 0) {
    a.q_out[((int64_t)r * a.heads + h) * 128 + d] = v * qs;
    return;
  }
  // k / v: the prepared row, and its codes and scale in the sequence's cache (the KvCache::store rule)
  (type == 1 ? a.k_out : a.v_out)[((int64_t)r * a.kv_heads + h) * 128 + d] = v;
  const float amax = max128(fabsf(v), red);
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
  if (type == 1)
    kv.kc[k_offset(h, slot, d, kv.slots)] = code;
  else
    kv.vc[v_offset(h, d, slot, kv.slots)] = code;
  if (d == 0) (type == 1 ? kv.ks : kv.vs)[(int64_t)h * kv.slots + slot] = sc;
}

constexpr int kSwThreads = 1024;

// one CTA per activation row (the 64 rows of the GEMM's activation tile; rows past a sequence's m, and past 8 nseq,
// get zero digits)
__global__ void __launch_bounds__(kSwThreads) swiglu_batch_kernel(const SwigluBatchArgs a) {
  extern __shared__ float vrow[];   // [features]
  __shared__ float red[32], redm[32];
  const int r = blockIdx.x, s = r / kMaxRows, i = r % kMaxRows, F = a.features, tid = threadIdx.x;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = s < a.nseq && i < a.params[s].m;
  const float* gu = a.gu + (int64_t)r * 2 * F;
  float ss = 0.f, mx = 0.f;
  for (int f = tid; f < F; f += kSwThreads) {
    float v = 0.f;
    if (live) {
      const int base = 128 * (f >> 6) + (f & 63);
      float gz = gu[base], gv = gu[base + 64];
      for (int k = 1; k < a.ksplit; ++k) {   // the K parts, in order
        gz += gu[k * a.split_stride + base];
        gv += gu[k * a.split_stride + base + 64];
      }
      const float z = gz * a.sg[f];
      const float u = gv * a.su[f];
      v = z / (1.f + expf(-z)) * u;
    }
    vrow[f] = v;
    ss += v * v;
    mx = fmaxf(mx, fabsf(v));
  }
  ss = warp_sum(ss);
  mx = warp_max(mx);
  if ((tid & 31) == 0) {
    red[tid >> 5] = ss;
    redm[tid >> 5] = mx;
  }
  __syncthreads();
  float tot = 0.f, amax = 0.f;
  for (int w = 0; w < kSwThreads / 32; ++w) {
    tot += red[w];
    amax = fmaxf(amax, redm[w]);
  }
  const float p = block_prescale(amax);
  if (tid == 0) a.act_post[r] = (1.f / sqrtf(tot + 1e-6f)) * (1.f / p);
  // the row's digits (4 per value, one prescale for the row: the GEMM's activation units)
  constexpr int kRows = 64, kDig = 4, kCode = 256 * 32, kUnit = kCode + 2 * 512;
  const int groups = F / 16, kblocks = (F + 63) / 64, ir = r % kRows;
  for (int g0 = 0; g0 < groups; g0 += kSwThreads / 4) {   // a quad per group; every lane takes part
    const int g = g0 + (tid >> 2), t = tid & 3;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (g < groups)
#pragma unroll
      for (int c = 0; c < 4; ++c) v[c] = vrow[16 * g + 4 * t + c];
    uint32_t code[kDig], sf[kDig];
    digitize16_quad_n<kDig>(v, code, sf, p);
    if (g < groups) {
      uint8_t* unit = a.act + (int64_t)(g >> 2) * kUnit;
      const int j = g & 3;
#pragma unroll
      for (int dd = 0; dd < kDig; ++dd) {
        const int n = kRows * dd + ir;
        *reinterpret_cast<uint16_t*>(unit + a_code_offset(n, 16 * j + 4 * t)) = (uint16_t)code[dd];
        if (t == 0) unit[kCode + (n >> 7) * 512 + sf_offset(n & 127, j)] = (uint8_t)sf[dd];
      }
    }
  }
  (void)kblocks;
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
  launch_with_pdl(embed_batch_kernel, dim3(kMaxRows, a.nseq), dim3(256), 0, a, s, a.pdl != 0);
}

void launch_qkv_prep(const QkvPrepArgs& a, cudaStream_t s) {
  XTG_REQUIRE(a.nseq >= 1 && a.nseq <= kMaxBatch && a.ksplit >= 1, "qkv_prep: 1..8 sequences");
  launch_with_pdl(qkv_prep_kernel, dim3(2 * a.heads + 2 * a.kv_heads, kMaxRows * a.nseq), dim3(128), 0, a, s,
                  a.pdl != 0);
}

void launch_swiglu_batch(const SwigluBatchArgs& a, cudaStream_t s) {
  XTG_REQUIRE(a.features % 64 == 0 && a.features * 4 <= 200 * 1024, "swiglu_batch: features a multiple of 64");
  static std::atomic<uint64_t> optin{0};
  const int smem = a.features * 4;
  if (smem > 48 * 1024) ensure_smem_optin((const void*)swiglu_batch_kernel, smem, optin);
  launch_with_pdl(swiglu_batch_kernel, dim3(64), dim3(kSwThreads), (size_t)smem, a, s, a.pdl != 0);
}

void launch_scale_argmax(const ScaleArgmaxArgs& a, cudaStream_t s) {
  launch_with_pdl(scale_argmax_kernel, dim3(kMaxRows * a.nseq), dim3(1024), 0, a, s, a.pdl != 0);
}

}  // namespace xtg
