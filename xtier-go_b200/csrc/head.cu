// The BF16 lm_head of a checkpoint (matmul_bf16, engine/src/kernels.cpp:140-155, then the logit scale of
// packs/dory/dory.cpp:566-576): logits[i][n] = (sum_j bf16(W[n][j]) x[i][j]) * logit_scale[n] for the step's rows,
// and per 128-row tile and row the argmax candidate the GEMV head also writes (ties to the lowest index).
//
// The head is 2 bytes per weight streamed once per step, so the kernel is an HBM stream. Each row x_i (f32) is split
// into two bf16 parts, x = hi + lo with lo = bf16(x - hi), which carry ~16 bits of x's mantissa. Both parts multiply
// the weights on the mma.sync bf16 tensor path with f32 accumulation (m16n8k16: 16 weight rows x 8 activation rows).
// The dot product's order of inputs is free, so a lane loads 16 contiguous bytes (8 inputs) of a weight row and the
// same 8 inputs of its activation row: the first two 4-byte words feed one k16 step, the last two the next one.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kHeadThreads = 256;    // 8 warps, 16 weight rows each: one 128-row tile per CTA pass
constexpr int kHeadUnroll = 4;       // 32-input steps in flight per warp

struct HeadArgs {
  const float* x;           // [8][hidden]
  const int* m_dev;         // rows, or null: m
  int m;
  const uint16_t* w;        // [vocab][hidden]
  int vocab, hidden, tiles;
  const float* logit_scale;
  float* logits;            // [8][vocab] or null
  ArgCand* cand;            // [tiles][8]
  int pdl;
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__global__ void __launch_bounds__(kHeadThreads) head_bf16_kernel(const HeadArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ ArgCand best_s[kHeadThreads / 32][kMaxRows];
  const int H = a.hidden, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  // x as two bf16 planes [8][H] (hi, then lo), rows 64 bytes apart beyond H * 2 so that the 8 rows a quarter warp
  // reads fall in different banks
  const int stride = 2 * H + 64;
  uint8_t* xhi = smem;
  uint8_t* xlo = smem + kMaxRows * stride;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const int m = a.m_dev ? *a.m_dev : a.m;
  for (int idx = tid; idx < kMaxRows * H; idx += kHeadThreads) {
    const int i = idx / H, k = idx - i * H;
    const float v = i < m ? a.x[(int64_t)i * H + k] : 0.f;
    const uint16_t hb = f32_to_bf16_bits(v);
    const uint16_t lb = f32_to_bf16_bits(v - bf16_bits_to_f32(hb));
    *reinterpret_cast<uint16_t*>(xhi + i * stride + 2 * k) = hb;
    *reinterpret_cast<uint16_t*>(xlo + i * stride + 2 * k) = lb;
  }
  __syncthreads();
  const int steps = H / 32;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    const int r0 = tile * 128 + warp * 16 + g, r1 = r0 + 8;
    const bool ok0 = r0 < a.vocab, ok1 = r1 < a.vocab;
    const uint16_t* w0 = a.w + (int64_t)(ok0 ? r0 : 0) * H + 8 * t;
    const uint16_t* w1 = a.w + (int64_t)(ok1 ? r1 : 0) * H + 8 * t;
    const uint8_t* bh = xhi + g * stride + 16 * t;
    const uint8_t* bl = xlo + g * stride + 16 * t;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < steps; s0 += kHeadUnroll) {
      uint4 A0[kHeadUnroll], A1[kHeadUnroll];
#pragma unroll
      for (int u = 0; u < kHeadUnroll; ++u) {
        const int s = s0 + u;
        A0[u] = (ok0 && s < steps) ? ld_stream(w0 + 32 * s) : make_uint4(0u, 0u, 0u, 0u);
        A1[u] = (ok1 && s < steps) ? ld_stream(w1 + 32 * s) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kHeadUnroll; ++u) {
        const int s = s0 + u;
        if (s < steps) {
          const uint4 h4 = *reinterpret_cast<const uint4*>(bh + 64 * s);
          const uint4 l4 = *reinterpret_cast<const uint4*>(bl + 64 * s);
          mma_bf16(acc, A0[u].x, A1[u].x, A0[u].y, A1[u].y, h4.x, h4.y);
          mma_bf16(acc, A0[u].z, A1[u].z, A0[u].w, A1[u].w, h4.z, h4.w);
          mma_bf16(acc, A0[u].x, A1[u].x, A0[u].y, A1[u].y, l4.x, l4.y);
          mma_bf16(acc, A0[u].z, A1[u].z, A0[u].w, A1[u].w, l4.z, l4.w);
        }
      }
    }
    // acc: (row r0, activation rows 2t, 2t + 1), (row r1, the same)
    const float ls0 = ok0 ? a.logit_scale[r0] : 0.f, ls1 = ok1 ? a.logit_scale[r1] : 0.f;
    float v[4] = {ok0 ? acc[0] * ls0 : -INFINITY, ok0 ? acc[1] * ls0 : -INFINITY, ok1 ? acc[2] * ls1 : -INFINITY,
                  ok1 ? acc[3] * ls1 : -INFINITY};
    const int n0 = 2 * t, n1 = 2 * t + 1;
    if (a.logits) {
      if (ok0 && n0 < m) a.logits[(int64_t)n0 * a.vocab + r0] = v[0];
      if (ok0 && n1 < m) a.logits[(int64_t)n1 * a.vocab + r0] = v[1];
      if (ok1 && n0 < m) a.logits[(int64_t)n0 * a.vocab + r1] = v[2];
      if (ok1 && n1 < m) a.logits[(int64_t)n1 * a.vocab + r1] = v[3];
    }
    // the warp's best row for each activation row: rows r0 < r1, then over the 8 lanes of a t (lane bits 2-4)
    float bv[2];
    int bi[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      bv[q] = v[q];
      bi[q] = r0;
      if (better(v[2 + q], r1, bv[q], bi[q])) {
        bv[q] = v[2 + q];
        bi[q] = r1;
      }
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv[q], o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi[q], o);
        if (better(ov, oi, bv[q], bi[q])) {
          bv[q] = ov;
          bi[q] = oi;
        }
      }
    }
    if (g == 0) {
      best_s[warp][n0] = ArgCand{bv[0], bi[0]};
      best_s[warp][n1] = ArgCand{bv[1], bi[1]};
    }
    __syncthreads();
    if (tid < kMaxRows) {
      ArgCand b = best_s[0][tid];
      for (int w = 1; w < kHeadThreads / 32; ++w) {
        const ArgCand c = best_s[w][tid];
        if (better(c.v, c.i, b.v, b.i)) b = c;
      }
      a.cand[(int64_t)tile * kMaxRows + tid] = b;
    }
    __syncthreads();
  }
}

}  // namespace

void launch_head_bf16(const HeadBf16Args& h, int num_sms, cudaStream_t s, bool pdl) {
  XTG_REQUIRE(h.hidden % 32 == 0 && h.hidden <= kMaxHeadBf16Hidden, "bf16 head: hidden a multiple of 32, at most 6144");
  XTG_REQUIRE(h.vocab > 0 && h.w && h.x && h.cand && h.logit_scale, "bf16 head: missing operand");
  XTG_REQUIRE(h.m_dev || (h.m >= 1 && h.m <= kMaxRows), "bf16 head: 1..8 rows");
  HeadArgs a = {};
  a.x = h.x;
  a.m_dev = h.m_dev;
  a.m = h.m;
  a.w = h.w;
  a.vocab = h.vocab;
  a.hidden = h.hidden;
  a.tiles = (h.vocab + 127) / 128;
  a.logit_scale = h.logit_scale;
  a.logits = h.logits;
  a.cand = h.cand;
  a.pdl = pdl ? 1 : 0;
  const int smem = 2 * kMaxRows * (2 * h.hidden + 64);
  static std::atomic<uint64_t> optin;
  ensure_smem_optin((const void*)head_bf16_kernel, 2 * kMaxRows * (2 * kMaxHeadBf16Hidden + 64), optin);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(a.tiles, 2 * num_sms));
  cfg.blockDim = dim3(kHeadThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, head_bf16_kernel, a));
}

}  // namespace xtg
