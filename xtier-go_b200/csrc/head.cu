// The BF16 lm_head of a checkpoint (matmul_bf16, engine/src/kernels.cpp:140-155, then the logit scale of
// packs/dory/dory.cpp:566-576): logits[i][n] = (sum_j bf16(W[n][j]) x[i][j]) * logit_scale[n] for the step's rows,
// and per 128-row tile and row the argmax candidate the GEMV head also writes (ties to the lowest index).
//
// The head is 2 bytes per weight streamed once per step, so the kernel is an HBM stream. One CTA per SM walks 128-row
// tiles; a producer warp brings each tile's 64-input blocks (16 KB) into a ring of shared-memory stages by TMA
// (cp.async.bulk.tensor 2D, 128-byte swizzle, rows past the vocabulary read as zeros; no multicast), and 8 consumer
// warps of 16 rows take their A fragments with ldmatrix. Each row x_i (f32) is split into two bf16 parts,
// x = hi + lo with lo = bf16(x - hi), which carry ~16 bits of x's mantissa; both multiply the weights on mma.sync
// m16n8k16 with f32 accumulation (16 weight rows x 8 activation rows), their B fragments by ldmatrix from x's planes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kConsumers = 8;                        // warps of 16 weight rows: one 128-row tile
constexpr int kHeadThreads = (kConsumers + 1) * 32;  // + the producer warp
constexpr int kBoxK = 64;                            // inputs per TMA box (128 bytes of bf16)
constexpr int kBoxBytes = 128 * kBoxK * 2;           // 16 KB
constexpr int kSmemLimit = 232448;

struct HeadArgs {
  const float* x;           // [8][hidden]
  const int* m_dev;         // rows, or null: m
  int m;
  int vocab, hidden, tiles, stages;
  const float* logit_scale;
  float* logits;            // [8][vocab] or null
  ArgCand* cand;            // [tiles][8]
  int* err;
  int pdl;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// shared memory: x's two bf16 planes [8][hidden + 8] (rows 16 bytes apart beyond 2 hidden: the 8 rows an ldmatrix
// reads fall in different banks), then the stages (1024-byte aligned for the swizzle), the barriers, the candidates
__host__ __device__ inline size_t planes_bytes(int hidden) { return (size_t)2 * kMaxRows * (2 * hidden + 16); }
__host__ __device__ inline size_t stages_offset(int hidden) { return (planes_bytes(hidden) + 1023) / 1024 * 1024; }
// (+ 1 KB: the kernel aligns its base to 1024 bytes, the 128-byte swizzle's atom)
__host__ __device__ inline size_t smem_bytes(int hidden, int stages) {
  return 1024 + stages_offset(hidden) + (size_t)stages * kBoxBytes + 2 * 8 * (size_t)stages +
         sizeof(ArgCand) * kConsumers * kMaxRows;
}

__global__ void __launch_bounds__(kHeadThreads, 1) head_bf16_kernel(const __grid_constant__ CUtensorMap map,
                                                                   const HeadArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // 1024-byte aligned
  const int H = a.hidden, S = a.stages, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int xs = 2 * H + 16;   // bytes between x rows
  uint8_t* xhi = smem;
  uint8_t* xlo = smem + kMaxRows * xs;
  uint8_t* stage = smem + stages_offset(H);
  uint64_t* full = reinterpret_cast<uint64_t*>(stage + (size_t)S * kBoxBytes);
  uint64_t* empty = full + S;
  ArgCand* best_s = reinterpret_cast<ArgCand*>(empty + S);   // [warp][row]
  const int KB = H / kBoxK;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    mbar_init_fence();
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ---- producer: the weights do not depend on the previous kernel, so they stream from the start ----
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x)
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int slot = it % S;
          if (it >= S) mbar_wait_bounded(&empty[slot], (uint32_t)((it / S) - 1) & 1u, a.err);
          mbar_expect_tx(&full[slot], kBoxBytes);
          tma_load_2d(stage + (size_t)slot * kBoxBytes, &map, kb * kBoxK, tile * 128, &full[slot]);
        }
      // every issued copy has landed before the CTA may exit
      for (int slot = 0; slot < S && slot < it; ++slot) {
        const int last = slot + ((it - 1 - slot) / S) * S;
        mbar_wait_bounded(&full[slot], (uint32_t)(last / S) & 1u, a.err);
      }
    }
    __syncwarp();
    return;
  }

  // ---- consumers ----
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const int m = a.m_dev ? *a.m_dev : a.m;
  for (int idx = tid; idx < kMaxRows * H; idx += kConsumers * 32) {
    const int i = idx / H, k = idx - i * H;
    const float v = i < m ? a.x[(int64_t)i * H + k] : 0.f;
    const uint16_t hb = f32_to_bf16_bits(v);
    const uint16_t lb = f32_to_bf16_bits(v - bf16_bits_to_f32(hb));
    *reinterpret_cast<uint16_t*>(xhi + i * xs + 2 * k) = hb;
    *reinterpret_cast<uint16_t*>(xlo + i * xs + 2 * k) = lb;
  }
  consumers_sync();
  const int g = lane >> 2, t = lane & 3;
  // ldmatrix row addresses. A: matrix q = lane / 8 is rows 8 (q & 1) .. + 7 of this warp's 16, input chunk q >> 1 of
  // the k16 step (the stage's row r holds its 16-byte chunk c at c ^ (r & 7)). B: lanes 0-15 the hi plane, 16-31 the
  // lo plane; row lane & 7, chunk (lane >> 3) & 1.
  const int ar = 16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1), ac = lane >> 4;
  const uint32_t b_base = smem_u32((lane < 16 ? xhi : xlo) + (lane & 7) * xs + 16 * ((lane >> 3) & 1));
  int it = 0;
  for (int tile = blockIdx.x; tile < a.tiles; tile += gridDim.x) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kb = 0; kb < KB; ++kb, ++it) {
      const int slot = it % S;
      mbar_wait_bounded(&full[slot], (uint32_t)(it / S) & 1u, a.err);
      const uint32_t a_row = smem_u32(stage + (size_t)slot * kBoxBytes + ar * 128);
#pragma unroll
      for (int j = 0; j < kBoxK / 16; ++j) {
        uint32_t a0, a1, a2, a3, bh0, bh1, bl0, bl1;
        ldsm_x4(a_row + ((uint32_t)((2 * j + ac) ^ (ar & 7)) << 4), a0, a1, a2, a3);
        ldsm_x4(b_base + (uint32_t)(2 * (kb * kBoxK + 16 * j)), bh0, bh1, bl0, bl1);
        mma_bf16(acc, a0, a1, a2, a3, bh0, bh1);
        mma_bf16(acc, a0, a1, a2, a3, bl0, bl1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    // acc: (row r0, activation rows 2t, 2t + 1), (row r1, the same)
    const int r0 = tile * 128 + warp * 16 + g, r1 = r0 + 8;
    const bool ok0 = r0 < a.vocab, ok1 = r1 < a.vocab;
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
      best_s[warp * kMaxRows + n0] = ArgCand{bv[0], bi[0]};
      best_s[warp * kMaxRows + n1] = ArgCand{bv[1], bi[1]};
    }
    consumers_sync();
    if (tid < kMaxRows) {
      ArgCand b = best_s[tid];
      for (int w = 1; w < kConsumers; ++w) {
        const ArgCand c = best_s[w * kMaxRows + tid];
        if (better(c.v, c.i, b.v, b.i)) b = c;
      }
      a.cand[(int64_t)tile * kMaxRows + tid] = b;
    }
    consumers_sync();
  }
}

// the tensor map of a [vocab][hidden] bf16 weight: boxes of 64 inputs x 128 rows, 128-byte swizzle, zeros past the end
CUtensorMap weight_map(const uint16_t* w, int vocab, int hidden) {
  static std::mutex mu;
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!encode) {
      cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
      void* fn = nullptr;
      XTG_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
      XTG_REQUIRE(fn && q == cudaDriverEntryPointSuccess, "bf16 head: no cuTensorMapEncodeTiled in the driver");
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)hidden, (cuuint64_t)vocab};
  const cuuint64_t strides[1] = {(cuuint64_t)hidden * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBoxK, 128u};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(w), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  XTG_REQUIRE(r == CUDA_SUCCESS, "bf16 head: cuTensorMapEncodeTiled failed");
  return map;
}

}  // namespace

void launch_head_bf16(const HeadBf16Args& h, int num_sms, cudaStream_t s, bool pdl) {
  XTG_REQUIRE(h.hidden % kBoxK == 0 && h.hidden <= kMaxHeadBf16Hidden,
              "bf16 head: hidden a multiple of 64, at most 5120");
  XTG_REQUIRE(h.vocab > 0 && h.w && h.x && h.cand && h.logit_scale, "bf16 head: missing operand");
  XTG_REQUIRE(h.m_dev || (h.m >= 1 && h.m <= kMaxRows), "bf16 head: 1..8 rows");
  XTG_REQUIRE((reinterpret_cast<uintptr_t>(h.w) & 15) == 0, "bf16 head: the weight must start on a 16-byte boundary");
  HeadArgs a = {};
  a.x = h.x;
  a.m_dev = h.m_dev;
  a.m = h.m;
  a.vocab = h.vocab;
  a.hidden = h.hidden;
  a.tiles = (h.vocab + 127) / 128;
  a.logit_scale = h.logit_scale;
  a.logits = h.logits;
  a.cand = h.cand;
  a.err = h.err;
  a.pdl = pdl ? 1 : 0;
  int stages = 8;
  while (stages > 2 && smem_bytes(h.hidden, stages) > (size_t)kSmemLimit) --stages;
  a.stages = stages;
  const size_t smem = smem_bytes(h.hidden, stages);
  XTG_REQUIRE(smem <= (size_t)kSmemLimit, "bf16 head: x and two stages do not fit in shared memory");
  const CUtensorMap map = weight_map(h.w, h.vocab, h.hidden);
  static std::atomic<uint64_t> optin;
  ensure_smem_optin((const void*)head_bf16_kernel, kSmemLimit, optin);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min(a.tiles, num_sms));
  cfg.blockDim = dim3(kHeadThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, head_bf16_kernel, map, a));
}

}  // namespace xtg
