// K2: the NVFP4 x activation GEMM for prefill chunks and batched rows (matmul_nvfp4's m > 2 path,
// engine/src/kernels.cpp:84-138, at M = 9 .. 4096) on the block-scaled FP4 tensor cores of sm_100a.
//
// The weights are the GEMV's packed units (kernels.h): tile t, K block b = 128 rows x 64 inputs, the codes in the MMA's
// K-major A layout and the E4M3 block scales in the scale-factor atom, so they stream to the tensor core untouched.
// tcgen05.mma kind::mxf4nvf4 needs both operands as E2M1 with UE4M3 block scales, so the activations become the B
// operand as kGDigits scaled E2M1 digits (the GEMV's representation with fewer digits): per activation row one
// power-of-two prescale p (from the row's max |x|, so that every K block of the row shares it and the products add
// up in TMEM), per 16-input group and digit a UE4M3 scale. An activation unit (9216 bytes) holds 256 digit rows
// (digit d of activation row i of the tile is row 64 d + i) x 64 inputs in the weight unit's K-major layout, then
// the scale atoms of digit rows 0-127 and 128-255.
//
// One MMA is 128 weight rows x 256 digit rows (64 activation rows) x 64 inputs: N = 256 takes one MMA and three scale
// copies per 4 MB of FP4 products, which is what the single issuing thread can keep up with. A persistent CTA per SM
// walks the (weight tile, activation tile) pairs, activation tiles fastest, so that the CTAs working at one time
// share their weight tiles in L2; one thread streams stages of 4 K blocks (weight units, activation units) through a
// ring (bulk copies), one issues the scale copies and the MMAs, four warps drain the TMEM accumulator (read out digit
// by digit, released before the arithmetic and the stores): y = sum of the digit columns / p * global.
#include <algorithm>

#include "common.cuh"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

namespace {

constexpr int kGDigits = kGemmDigits;             // activation digits of the B operand (fp4mma.cuh)
constexpr int kGN = 256;                          // the MMA's N: digit rows
constexpr int kActRows = kGemmRows;               // activation rows per unit (64)
constexpr int kActCodeBytes = kGemmCodeBytes;     // 8192
constexpr int kActUnitBytes = kGemmUnitBytes;
static_assert(kGN == kActRows * kGDigits, "the activation unit's digit rows");
constexpr int kGUnits = 4;      // K blocks per ring stage: one bulk copy of weight units, one of activation units
constexpr int kGStageBytes = kGUnits * (kUnitBytes + kActUnitBytes);
constexpr int kGStages = 3;     // ring stages (166 KB: one CTA per SM, which owns the TMEM it allocates)
constexpr int kGThreads = 256;
constexpr int kGAccCols = kGN;                    // TMEM columns of the accumulator
constexpr int kGSfCols = 12;                      // per K block: the weight scales (4 columns), the activations' (8)
constexpr uint32_t kGTmemCols = 512;              // the accumulator + the ring's scale factors
constexpr uint32_t kIdescGemm = (1u << 7) | (1u << 10) | ((uint32_t)(kGN >> 3) << 17) | ((128u >> 4) << 24);
static_assert(kGAccCols + kGStages * kGUnits * kGSfCols <= (int)kGTmemCols, "TMEM columns");

struct GemmParams {
  const uint8_t* w;          // weight units [wtiles][kblocks]
  int wtiles, kblocks;
  const uint8_t* act;        // activation units [atiles][kblocks]
  const float* act_post;     // [atiles * 64] per row: 1 / its prescale, times an optional row scale
  int atiles, m;
  const TileOut* outs;       // [wtiles]
  // K split ksplit ways (few activation rows: more CTAs than weight tiles): part ks of a tile sums K blocks
  // [kblocks ks / ksplit, kblocks (ks + 1) / ksplit) and writes its own partial output, split_stride floats after
  // part ks - 1's (the reader sums the parts in order)
  int ksplit;
  int64_t split_stride;
  int pdl;                   // launched as a programmatic dependent (the weights of the first stages go out first)
  int* err;
};

__device__ __forceinline__ void tc_mma_gemm(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t tsfa, uint32_t tsfb,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(kIdescGemm), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

__global__ void __launch_bounds__(kGThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KB = P.kblocks, ntiles = P.wtiles * P.ksplit * P.atiles;
  const int my_tiles = (int)blockIdx.x < ntiles ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  uint8_t* ring = smem;   // stage s: kGUnits weight units at s * kGStageBytes, then kGUnits activation units
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kGStages * kGStageBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kGStages;
  uint64_t* accfull = bars + 2 * kGStages;        // [2] (phases alternate per tile)
  uint64_t* accempty = bars + 2 * kGStages + 2;   // [2]
  uint64_t* done = bars + 2 * kGStages + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kGStages + 6);

  if (warp == 2) tmem_alloc(tmem_slot, kGTmemCols);
  if (tid == 0) {
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kTileRows);
    }
    mbar_init(done, 1);
    mbar_init_fence();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // tile i of this CTA: weight tile wt, K part ks (K blocks [k0, k0 + nk)), activation tile at
  auto tile_of = [&](int i, int& wt, int& ks, int& at, int& k0, int& nk) {
    const int q = (int)blockIdx.x + i * (int)gridDim.x;
    const int vt = q / P.atiles;
    at = q - vt * P.atiles;
    wt = vt / P.ksplit;
    ks = vt - wt * P.ksplit;
    k0 = KB * ks / P.ksplit;
    nk = KB * (ks + 1) / P.ksplit - k0;
  };

  // a tile's K blocks go in stages of kGUnits (the last one may be short); stages never span tiles
  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      // As a dependent launch the first stages' weight units (which no kernel writes) go out before the wait, their
      // activation units after it.
      const int early = P.pdl ? kGStages : 0;
      if (P.pdl) {
        int v = 0;
        for (int i = 0; i < my_tiles && v < early; ++i) {
          int wt, ks, at, k0, nk;
          tile_of(i, wt, ks, at, k0, nk);
          const uint8_t* wsrc = P.w + ((int64_t)wt * KB + k0) * kUnitBytes;
          for (int kb0 = 0; kb0 < nk && v < early; kb0 += kGUnits, ++v) {
            const int cnt = min(kGUnits, nk - kb0);
            mbar_expect_tx(&full[v], (uint32_t)(cnt * (kUnitBytes + kActUnitBytes)));
            bulk_g2s(ring + v * kGStageBytes, wsrc + (int64_t)kb0 * kUnitBytes, (uint32_t)(cnt * kUnitBytes), &full[v]);
          }
        }
        pdl_wait();
        pdl_launch_next();
      }
      int u = 0;
      for (int i = 0; i < my_tiles; ++i) {
        int wt, ks, at, k0, nk;
        tile_of(i, wt, ks, at, k0, nk);
        const uint8_t* wsrc = P.w + ((int64_t)wt * KB + k0) * kUnitBytes;
        const uint8_t* asrc = P.act + ((int64_t)at * KB + k0) * kActUnitBytes;
        const int spt = (nk + kGUnits - 1) / kGUnits;
        for (int st = 0; st < spt; ++st, ++u) {
          const int slot = u % kGStages, kb0 = st * kGUnits, cnt = min(kGUnits, nk - kb0);
          if (u >= kGStages) mbar_wait_bounded(&empty[slot], (uint32_t)((u / kGStages) - 1) & 1u, P.err);
          uint8_t* dst = ring + slot * kGStageBytes;
          if (u >= early) {
            mbar_expect_tx(&full[slot], (uint32_t)(cnt * (kUnitBytes + kActUnitBytes)));
            bulk_g2s(dst, wsrc + (int64_t)kb0 * kUnitBytes, (uint32_t)(cnt * kUnitBytes), &full[slot]);
          }
          bulk_g2s(dst + kGUnits * kUnitBytes, asrc + (int64_t)kb0 * kActUnitBytes, (uint32_t)(cnt * kActUnitBytes),
                   &full[slot]);
        }
      }
      // every copy has landed before the CTA may exit (normally long since)
      for (int v = std::max(0, u - kGStages); v < u; ++v)
        mbar_wait_bounded(&full[v % kGStages], (uint32_t)(v / kGStages) & 1u, P.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: per K block the two scale atoms to TMEM, then one MMA; a full stage is straight-line code ----
    if (lane == 0) {
      tc_fence_after();
      const uint32_t ring_addr = smem_u32(ring);
      const uint32_t sf0 = tbase + kGAccCols;   // stage s, unit j: SFA at sf0 + 12 (kGUnits s + j), SFB at + 4, + 8
      int u = 0;
      for (int i = 0; i < my_tiles; ++i) {
        const int acc = i & 1;
        const uint32_t tacc = tbase;
        if (i >= 1) {   // the epilogue has read the previous tile's accumulator out
          mbar_wait_bounded(&accempty[acc ^ 1], (uint32_t)((i - 1) >> 1) & 1u, P.err);
          tc_fence_after();
        }
        int wt, ks, at, k0, nk;
        tile_of(i, wt, ks, at, k0, nk);
        const int spt = (nk + kGUnits - 1) / kGUnits;
        for (int st = 0; st < spt; ++st, ++u) {
          const int slot = u % kGStages, kb0 = st * kGUnits, cnt = min(kGUnits, nk - kb0);
          mbar_wait_bounded(&full[slot], (uint32_t)(u / kGStages) & 1u, P.err);
          tc_fence_after();
          const uint32_t a0 = ring_addr + (uint32_t)(slot * kGStageBytes), b0 = a0 + kGUnits * kUnitBytes;
          const uint32_t sfs = sf0 + kGSfCols * kGUnits * (uint32_t)slot;
          auto unit = [&](int j) {
            const uint32_t au = a0 + (uint32_t)(j * kUnitBytes), bu = b0 + (uint32_t)(j * kActUnitBytes);
            const uint32_t sfa = sfs + kGSfCols * (uint32_t)j;
            tc_cp_sf(sfa, sf_desc(au + kUnitCodeBytes));
            tc_cp_sf(sfa + 4, sf_desc(bu + kActCodeBytes));
            tc_cp_sf(sfa + 8, sf_desc(bu + kActCodeBytes + 512));
            tc_mma_gemm(tacc, a_desc(au), a_desc(bu), sfa, sfa + 4, (kb0 + j) > 0 ? 1u : 0u);
          };
          if (cnt == kGUnits) {
#pragma unroll
            for (int j = 0; j < kGUnits; ++j) unit(j);
          } else {
            for (int j = 0; j < cnt; ++j) unit(j);
          }
          tc_commit(&empty[slot]);
        }
        tc_commit(&accfull[acc]);
      }
      tc_commit(done);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ---- epilogue: TMEM lane quarter q = warp - 4 holds weight rows 32 q .. 32 q + 31 ----
    const int q = warp - 4, r = 32 * q + lane;
    if (P.pdl) pdl_wait();   // the rows' factors come from the kernel before
    for (int i = 0; i < my_tiles; ++i) {
      int wt, ks, at, k0, nk;
      tile_of(i, wt, ks, at, k0, nk);
      const int acc = i & 1;
      TileOut o = P.outs[wt];
      o.y += (int64_t)ks * P.split_stride;
      mbar_wait_bounded(&accfull[acc], (uint32_t)(i >> 1) & 1u, lane == 0 ? P.err : nullptr);
      tc_fence_after();
      float y[kActRows];
      const uint32_t taddr = tbase + ((uint32_t)(32 * q) << 16);
#pragma unroll
      for (int d = 0; d < kGDigits; ++d) {   // a digit's 64 columns in four loads and one wait
        float v[kActRows];
#pragma unroll
        for (int c = 0; c < kActRows; c += 16)
          tmem_ld16(taddr + (uint32_t)(kActRows * d + c), *reinterpret_cast<float(*)[16]>(&v[c]));
        tmem_ld_wait();
#pragma unroll
        for (int ii = 0; ii < kActRows; ++ii) y[ii] = d == 0 ? v[ii] : y[ii] + v[ii];
      }
      tc_fence_before();
      mbar_arrive(&accempty[acc]);   // the next tile's products may start
      const float g = r < 64 ? o.global_lo : o.global_hi;
      if (r < o.rows)
#pragma unroll
        for (int ii = 0; ii < kActRows; ++ii) {
          const int row = at * kActRows + ii;
          if (row < P.m) o.y[(int64_t)row * o.ld + r] = y[ii] * P.act_post[row] * g;
        }
    }
  }
  // ---- teardown: every tcgen05 operation has completed before the columns go back ----
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    if (lane == 0) mbar_wait_bounded(done, 0, P.err);
    __syncwarp();
    tmem_dealloc(tbase, kGTmemCols);
  }
}

// One CTA per activation row (grid: every row of the activation tiles; rows past m get zero digits): the row's max
// |x| gives its prescale, then the quads of threads digitize its 16-input groups.
// Optional row scale (a justnorm of x applied to the product): 1 / sqrt(sum_p sumsq[p * ld + row] + 1e-6), the parts
// summed in order. act_post[row] = row scale / the prescale (a power of two: exact).
__global__ void __launch_bounds__(256) act_digitize_kernel(const float* x, int m, int k, int kblocks, uint8_t* act,
                                                          float* act_post, const float* sumsq, int nparts, int ld,
                                                          int pdl) {
  __shared__ float red[8];
  const int row = blockIdx.x, tid = threadIdx.x;
  if (pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = row < m;
  const float* xr = x + (int64_t)row * k;
  float mx = 0.f;
  if (live)
    for (int c = tid * 4; c < k; c += 256 * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xr + c);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
  const float p = block_prescale(mx);
  if (tid == 0) {
    float rs = 1.f;
    if (sumsq && live) {
      float t = 0.f;
      for (int q = 0; q < nparts; ++q) t += sumsq[(int64_t)q * ld + row];
      rs = 1.f / sqrtf(t + 1e-6f);
    }
    act_post[row] = rs * (1.f / p);
  }
  const int groups = k / 16, i = row % kActRows;
  uint8_t* units = act + (int64_t)(row / kActRows) * kblocks * kActUnitBytes;
  for (int g0 = 0; g0 < groups; g0 += 64) {   // 64 groups per pass, a quad each; every lane takes part
    const int g = g0 + (tid >> 2), t = tid & 3;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (live && g < groups) {
      const float4 x4 = *reinterpret_cast<const float4*>(xr + 16 * g + 4 * t);
      v[0] = x4.x; v[1] = x4.y; v[2] = x4.z; v[3] = x4.w;
    }
    uint32_t code[kGDigits], sf[kGDigits];
    digitize16_quad_n<kGDigits>(v, code, sf, p);
    if (g < groups) store_gemm_digits_quad(units, i, g, t, code, sf);
  }
}

}  // namespace

int gemm_padded_rows(int m) { return ((m + kActRows - 1) / kActRows) * kActRows; }

int64_t gemm_act_bytes(int m, int k) {
  return (int64_t)((m + kActRows - 1) / kActRows) * packed_kblocks(k) * kActUnitBytes;
}

void gemm_digitize(const float* x, int m, int k, uint8_t* act, float* act_post, cudaStream_t s, const float* sumsq,
                   int nparts, int ld, bool pdl) {
  XTG_REQUIRE(m >= 1 && k % 16 == 0, "gemm: m >= 1 rows, k a multiple of 16");
  const int atiles = (m + kActRows - 1) / kActRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(atiles * kActRows);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, act_digitize_kernel, x, m, k, packed_kblocks(k), act, act_post, sumsq, nparts, ld,
                              pdl ? 1 : 0));
}

void launch_gemm(const uint8_t* w, int wtiles, int kblocks, const uint8_t* act, const float* act_post, int m,
                 const TileOut* outs, int num_sms, int* err, cudaStream_t s, int ksplit, int64_t split_stride,
                 bool pdl) {
  XTG_REQUIRE(m >= 1 && wtiles >= 1 && kblocks >= 1, "gemm: empty problem");
  XTG_REQUIRE(ksplit >= 1 && ksplit <= kblocks, "gemm: 1..kblocks K parts");
  GemmParams P = {};
  P.w = w;
  P.wtiles = wtiles;
  P.kblocks = kblocks;
  P.act = act;
  P.act_post = act_post;
  P.atiles = (m + kActRows - 1) / kActRows;
  P.m = m;
  P.outs = outs;
  P.ksplit = ksplit;
  P.split_stride = split_stride;
  P.pdl = pdl ? 1 : 0;
  P.err = err;
  const size_t smem = (size_t)kGStages * kGStageBytes + (2 * kGStages + 8) * 8;
  static std::atomic<uint64_t> optin{0};
  ensure_smem_optin((const void*)gemm_kernel, (int)smem, optin);
  const int ntiles = wtiles * ksplit * P.atiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(ntiles, num_sms));
  cfg.blockDim = dim3(kGThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, gemm_kernel, P));
}

}  // namespace xtg
