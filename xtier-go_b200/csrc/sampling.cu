// The candidates of the reference's sampler on the device (engine/src/sampler.cpp): for each logits row the k most
// likely entries, most likely first -- value descending, ties to the lowest index, the order of more_likely
// (sampler.cpp:26-28) that top_logprobs (30-40) and Sampler::sample's partial sorts (55-70) use -- with the row's max
// and total = sum_i exp((l_i - max) / T) (the normaliser of sample, 45-52, and of top_logprobs' log-sum-exp at T = 1).
// A caller then draws from k candidates instead of reading the whole 131,072-entry row back.
//
// One cluster of 8 CTAs per row, 1024 threads each, 16 consecutive entries per thread held in registers as order-
// preserving 32-bit keys. An exact radix select finds the k-th largest key in three digit passes (11, 11, 10 bits):
// each CTA counts its entries in shared memory, every CTA sums the 8 histograms over distributed shared memory and
// picks the same digit. The entries above the threshold and the first ones equal to it (in index order) go to the
// leader CTA, which sorts them (bitonic, 64-bit composite keys) and writes them out.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "../../include/xtg_cuda.h"
#include "common.cuh"
#include "sampling.h"

namespace cg = cooperative_groups;

namespace xtg {
namespace {

constexpr int kTkCtas = 8;
constexpr int kTkThreads = 1024;
constexpr int kTkPer = 16;   // entries per thread: 8 x 1024 x 16 = 131,072 per row at most

// float -> key with the same order (larger value, larger key); -0 and +0 compare equal as floats do (more_likely
// breaks their tie by index), so both get +0's key. NaN is not expected in logits.
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Exclusive prefix sum over the block of one value per thread (1024 threads); also returns the block's total.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_tot, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t t = warp_tot[lane], s = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_tot[lane] = s - t;   // exclusive offsets of the warps
    if (lane == 31) warp_tot[32] = s;
  }
  __syncthreads();
  total = warp_tot[32];
  const uint32_t r = warp_tot[warp] + x - v;
  __syncthreads();   // warp_tot is reused by the next scan
  return r;
}

__global__ void __cluster_dims__(kTkCtas, 1, 1) __launch_bounds__(kTkThreads, 1)
    topk_kernel(const float* __restrict__ logits, int vocab, int k, float inv_t, int vec4, int32_t* out_idx,
                float* out_val, float* out_max, double* out_total) {
  cg::cluster_group cl = cg::this_cluster();
  const int crank = (int)cl.block_rank();
  const int row = blockIdx.y;
  __shared__ uint32_t hist[2][2048];       // this CTA's digit counts, alternating by pass
  __shared__ uint32_t scan_tmp[33];
  __shared__ uint32_t pick[2];             // the chosen digit, the count of entries above its bin
  __shared__ float cta_max;
  __shared__ double cta_sum;
  __shared__ uint32_t cta_cnt[2];          // this CTA's entries above / at the threshold
  __shared__ unsigned long long cand[1024];   // leader: the candidates, (key << 32) | (0xffffffff - index)
  __shared__ float wmax[32];
  __shared__ double wsum[32];

  // ---- this thread's 16 entries ----
  const int e0 = (crank * kTkThreads + (int)threadIdx.x) * kTkPer;
  const float* src = logits + (int64_t)row * vocab;
  uint32_t key[kTkPer];
  float mx = -INFINITY;
  if (vec4 && e0 + kTkPer <= vocab) {   // vec4: 16-byte aligned rows
#pragma unroll
    for (int q = 0; q < kTkPer / 4; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(src + e0 + 4 * q);
      key[4 * q] = order_key(v.x);
      key[4 * q + 1] = order_key(v.y);
      key[4 * q + 2] = order_key(v.z);
      key[4 * q + 3] = order_key(v.w);
      mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
  } else {
#pragma unroll
    for (int e = 0; e < kTkPer; ++e) {
      const float v = e0 + e < vocab ? src[e0 + e] : -INFINITY;
      key[e] = order_key(v);
      mx = fmaxf(mx, v);
    }
  }
  const int nvalid = max(0, min(kTkPer, vocab - e0));   // entries past the row take part in nothing
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = mx;

  // ---- radix select of the k-th largest key: digits [31:21], [20:10], [9:0] ----
  uint32_t prefix = 0, pmask = 0;
  uint32_t krem = (uint32_t)k;
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const int nb = pass == 2 ? 1024 : 2048;
    uint32_t* h = hist[pass & 1];
    h[threadIdx.x] = 0;
    h[threadIdx.x + 1024] = 0;
    __syncthreads();
#pragma unroll
    for (int e = 0; e < kTkPer; ++e)
      if (e < nvalid && (key[e] & pmask) == prefix) atomicAdd(&h[(key[e] >> shift) & (nb - 1)], 1u);
    if (pass == 0 && threadIdx.x < 32) {
      float m = wmax[threadIdx.x];
      m = warp_max(m);
      if (threadIdx.x == 0) cta_max = m;
    }
    cl.sync();   // every CTA's counts (and, in pass 0, its max) are complete
    // every CTA sums the 8 histograms itself: thread t takes bins nb-1-2t and nb-2-2t (descending order)
    uint32_t c0 = 0, c1 = 0;
    const int b0 = nb - 1 - 2 * (int)threadIdx.x, b1 = b0 - 1;
    if (b1 >= 0) {
#pragma unroll
      for (int r = 0; r < kTkCtas; ++r) {
        const uint32_t* hr = cl.map_shared_rank(h, r);
        c0 += hr[b0];
        c1 += hr[b1];
      }
    }
    uint32_t tot;
    const uint32_t ex = block_exclusive_scan(c0 + c1, scan_tmp, tot);
    if (b1 >= 0) {
      if (ex < krem && ex + c0 >= krem) {
        pick[0] = (uint32_t)b0;
        pick[1] = ex;
      } else if (ex + c0 < krem && ex + c0 + c1 >= krem) {
        pick[0] = (uint32_t)b1;
        pick[1] = ex + c0;
      }
    }
    __syncthreads();
    prefix |= pick[0] << shift;
    pmask |= (uint32_t)(nb - 1) << shift;
    krem -= pick[1];
    __syncthreads();   // pick is rewritten by the next pass
  }
  // prefix is now the k-th largest key; krem entries equal to it are taken, lowest index first

  // ---- the row max and the total, exp((l - max) / T) summed in double ----
  float rmax = -INFINITY;
#pragma unroll
  for (int r = 0; r < kTkCtas; ++r) rmax = fmaxf(rmax, *cl.map_shared_rank(&cta_max, r));
  double s = 0.0;
#pragma unroll
  for (int e = 0; e < kTkPer; ++e)
    if (e < nvalid) s += (double)expf((key_value(key[e]) - rmax) * inv_t);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = s;

  // ---- positions of the candidates, in index order (CTA, thread, entry) ----
  uint32_t ngt = 0, neq = 0;
#pragma unroll
  for (int e = 0; e < kTkPer; ++e) {
    ngt += e < nvalid && key[e] > prefix;
    neq += e < nvalid && key[e] == prefix;
  }
  uint32_t tgt, teq;
  const uint32_t xgt = block_exclusive_scan(ngt, scan_tmp, tgt);
  const uint32_t xeq = block_exclusive_scan(neq, scan_tmp, teq);
  if (threadIdx.x == 0) {
    cta_cnt[0] = tgt;
    cta_cnt[1] = teq;
    double t = 0.0;
    for (int w = 0; w < kTkThreads / 32; ++w) t += wsum[w];
    cta_sum = t;
  }
  if (crank == 0)   // the leader pads the sort to a power of two with keys below every candidate
    for (int i = k + (int)threadIdx.x; i < 1024; i += kTkThreads) cand[i] = 0ull;
  cl.sync();
  if (crank == 0 && threadIdx.x == 0) {   // every CTA's sum is in: the leader writes the row's max and total
    double t = 0.0;
    for (int r = 0; r < kTkCtas; ++r) t += *cl.map_shared_rank(&cta_sum, r);
    out_total[row] = t;
    out_max[row] = rmax;
  }
  uint32_t gt_base = 0, eq_base = 0, gt_all = 0;
#pragma unroll
  for (int r = 0; r < kTkCtas; ++r) {
    const uint32_t* cr = cl.map_shared_rank(cta_cnt, r);
    if (r < crank) {
      gt_base += cr[0];
      eq_base += cr[1];
    }
    gt_all += cr[0];
  }
  unsigned long long* lead = cl.map_shared_rank(cand, 0);
  uint32_t pg = gt_base + xgt, pe = eq_base + xeq;
#pragma unroll
  for (int e = 0; e < kTkPer; ++e) {
    if (e >= nvalid) continue;
    const unsigned long long ck =
        ((unsigned long long)key[e] << 32) | (unsigned long long)(0xffffffffu - (uint32_t)(e0 + e));
    if (key[e] > prefix) {
      lead[pg++] = ck;
    } else if (key[e] == prefix) {
      if (pe < krem) lead[gt_all + pe] = ck;
      ++pe;
    }
  }
  cl.sync();   // the leader holds all k candidates; every CTA is done with the others' shared memory
  if (crank != 0) return;
  // ---- bitonic sort of the first P composite keys (P: the power of two at or above k), descending ----
  int P = 2;
  while (P < k) P <<= 1;
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = (int)threadIdx.x, j = i ^ stride;
      if (j > i && j < P) {
        const unsigned long long a = cand[i], b = cand[j];
        const bool desc = (i & size) == 0;
        if (desc ? a < b : a > b) {
          cand[i] = b;
          cand[j] = a;
        }
      }
      __syncthreads();
    }
  }
  if ((int)threadIdx.x < k) {
    const unsigned long long c = cand[threadIdx.x];
    const int32_t i = (int32_t)(0xffffffffu - (uint32_t)(c & 0xffffffffull));
    out_idx[(int64_t)row * k + threadIdx.x] = i;
    out_val[(int64_t)row * k + threadIdx.x] = src[i];   // the logit as given (a -0 keeps its sign)
  }
}

}  // namespace

void launch_topk(const float* logits, int rows, int vocab, int k, float temperature, int32_t* idx, float* val,
                 float* row_max, double* total, cudaStream_t s) {
  XTG_REQUIRE(rows >= 1, "topk: at least one row");
  XTG_REQUIRE(vocab >= 1 && vocab <= kTkCtas * kTkThreads * kTkPer, "topk: 1..131072 entries per row");
  XTG_REQUIRE(k >= 1 && k <= kMaxTopK && k <= vocab, "topk: k in 1..min(1024, vocab)");
  const float inv_t = temperature > 0.f ? 1.f / temperature : 1.f;
  // 16-byte loads only where every row starts on a 16-byte boundary (a caller's pointer may sit anywhere)
  const int vec4 = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (vocab & 3) == 0;
  topk_kernel<<<dim3(kTkCtas, rows), kTkThreads, 0, s>>>(logits, vocab, k, inv_t, vec4, idx, val, row_max, total);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg

// Sampler::sample (sampler.cpp:41-94) from the k most likely entries of a row. The reference orders its candidates
// by weight exp((l - max) / T) and index; these come ordered by logit and index, which is the same order except among
// distinct logits whose weights round to the same float (the draw's cumulative sums there are equal either way).
extern "C" int xtg_cuda_sample_candidates(const int32_t* idx, const float* logit, int k, float row_max, double total,
                                          int vocab, const xtg_cuda_sampling* p, double u) {
  constexpr int kUndecided = -2;
  if (!idx || !logit || !p || k < 1 || vocab < 1 || k > vocab || !(u >= 0.0 && u < 1.0)) return -1;
  if (p->temperature <= 0.f) return idx[0];   // argmax: the first index of the maximum
  const float inv_t = 1.f / p->temperature;
  std::vector<float> w((size_t)k);
  for (int i = 0; i < k; ++i) w[(size_t)i] = std::exp((logit[i] - row_max) * inv_t);
  size_t keep = (size_t)vocab;
  double tot = total;
  if (p->top_k > 0 && p->top_k < vocab) {
    if (p->top_k > k) return kUndecided;
    keep = (size_t)p->top_k;
    tot = 0.0;
    for (size_t i = 0; i < keep; ++i) tot += w[i];
  } else if (p->top_p < 1.f || p->min_p > 0.f) {
    const size_t head = std::min<size_t>((size_t)vocab, 1024);
    if ((size_t)k < head) return kUndecided;
    double cum = 0.0;
    for (size_t i = 0; i < head; ++i) cum += w[i];
    if (head < (size_t)vocab && p->top_p < 1.f && cum < total * (double)p->top_p) return kUndecided;
  } else {
    return kUndecided;   // no filter: the reference draws over the whole row in index order
  }
  if (p->min_p > 0.f) {
    const float floor = p->min_p * w[0];
    size_t n = 0;
    double t = 0.0;
    while (n < keep && w[n] >= floor) {
      t += w[n++];
      if (n == (size_t)k && n < keep) return kUndecided;
    }
    keep = std::max<size_t>(1, n);
    tot = n ? t : (double)w[0];
  }
  if (p->top_p < 1.f) {
    const double target = tot * (double)p->top_p;
    double cum = 0.0;
    size_t n = 0;
    while (n < keep) {
      if (n == (size_t)k) return kUndecided;
      cum += w[n];
      ++n;
      if (cum >= target) break;
    }
    keep = std::max<size_t>(1, n);
    tot = cum;
  }
  const double r = u * tot;
  double cum = 0.0;
  for (size_t i = 0; i < keep; ++i) {
    if (i == (size_t)k) return kUndecided;
    cum += w[i];
    if (r < cum) return idx[i];
  }
  return keep <= (size_t)k ? idx[keep - 1] : kUndecided;
}
