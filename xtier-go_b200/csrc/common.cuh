// Shared device helpers of libxtg_cuda: number formats, the seeded generators, programmatic-dependent-launch hooks,
// warp reductions. sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <stdexcept>
#include <string>

namespace xtg {

// ---- host error handling: an exception inside the library, a -1 + message at the C ABI ----
struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

#define XTG_CUDA(call)                                                                                   \
  do {                                                                                                   \
    cudaError_t e_ = (call);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      throw ::xtg::CudaError(std::string(#call) + ": " + cudaGetErrorString(e_) + " (" __FILE__ ":" +  \
                             std::to_string(__LINE__) + ")");                                            \
  } while (0)

#define XTG_REQUIRE(cond, msg)                       \
  do {                                               \
    if (!(cond)) throw ::xtg::CudaError(std::string(msg)); \
  } while (0)

// The opt-in to more than 48 KB of dynamic shared memory: cudaFuncSetAttribute applies to the current device only,
// so each kernel keeps the set of devices (ordinals below 64) that already have it. Thread-safe: threads that race
// both set the attribute, which is harmless; a device at 64 or above sets it on every launch.
inline void ensure_smem_optin(const void* func, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  XTG_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return;
  XTG_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
}

// ---- programmatic dependent launch: a kernel waits for its predecessor's results only where it reads them ----
// Every kernel of the step lets its dependent launch only once its own wait is over: the next kernel's CTAs then
// prefetch (weights, cache chunks) while this one runs, but no kernel two or more ahead floods the memory system
// with prefetches while this one's dependent loads are on the critical path (measured: 2.76 -> 2.70 ms per step).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Prefetch [p, p + bytes) into L2 (no shared memory, no completion to wait for). p and bytes 16-byte aligned.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- mbarriers and bulk copies (global -> shared, no multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// global -> shared bulk copy completing on `bar` (16-byte aligned addresses, a multiple of 16 bytes)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// An L2 policy for data read once per step (weights, the global KV caches): its lines are the first evicted, so the
// stream does not push the kernels' code, the activations and the ring caches out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

constexpr uint32_t kMaxSpins = 1u << 24;   // bound on every mbarrier wait

// Wait for phase `parity` of an mbarrier; after kMaxSpins polls give up, set *err (if given) and return false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins > kMaxSpins) {
      if (err) atomicExch(err, 1);
      return false;
    }
  }
  return true;
}

// ---- words between GPUs (another process's memory, mapped over NVLink) ----
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// A value and a sequence number in one 64-bit word: an aligned 64-bit store is seen whole or not at all, so the
// reader knows the value is this round's once the number matches.
__device__ __forceinline__ void put_seq_word(uint64_t* p, float v, uint32_t seq) {
  const uint64_t w = ((uint64_t)seq << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

// The value of *p once its number is seq. After wait_ns, or at once when *err is set (another wait of this step
// gave up), set *err and return 0: a process that stopped stepping costs one timeout per step, not one per wait.
__device__ __forceinline__ float take_seq_word(const uint64_t* p, uint32_t seq, uint64_t wait_ns, int* err) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  if ((uint32_t)(w >> 32) != seq) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      __nanosleep(32);
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
      if ((uint32_t)(w >> 32) == seq) break;
      if ((it & 63) == 0 && (*reinterpret_cast<volatile int*>(err) != 0 || globaltimer_ns() - t0 > wait_ns)) {
        atomicExch(err, 2);
        return 0.f;
      }
    }
  }
  return __uint_as_float((uint32_t)w);
}

// A named barrier over `threads` threads (a multiple of 32) of the CTA; barrier 0 is __syncthreads'.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- number formats ----
// E4M3 decode (bias 7, subnormal steps of 2^-9, 0x7f NaN), FP32 exact.
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  const int e = (b >> 3) & 15, m = b & 7;
  float mag;
  if ((b & 0x7f) == 0x7f)
    mag = __int_as_float(0x7fc00000);
  else if (e == 0)
    mag = __int2float_rn(m) * 0.001953125f;   // 2^-9
  else
    mag = __int2float_rn(8 + m) * __int_as_float((e - 10 + 127) << 23);
  return (b & 0x80) ? -mag : mag;
}

// FP32 -> E4M3, round to nearest even, saturating to 448 (the rule of the reference's f32_to_e4m3 / e4m3_bits).
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint8_t sign = (u >> 24) & 0x80;
  const uint32_t a = u & 0x7fffffffu;
  if (a > 0x7f800000u) return sign | 0x7f;
  if (a >= 0x43e00000u) return sign | 0x7e;            // >= 448 (and infinity)
  if (a < 0x3c800000u) {                                // below 2^-6: multiples of 2^-9
    const float t = __fmul_rn(__uint_as_float(a), 512.f);
    return sign | (uint8_t)__float2int_rn(t);
  }
  const int e = (int)(a >> 23) - 127;                   // -6 .. 8
  const float t = __fmul_rn(__uint_as_float(a), __int_as_float((127 + 3 - e) << 23));   // [8, 16)
  int mant = __float2int_rn(t);
  int exp = e + 7;
  if (mant == 16) {
    mant = 8;
    ++exp;
  }
  int code = (exp << 3) | (mant - 8);
  return sign | (uint8_t)(code > 0x7e ? 0x7e : code);
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ float e2m1_to_f32(uint32_t nib) {
  const uint32_t m = nib & 7;
  // 0, 0.5, 1, 1.5, 2, 3, 4, 6
  const float v = m < 4 ? 0.5f * (float)m : (float)(2u << ((m - 4) >> 1)) * ((m & 1) ? 1.5f : 1.f);
  return (nib & 8) ? -v : v;
}

// Nearest E2M1 code, ties to the even code, saturating to 6 (the quantizer's rounding).
__device__ __forceinline__ uint8_t e2m1_code(float q) {
  const float a = fabsf(q);
  int c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) + (a >= 3.5f) + (a > 5.f);
  if (q < 0.f) c |= 8;
  return (uint8_t)c;
}

// Two E2M1 codes of a byte -> f16x2 (low nibble in the low half); exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
  uint32_t r;
  asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(r) : "r"(byte));
  return r;
}

// Two floats -> a byte of two E2M1 codes (lo in the low nibble), nearest, saturating to +-6.
__device__ __forceinline__ uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{ .reg .b8 t; cvt.rn.satfinite.e2m1x2.f32 t, %2, %1; cvt.u32.u8 %0, t; }" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

// Two E4M3 bytes (low, high of a 16-bit value) -> f16x2; exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t r;
  const uint16_t h = (uint16_t)two;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(h));
  return r;
}

// Two signed bytes (low, high of a 16-bit value in bits 0-15 of w) -> f16x2, exact: 1024 + 128 + b as a half, less
// 1152.
__device__ __forceinline__ uint32_t s8x2_to_f16x2(uint32_t biased_word, uint32_t sel) {
  uint32_t r = __byte_perm(biased_word, 0x64646464u, sel);
  const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&r), __halves2half2(__ushort_as_half(0x6480),
                                                                                   __ushort_as_half(0x6480)));
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulation.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x on the special-function unit (ex2.approx, flush-to-zero; a few ulp): 2^-inf = 0
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// D = A(16x32, row) * B(32x8, col) + D, signed 8-bit inputs, exact 32-bit integer accumulation.
__device__ __forceinline__ void mma_s8(int (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// ---- seeded generators, bit-identical to the oracle's xo_rand_bits / xo_gen_* ----
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

__host__ __device__ __forceinline__ uint64_t rand_key(uint64_t seed, uint64_t stream) {
  return mix64(seed + 0x9e3779b97f4a7c15ull * (stream + 1));
}

__host__ __device__ __forceinline__ uint64_t rand_bits(uint64_t key, uint64_t index) {
  return mix64(key + 0x9e3779b97f4a7c15ull * (index + 1));
}

__device__ __forceinline__ float normal_from_bits(uint64_t b) {
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) s = __fadd_rn(s, __fadd_rn((float)((b >> (16 * j)) & 0xffff), 0.5f));
  const float c = __fsub_rn(__fmul_rn(s, 1.f / 65536.f), 2.f);
  return __fmul_rn(c, 1.7320508f);
}

__device__ __forceinline__ float uniform_from_bits(uint64_t b, float lo, float span) {
  const float u = __fmul_rn((float)(b >> 40), 0x1p-24f);
  return __fadd_rn(lo, __fmul_rn(span, u));
}

// ---- reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sums of 8 values over the warp, each total returned in every lane: a transposing reduction (halves of the set
// exchanged at lane offsets 16, 8, 4 -- lane l then holds value (l >> 2) & 7 over 8 lanes --, a butterfly over the
// last 4 lanes, then a broadcast from lane 4 j): 17 shuffles where 8 butterflies take 40.
__device__ __forceinline__ void warp_sum8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float a4[4], a2[2];
#pragma unroll
  for (int k = 0; k < 4; ++k)   // value k + 4 b4
    a4[k] = (b4 ? v[k + 4] : v[k]) + __shfl_xor_sync(0xffffffffu, b4 ? v[k] : v[k + 4], 16);
#pragma unroll
  for (int k = 0; k < 2; ++k)   // value k + 2 b3 + 4 b4
    a2[k] = (b3 ? a4[k + 2] : a4[k]) + __shfl_xor_sync(0xffffffffu, b3 ? a4[k] : a4[k + 2], 8);
  float a1 = (b2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? a2[0] : a2[1], 4);   // value (lane >> 2) & 7
  a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
  a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __shfl_sync(0xffffffffu, a1, 4 * j);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum in a fixed order (deterministic), every thread gets the result. red: >= 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}


constexpr int kMaxRows = 8;   // activation rows of a verify step (mma N = 8)

}  // namespace xtg
