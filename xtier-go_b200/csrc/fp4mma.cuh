// The block-scaled FP4 tensor-core path of sm_100a: tcgen05.mma kind::mxf4nvf4 with the E4M3 scale of every 16
// inputs applied by the tensor core, the shared-memory operand layouts it reads, the TMEM helpers, and the
// activation "digits" that let 8 activation rows ride on an FP4 B operand.
//
// Operand A (weights): 128 rows x 64 inputs per MMA, K-major with no swizzle: 8-row x 16-byte core matrices, row
// group g at byte 256 g, input half h (32 inputs) at +128 h, row r % 8 at +16 (r % 8); byte j of a 16-byte row holds
// inputs 2j (low nibble) and 2j + 1.
// Scale factors (A and B alike): per 64 inputs a 512-byte atom, the scale of row r and 16-input group j at byte
// 16 (r % 32) + 4 (r / 32) + j; tcgen05.cp .32x128b.warpx4 copies it into 4 TMEM columns of every lane quarter.
//
// Operand B (activations): each 16-input group of an activation row x is brought into (1344, 2688] by a power of
// two p (kept beside the digits) and written as kDigits rows of E2M1 digits q_d with a UE4M3 scale s_d each,
// x p ~= sum_d s_d q_d: s_1 = the smallest UE4M3 >= max |x p| / 6, q_1 = the nearest E2M1 of x p / s_1, and each next
// digit encodes what is left. After a digit of scale s every residual is at most s (E2M1 rounding errs by at most one
// unit), so 4 digits leave |x - sum / p| <= ~8e-4 of the group's largest |x| in the worst case, and ~1e-4 typically:
// finer than a bf16 rounding of the group's largest element (2^-9 of it). A GEMV CTA brings the groups of its K slice
// to one prescale per row (the slice's smallest p) by scaling their s_d down, exactly unless they turn subnormal.
// Digit row n = 8 d + i (digit d of activation row i), N = 32, so one MMA multiplies 128 weight rows by every digit
// of all 8 rows; the epilogue adds the 4 digit columns of each row.
#pragma once

#include "common.cuh"

namespace xtg {

constexpr int kTileRows = 128;               // weight rows per tile (the MMA's M)
constexpr int kKBlock = 64;                  // inputs per MMA
constexpr int kUnitBytes = 4608;             // one (tile, K block) of A: 4096 code bytes + 512 scale bytes
constexpr int kUnitCodeBytes = 4096;
constexpr int kDigits = 4;
constexpr int kDigitRows = 8 * kDigits;      // the MMA's N
constexpr int kBCodeBytes = kDigits * 256;   // 8 rows x 64 inputs x 4 bits per digit
constexpr int kBBlockBytes = kBCodeBytes + 512;   // one K block of B: 1024 digit bytes + 512 scale bytes

// ---- operand layouts ----

// byte of A unit holding input k (0..63, even) of tile row r
__host__ __device__ __forceinline__ int a_code_offset(int r, int k) {
  return (r >> 3) * 256 + (k >> 5) * 128 + (r & 7) * 16 + ((k & 31) >> 1);
}
__host__ __device__ __forceinline__ int sf_offset(int r, int j) { return (r & 31) * 16 + (r >> 5) * 4 + j; }
// the 8 code bytes of 16-input group j (0..3) of digit d of activation row i in a B block
__host__ __device__ __forceinline__ int b_code_offset(int d, int i, int j) {
  return d * 256 + (j >> 1) * 128 + i * 16 + (j & 1) * 8;
}

// ---- descriptors (sm_100 shared-memory matrix descriptor, version 1, no swizzle) ----

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
__device__ __forceinline__ uint64_t a_desc(uint32_t saddr) { return smem_desc(saddr, 128, 256); }
__device__ __forceinline__ uint64_t sf_desc(uint32_t saddr) { return smem_desc(saddr, 0, 128); }

// kind::mxf4nvf4 instruction descriptor: E2M1 A and B, K-major, UE4M3 scales, M = 128, N = 32, K = 64
constexpr uint32_t kIdescFp4 = (1u << 7) | (1u << 10) | ((uint32_t)(kDigitRows >> 3) << 17) | ((128u >> 4) << 24);

// ---- tcgen05 ----

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t desc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}
// D (+)= A * B with the block scales at tsfa / tsfb; accumulate = 0 overwrites D
__device__ __forceinline__ void tc_mma_fp4(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t tsfa, uint32_t tsfb,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(kIdescFp4), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}
// the mbarrier completes once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 16 consecutive TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar)) : "memory");
}

// ---- cluster ----

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A cluster phase in two halves: every CTA arrives at its start, and waits before its first store into another CTA's
// shared memory, so that every CTA of the cluster has started by then.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// store a float into CTA `rank`'s copy of the shared array `local` points into
__device__ __forceinline__ void st_cluster_f32(float* local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// store 8 floats into CTA `rank`'s copy of the shared array `local` points into (16-byte aligned)
__device__ __forceinline__ void st_cluster_f32x8(float* local, uint32_t rank, const float (&v)[8]) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote), "f"(v[0]), "f"(v[1]), "f"(v[2]),
               "f"(v[3])
               : "memory");
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote + 16), "f"(v[4]), "f"(v[5]),
               "f"(v[6]), "f"(v[7])
               : "memory");
}

// ---- activation digits ----

// the smallest UE4M3 code whose value is >= t (0 <= t <= 448), and that value; no branches
__device__ __forceinline__ uint32_t ue4m3_ceil(float t, float& value) {
  // below 2^-6 the subnormal grid of 2^-9 (code 8 = 2^-6, the first normal code, when t rounds up to it); above, the
  // f32 mantissa rounded up to 3 bits
  const float sub = ceilf(t * 512.f);
  const uint32_t bits = (__float_as_uint(t) + 0xFFFFFu) & 0xFFF00000u;
  const uint32_t cn = (bits >> 20) - (120u << 3);
  const bool is_sub = t < 0.015625f, pos = t > 0.f;
  value = !pos ? 0.f : is_sub ? sub * 0.001953125f : __uint_as_float(bits);
  return !pos ? 0u : is_sub ? (uint32_t)sub : (cn > 0x7eu ? 0x7eu : cn);
}

// the power of two that brings max |x| into (1344, 2688]; 2^126 for all zeros, so that an empty group never sets
// the common prescale of a K slice (its digits and scales are zero at any prescale)
__device__ __forceinline__ float block_prescale(float amax) {
  if (!(amax > 0.f)) return __int_as_float((127 + 126) << 23);
  int e;
  const float f = frexpf(amax, &e);   // amax = f 2^e, f in [0.5, 1)
  int p = (f <= 0.65625f ? 12 : 11) - e;
  p = p > 126 ? 126 : (p < -126 ? -126 : p);
  return __int_as_float((127 + p) << 23);
}

// The digits of one 16-input group, computed by the 4 lanes of a quad (lanes 4g .. 4g + 3 of a warp, every lane of
// the warp taking part), each holding 4 consecutive inputs x[4 t .. 4 t + 3] (t = lane & 3). The group's power-of-two
// prescale p (returned) is `fixed` if given (> 0; the caller guarantees max |x| fixed <= 2688), else its own. Per
// digit, lane t gets the 2 code bytes of its inputs (code[d]: bits 0-15) and every lane the scale byte sf[d].
// Digit scales: E2M1 rounding of |y| <= 6 errs by at most 1 (the step from 4 to 6), so after a digit of scale s every
// residual is at most s and ceil(s / 6) is a safe next scale without looking at the residuals. Even digits take
// their scale from the group's residual maximum (a max over the quad), odd digits from that bound: half the shuffles
// of a per-digit maximum, for a reconstruction error within ~1.5x of it. A digit's value r / s only picks the code
// (the residual keeps the exact r - s q), so 1 / s may be the fast reciprocal.
template <int D>
__device__ __forceinline__ float digitize16_quad_n(const float (&x)[4], uint32_t (&code)[D], uint32_t (&sf)[D],
                                                   float fixed = 0.f) {
  float m = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  const float p = fixed > 0.f ? fixed : block_prescale(m);
  float r[4] = {x[0] * p, x[1] * p, x[2] * p, x[3] * p};
  m *= p;
  float s = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    float t;
    if (d & 1) {
      t = s * 0.16666668f;   // 1 / 6 rounded up
    } else {
      if (d > 0) {
        m = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
      }
      t = fminf(m * 0.16666668f, 448.f);
    }
    const uint32_t sb = ue4m3_ceil(t, s);
    sf[d] = sb;
    const float inv = sb ? __fdividef(1.f, s) : 0.f;
    const uint32_t b0 = f32x2_to_e2m1x2(r[0] * inv, r[1] * inv), b1 = f32x2_to_e2m1x2(r[2] * inv, r[3] * inv);
    code[d] = b0 | (b1 << 8);
    const uint32_t h0 = e2m1x2_to_f16x2(b0), h1 = e2m1x2_to_f16x2(b1);
    const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&h0));
    const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&h1));
    r[0] = fmaf(-s, v0.x, r[0]);
    r[1] = fmaf(-s, v0.y, r[1]);
    r[2] = fmaf(-s, v1.x, r[2]);
    r[3] = fmaf(-s, v1.y, r[3]);
  }
  return p;
}
__device__ __forceinline__ float digitize16_quad(const float (&x)[4], uint32_t (&code)[kDigits],
                                                 uint32_t (&sf)[kDigits], float fixed = 0.f) {
  return digitize16_quad_n<kDigits>(x, code, sf, fixed);
}

// ---- the GEMM's activation units (gemm.cu): 64 activation rows x 64 inputs, 4 digits each (N = 256 digit rows,
// digit d of row i at row 64 d + i) in the weight unit's K-major layout, then the scale atoms of digit rows 0-127 and
// 128-255; one power-of-two prescale per activation row ----
constexpr int kGemmDigits = 4;
constexpr int kGemmRows = 64;
constexpr int kGemmCodeBytes = kGemmRows * kGemmDigits * 32;   // 8192
constexpr int kGemmUnitBytes = kGemmCodeBytes + 2 * 512;
// Lane t of the quad stores its part of 16-input group g of activation row `row` (of the 64-row tile at act)
__device__ __forceinline__ void store_gemm_digits_quad(uint8_t* act, int row, int g, int t,
                                                       const uint32_t (&code)[kGemmDigits],
                                                       const uint32_t (&sf)[kGemmDigits]) {
  uint8_t* unit = act + (int64_t)(g >> 2) * kGemmUnitBytes;
  const int j = g & 3, i = row % kGemmRows;
#pragma unroll
  for (int d = 0; d < kGemmDigits; ++d) {
    const int n = kGemmRows * d + i;
    *reinterpret_cast<uint16_t*>(unit + a_code_offset(n, 16 * j + 4 * t)) = (uint16_t)code[d];
    if (t == 0) unit[kGemmCodeBytes + (n >> 7) * 512 + sf_offset(n & 127, j)] = (uint8_t)sf[d];
  }
}

// the prescale of groups nobody wrote (all-zero digits): never the smallest of a slice
constexpr float kEmptyPrescale = 8.507059e37f;   // 2^126

// Lane t of the quad stores its part of group j (0..3 within the block) of activation row i; lane 0 the scales.
__device__ __forceinline__ void store_digits_quad(uint8_t* blk, int i, int j, int t, const uint32_t (&code)[kDigits],
                                                  const uint32_t (&sf)[kDigits]) {
#pragma unroll
  for (int d = 0; d < kDigits; ++d) {
    *reinterpret_cast<uint16_t*>(blk + b_code_offset(d, i, j) + 2 * t) = (uint16_t)code[d];
    if (t == 0) blk[kBCodeBytes + sf_offset(8 * d + i, j)] = (uint8_t)sf[d];
  }
}

// A UE4M3 scale times 2^-k (k >= 0): exact while it stays normal, then rounded to the subnormal grid (2^-9).
__device__ __forceinline__ uint32_t ue4m3_scale_down(uint32_t c, int k) {
  if (k <= 0 || c == 0u) return c;
  const int e = (int)(c >> 3), m = (int)(c & 7);
  if (e - k >= 1) return c - 8u * (uint32_t)k;
  // value / 2^-9 = (8 + m) 2^(e - 1 - k) for e >= 1, m 2^-k for e = 0
  const int num = e >= 1 ? 8 + m : m, sh = e >= 1 ? 1 + k - e : k;
  if (sh >= 31) return 0u;
  return (uint32_t)((num + ((1 << sh) >> 1)) >> sh);
}

}  // namespace xtg
