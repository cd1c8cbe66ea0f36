// K4 / K5 helpers of the step: the embedding of a tied NVFP4 head (nvfp4_row, engine/src/kernels.cpp:34-45) or of a
// checkpoint's BF16 table (bf16_row, kernels.cpp:157-160) with the
// step's RoPE tables and ring bookkeeping, the nGPT residual updates (slerp_residual and the loop norms,
// kernels.cpp:177-189 and packs/dory/dory.cpp:530-542), the argmax over the head's tile candidates
// (engine/src/sampler.cpp:8-13), and the KV writes outside the attention kernel (KvCache::store, kv.cpp:75-112, in
// this library's layout) plus the seeded KV prefill.
#include "attention.h"
#include "common.cuh"
#include "elementwise.h"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

namespace {

__device__ __forceinline__ float packed_weight(const uint8_t* w, int kblocks, float global, int row, int k) {
  const int t = row / kTileRows, r = row % kTileRows, b = k / kKBlock, kk = k % kKBlock;
  const uint8_t* unit = w + ((int64_t)t * kblocks + b) * kUnitBytes;
  const uint8_t byte = unit[a_code_offset(r, kk & ~1)];
  const uint8_t sc = unit[kUnitCodeBytes + sf_offset(r, kk >> 4)];
  const float s = __fmul_rn(e4m3_to_f32(sc), global);
  return __fmul_rn(e2m1_to_f32((kk & 1) ? byte >> 4 : byte & 15), s);
}

// Activation row i (hidden values in shared memory) -> its B digits in xb and the prescale of every 16-input group
// in xb_pre (zero digits for zero rows); every thread of the CTA takes part (a quad per group). The other rows' bytes
// of xb are left alone.
__device__ __forceinline__ void digitize_row(const float* row, int hidden, int i, bool zero, uint8_t* xb,
                                             float* xb_pre, float fixed) {
  const int groups = (hidden + 15) / 16;
  for (int q0 = 0; q0 < groups * 4; q0 += blockDim.x) {
    const int q = q0 + (int)threadIdx.x, g = q >> 2, t = q & 3;
    const bool active = g < groups;
    float v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int k = 16 * g + 4 * t + c;
      v[c] = (active && !zero && k < hidden) ? row[k] : 0.f;
    }
    uint32_t code[kDigits], sf[kDigits];
    const float p = digitize16_quad(v, code, sf, fixed);   // whole warps take part
    if (active) {
      store_digits_quad(xb + (int64_t)(g >> 2) * kBBlockBytes, i, g & 3, t, code, sf);
      if (t == 0) xb_pre[(int64_t)g * 8 + i] = p;
    }
  }
}

__global__ void embed_kernel(const EmbedArgs a) {
  extern __shared__ float rowbuf[];   // [hidden]
  const int r = blockIdx.x;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const StepParams* p = a.params;
  const int m = p->m;
  const int64_t pos0 = p->pos0;
  if (r < m) {
    const int tok = p->tokens[r];
    for (int k = threadIdx.x; k < a.hidden; k += blockDim.x) {
      const float v = a.table ? bf16_bits_to_f32(a.table[(int64_t)tok * a.hidden + k])
                              : packed_weight(a.head, a.kblocks, a.global, tok, k);
      a.h[(int64_t)r * a.hidden + k] = v;
      rowbuf[k] = v;
    }
  }
  __syncthreads();
  digitize_row(rowbuf, a.hidden, r, r >= m, a.xb, a.xb_pre, 0.f);
  // RoPE tables of this step's positions (FP32(pos) * inv_freq, then cos / sin), one per theta
  if (r < a.n_thetas) {
    const int half = a.rope_half > 0 ? a.rope_half : 64;
    for (int idx = threadIdx.x; idx < kMaxRows * half; idx += blockDim.x) {
      const int i = idx / half, e = idx % half;
      const float ang = __fmul_rn((float)(pos0 + i), a.inv_freq[r * half + e]);
      float s, c;
      sincosf(ang, &s, &c);
      a.rope_cos[(r * kMaxRows + i) * half + e] = c;
      a.rope_sin[(r * kMaxRows + i) * half + e] = s;
    }
  }
  // the ring's slot -> position table gains this step's rows (attention masks positions >= pos0 anyway)
  if (r == 0 && a.ring_pos && threadIdx.x < m) {
    const int64_t q = pos0 + threadIdx.x;
    a.ring_pos[q % a.ring] = (int32_t)q;
  }
}

// the residual stream is unit-norm after every update (|h| <= 1): one prescale for all its groups (2^11)
constexpr float kUnitNorm = kUnitPrescale;

// Block-wide sums of two values at once (fixed order, deterministic).
__device__ __forceinline__ float2 block_sum2(float x, float y, float2* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  x = warp_sum(x);
  y = warp_sum(y);
  __syncthreads();
  if (lane == 0) red[warp] = make_float2(x, y);
  __syncthreads();
  float2 t = lane < nw ? red[lane] : make_float2(0.f, 0.f);
  t.x = warp_sum(t.x);
  t.y = warp_sum(t.y);
  return t;
}

// One CTA per activation row: the residual updates. All norms are justnorm: x / sqrt(sum x^2 + 1e-6). Thread t holds
// the 4 consecutive elements 4 c .. 4 c + 3 of each of its chunks c = t + j * blockDim (j < kChunks) in registers, so
// that the 4 threads of a quad hold one 16-input group and digitize it straight from registers.
constexpr int kResidThreads = 1024;
constexpr int kChunks = 2;   // hidden <= 8192

__device__ __forceinline__ float4 ld4(const float* p, int c, bool ok) {
  return ok ? reinterpret_cast<const float4*>(p)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ void st4(float* p, int c, const float (&v)[4]) {
  reinterpret_cast<float4*>(p)[c] = make_float4(v[0], v[1], v[2], v[3]);
}

__global__ void __launch_bounds__(kResidThreads) resid_kernel(const ResidArgs a) {
  __shared__ float2 red[32];
  const int r = blockIdx.x, H = a.hidden;
  bool ok[kChunks];
  int ch[kChunks];
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    ch[j] = (int)threadIdx.x + j * kResidThreads;
    ok[j] = 4 * ch[j] < H;
  }
  // the slerp's per-dimension rate is a parameter: loaded before the dependency wait
  float lr[kChunks][4];
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const float4 l4 = ld4(a.lr, ch[j], a.mode == kResidSlerp && ok[j]);
    lr[j][0] = l4.x; lr[j][1] = l4.y; lr[j][2] = l4.z; lr[j][3] = l4.w;
  }
  // live rows: one sequence's rows below m, or (batched) row r % 8 of sequence r / 8 below that sequence's m
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = a.nseq > 0 ? (r % kMaxRows) < a.params[r / kMaxRows].m : r < (a.params ? a.params->m : a.m);
  float* h = a.h + (int64_t)r * H;
  float v[kChunks][4];
  if (!live) {
#pragma unroll
    for (int j = 0; j < kChunks; ++j) v[j][0] = v[j][1] = v[j][2] = v[j][3] = 0.f;
  } else if (a.mode == kResidSlerp) {
    const float* o = a.o + (int64_t)r * H;
    float hv[kChunks][4], ov[kChunks][4];
    float sa = 0.f, sb = 0.f;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const float4 h4 = ld4(h, ch[j], ok[j]);
      float4 o4 = ld4(o, ch[j], ok[j]);
      for (int q = 1; q < a.o_parts; ++q) {   // a K-split GEMM's partial outputs, in order
        const float4 p4 = ld4(o + q * a.o_stride, ch[j], ok[j]);
        o4.x += p4.x;
        o4.y += p4.y;
        o4.z += p4.z;
        o4.w += p4.w;
      }
      hv[j][0] = h4.x; hv[j][1] = h4.y; hv[j][2] = h4.z; hv[j][3] = h4.w;
      ov[j][0] = o4.x; ov[j][1] = o4.y; ov[j][2] = o4.z; ov[j][3] = o4.w;
    }
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        sa += hv[j][c] * hv[j][c];
        sb += ov[j][c] * ov[j][c];
      }
    const float2 n2 = block_sum2(sa, sb, red);
    const float fa = 1.f / sqrtf(n2.x + 1e-6f), fb = 1.f / sqrtf(n2.y + 1e-6f);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float ya = hv[j][c] * fa, yb = ov[j][c] * fb;
        v[j][c] = ya + lr[j][c] * (yb - ya);
        ss += v[j][c] * v[j][c];
      }
    const float f = 1.f / sqrtf(block_sum2(ss, 0.f, red).x + 1e-6f);
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) v[j][c] *= f;
  } else {
    float* st = a.state + (int64_t)r * H;
    float* in = a.input + (int64_t)r * H;
    float hv[kChunks][4], iv[kChunks][4];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const float4 h4 = ld4(h, ch[j], ok[j]), i4 = ld4(in, ch[j], ok[j] && a.mode != kResidLoopBegin);
      hv[j][0] = h4.x; hv[j][1] = h4.y; hv[j][2] = h4.z; hv[j][3] = h4.w;
      iv[j][0] = i4.x; iv[j][1] = i4.y; iv[j][2] = i4.z; iv[j][3] = i4.w;
    }
    if (a.mode == kResidLoopBegin) {   // input = state = h
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
        if (ok[j]) {
          st4(st, ch[j], hv[j]);
          st4(in, ch[j], hv[j]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) iv[j][c] = hv[j][c];
      }
    } else {   // the loop that ends: state = justnorm(h)
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) s += hv[j][c] * hv[j][c];
      const float f = 1.f / sqrtf(block_sum2(s, 0.f, red).x + 1e-6f);
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
#pragma unroll
        for (int c = 0; c < 4; ++c) hv[j][c] *= f;
        if (ok[j]) st4(st, ch[j], hv[j]);
      }
    }
    if (a.mode == kResidLoopEnd) {   // h = state
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) v[j][c] = hv[j][c];
    } else {   // a loop begins: h = justnorm(state + input)
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          v[j][c] = hv[j][c] + iv[j][c];
          s += v[j][c] * v[j][c];
        }
      const float f = 1.f / sqrtf(block_sum2(s, 0.f, red).x + 1e-6f);
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) v[j][c] *= f;
    }
  }
  // the new h, and its digits: the quad of threads 4 g .. 4 g + 3 of chunk j holds group g + 256 j
  if (a.gemm_act) {   // the batched step's GEMM digits of the new h (4 per value, the unit prescale)
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      if (j * kResidThreads < H / 4) {   // whole warps take part in the quad's shuffles
        uint32_t code[kGemmDigits], sf[kGemmDigits];
        digitize16_quad_n<kGemmDigits>(v[j], code, sf, kUnitNorm);
        if (ok[j]) store_gemm_digits_quad(a.gemm_act, r, ch[j] >> 2, ch[j] & 3, code, sf);
      }
    }
    if (threadIdx.x == 0) a.gemm_post[r] = 1.f / kUnitNorm;
  }
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    if (live && ok[j]) st4(h, ch[j], v[j]);
    if (a.xb && j * kResidThreads < H / 4) {   // whole warps take part in the quad's shuffles
      uint32_t code[kDigits], sf[kDigits];
      const float p = digitize16_quad(v[j], code, sf, kUnitNorm);
      if (ok[j]) {
        const int g = ch[j] >> 2, t = ch[j] & 3;
        store_digits_quad(a.xb + (int64_t)(g >> 2) * kBBlockBytes, r, g & 3, t, code, sf);
        if (t == 0) a.xb_pre[(int64_t)g * 8 + r] = p;
      }
    }
  }
}

// The slerp update from the producer's row sums (GemvArgs::rsum): |h|^2, |o|^2 and the three sums that give
// |(1 - lr) fa h + lr fb o|^2 = fa^2 A + 2 fa fb B + fb^2 C, so a CTA needs only its own dims. Grid (slices of 256
// dims, 8 activation rows), 64 threads; thread t holds dims 256 s + 4 t .. + 3, a quad of threads one 16-input group.
constexpr int kSlerpDims = 256, kSlerpThreads = kSlerpDims / 4;
constexpr int kSlerpPartLoads = 5;   // partials per thread: at most 320 producer CTAs

__global__ void __launch_bounds__(kSlerpThreads) resid_slerp_kernel(const ResidArgs a) {
  __shared__ float red[kSlerpThreads / 32][5];
  const int r = blockIdx.y, t = threadIdx.x, H = a.hidden, lane = t & 31, warp = t >> 5;
  const int c = blockIdx.x * kSlerpThreads + t;   // this thread's float4 of the row
  const bool ok = 4 * c < H;
  const float4 l4 = ld4(a.lr, c, ok);   // a parameter: before the dependency wait
  const int m = a.params ? a.params->m : a.m;
  if (a.pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  const bool live = r < m;
  // one wave of loads: this thread's share of the partials (parts t, t + 64, ..., summed in order), h and o
  float pv[kSlerpPartLoads][5];
#pragma unroll
  for (int it = 0; it < kSlerpPartLoads; ++it) {
    const int q = t + it * kSlerpThreads;
    const bool lq = live && q < a.nparts;
#pragma unroll
    for (int k = 0; k < 5; ++k) pv[it][k] = lq ? a.rsum[((int64_t)k * 8 + r) * a.nparts + q] : 0.f;
  }
  float* h = a.h + (int64_t)r * H;
  const float4 h4 = ld4(h, c, ok && live), o4 = ld4(a.o + (int64_t)r * H, c, ok && live);
  float s5[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    s5[k] = pv[0][k];
#pragma unroll
    for (int it = 1; it < kSlerpPartLoads; ++it) s5[k] += pv[it][k];
  }
#pragma unroll
  for (int k = 0; k < 5; ++k) s5[k] = warp_sum(s5[k]);
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < 5; ++k) red[warp][k] = s5[k];
  __syncthreads();
  float tot[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) tot[k] = red[0][k] + red[1][k];
  const float fa = 1.f / sqrtf(tot[0] + 1e-6f), fb = 1.f / sqrtf(tot[1] + 1e-6f);
  const float f = 1.f / sqrtf(fa * fa * tot[2] + 2.f * fa * fb * tot[3] + fb * fb * tot[4] + 1e-6f);
  const float hv[4] = {h4.x, h4.y, h4.z, h4.w}, ov[4] = {o4.x, o4.y, o4.z, o4.w}, lv[4] = {l4.x, l4.y, l4.z, l4.w};
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = live ? ((1.f - lv[k]) * fa * hv[k] + lv[k] * fb * ov[k]) * f : 0.f;
  if (live && ok) st4(h, c, v);
  uint32_t code[kDigits], sf[kDigits];
  const float p = digitize16_quad(v, code, sf, kUnitNorm);   // whole warps take part
  if (ok) {
    const int g = c >> 2, q = c & 3;
    store_digits_quad(a.xb + (int64_t)(g >> 2) * kBBlockBytes, r, g & 3, q, code, sf);
    if (q == 0) a.xb_pre[(int64_t)g * 8 + r] = p;
  }
}

__global__ void argmax_kernel(const ArgCand* cand, int tiles, const StepParams* params, int32_t* out,
                              float* out_val, uint32_t* epoch, int pdl) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int n = blockIdx.x;
  if (pdl) {
    pdl_wait();
    pdl_launch_next();
  }
  // the step's last kernel: every earlier one has finished, so the step count moves on here
  if (epoch && n == 0 && threadIdx.x == 0) *epoch += 1u;
  if (n >= params->m) return;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int t = threadIdx.x; t < tiles; t += blockDim.x) {
    const ArgCand c = cand[t * kMaxRows + n];
    if (c.v > v || (c.v == v && c.i < idx)) {
      v = c.v;
      idx = c.i;
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
    if (lane == 0) {
      out[n] = idx;
      if (out_val) out_val[n] = v;
    }
  }
}

// KvCache::store in this library's layout: rows [n][kv_heads][128] at positions pos .. pos + n - 1 (a ring keeps
// the last `slots`); one warp per (row, head, K or V).
__global__ void kv_store_kernel(const KvStoreArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t task = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t total = (int64_t)a.n * a.kv_heads * 2;
  if (task >= total) return;
  const int kv = (int)(task % 2), h = (int)((task / 2) % a.kv_heads);
  const int64_t r = task / (2 * a.kv_heads);
  if (a.ring && r < a.n - a.slots) return;   // a long chunk leaves only its last `slots` rows in a ring
  const int64_t p = a.pos + r, slot = a.ring ? p % a.slots : p;
  const float* src = (kv ? a.v : a.k) + (r * a.kv_heads + h) * 128;
  const float x[4] = {src[lane], src[lane + 64], src[lane + 32], src[lane + 96]};
  float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  amax = warp_max(amax);
  const float top = a.dtype == kKvFp8 ? 448.f : 127.f;
  const float sc = amax > 0.f ? __fdiv_rn(amax, top) : 1.f;
  const float inv = __fdiv_rn(1.f, sc);
  const int idx[4] = {lane, lane + 64, lane + 32, lane + 96};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float t = __fmul_rn(x[j], inv);
    uint8_t c;
    if (a.dtype == kKvFp8) {
      c = f32_to_e4m3(t);
    } else {
      float q = fminf(fmaxf(rintf(t), -127.f), 127.f);
      c = (uint8_t)(int8_t)(int)q;
    }
    if (kv)
      a.vc[v_offset(h, idx[j], slot, a.slots)] = c;
    else
      a.kc[k_offset(h, slot, idx[j], a.slots)] = c;
  }
  if (lane == 0) (kv ? a.vs : a.ks)[(int64_t)h * a.slots + slot] = sc;
}

// The seeded prefill of one instance (the oracle's xo_synth_state_new): element (slot, head, e) of K / V codes is
// draw (slot * kv_heads + head) * 128 + e of its stream, scales draw slot * kv_heads + head; `filled` slots.
__global__ void kv_prefill_kernel(uint64_t key_k, uint64_t key_v, uint64_t key_ks, uint64_t key_vs, float lo,
                                  float span, int64_t filled, int kv_heads, int hd, int64_t slots, uint8_t* kc,
                                  uint8_t* vc, float* ks, float* vs) {
  const int64_t total = filled * kv_heads * hd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)(i % hd);
    const int64_t sh = i / hd;   // slot * kv_heads + head
    const int h = (int)(sh % kv_heads);
    const int64_t s = sh / kv_heads;
    kc[k_offset(h, s, e, slots, hd)] = (uint8_t)(int8_t)((int)(rand_bits(key_k, i) % 255u) - 127);
    vc[v_offset(h, e, s, slots, hd)] = (uint8_t)(int8_t)((int)(rand_bits(key_v, i) % 255u) - 127);
    if (e == 0) {
      ks[(int64_t)h * slots + s] = uniform_from_bits(rand_bits(key_ks, sh), lo, span);
      vs[(int64_t)h * slots + s] = uniform_from_bits(rand_bits(key_vs, sh), lo, span);
    }
  }
}

template <class Args>
void launch_pdl(void (*kernel)(Args), dim3 grid, dim3 block, const Args& args, cudaStream_t s, bool pdl,
                size_t smem = 0) {
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

}  // namespace

void launch_embed(const EmbedArgs& a_in, cudaStream_t s, bool pdl) {
  EmbedArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  XTG_REQUIRE(a.hidden <= 8192, "embed: hidden above 8192");
  launch_pdl(embed_kernel, dim3(kMaxRows), dim3(256), a, s, pdl, (size_t)a.hidden * sizeof(float));
}

void launch_resid(const ResidArgs& a_in, cudaStream_t s, bool pdl) {
  ResidArgs a = a_in;
  a.pdl = pdl ? 1 : 0;
  XTG_REQUIRE(a.hidden <= 4 * kChunks * kResidThreads && a.hidden % 64 == 0, "resid: hidden a multiple of 64, at most 8192");
  if (a.mode == kResidSlerp && a.rsum) {
    XTG_REQUIRE(a.nparts <= kSlerpPartLoads * kSlerpThreads, "resid: at most 320 row-sum partials");
    launch_pdl(resid_slerp_kernel, dim3((a.hidden + kSlerpDims - 1) / kSlerpDims, kMaxRows), dim3(kSlerpThreads), a,
               s, pdl, 0);
    return;
  }
  XTG_REQUIRE(a.nseq >= 0 && a.nseq <= 64, "resid: at most 64 sequences");
  XTG_REQUIRE(!a.gemm_act || (a.nseq >= 1 && a.nseq <= 8 && a.gemm_post), "resid: GEMM digits for 1..8 sequences");
  if (a.o_parts < 1) a.o_parts = 1;
  launch_pdl(resid_kernel, dim3(kMaxRows * (a.nseq > 0 ? a.nseq : 1)), dim3(kResidThreads), a, s, pdl, 0);
}

void launch_argmax(const ArgCand* cand, int tiles, const StepParams* params, int32_t* out, float* out_val,
                   uint32_t* epoch, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kMaxRows);
  cfg.blockDim = dim3(1024);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  XTG_CUDA(cudaLaunchKernelEx(&cfg, argmax_kernel, cand, tiles, params, out, out_val, epoch, pdl ? 1 : 0));
}

void launch_kv_store(const KvStoreArgs& a, cudaStream_t s) {
  const int64_t tasks = (int64_t)a.n * a.kv_heads * 2;
  if (tasks == 0) return;
  const int grid = (int)((tasks + 7) / 8);
  kv_store_kernel<<<grid, 256, 0, s>>>(a);
  XTG_CUDA(cudaGetLastError());
}

void kv_prefill(uint64_t seed, uint64_t stream_base, float lo, float hi, int64_t filled, int kv_heads, int hd,
                int64_t slots, uint8_t* kc, uint8_t* vc, float* ks, float* vs, cudaStream_t s) {
  if (filled <= 0) return;
  const int64_t total = filled * kv_heads * hd;
  const int64_t g = (total + 255) / 256;
  const int grid = (int)(g < 148 * 16 ? g : 148 * 16);
  kv_prefill_kernel<<<grid, 256, 0, s>>>(rand_key(seed, stream_base + 0), rand_key(seed, stream_base + 1),
                                         rand_key(seed, stream_base + 2), rand_key(seed, stream_base + 3), lo,
                                         hi - lo, filled, kv_heads, hd, slots, kc, vc, ks, vs);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg
