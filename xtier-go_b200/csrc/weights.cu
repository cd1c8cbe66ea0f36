// NVFP4 weights on the device: the seeded synthetic generators, the NVFP4 quantizer, and the repack from ModelOpt's
// row layout (engine/include/xtg/kernels.h:13-20) into the GEMV's streaming layout.
//
// The packed layout is the tensor-core unit of fp4mma.cuh: per (128-row tile, 64-input block) 4096 code bytes in
// the MMA's A layout and 512 E4M3 scale bytes in the scale-factor atom, units in tile-major order. Rows past n_out
// and inputs past k are zero codes with zero scales. An interleaved pack puts 64 rows of weight A (gate) in tile rows
// 0-63 and the same 64 rows of weight B (up) in rows 64-127, so that gate and up of a feature finish in one tile.
#include "common.cuh"
#include "fp4mma.cuh"
#include "kernels.h"

namespace xtg {

// ---- generators (the oracle's xo_gen_*; stream / index -> the same bits) ----

__global__ void gen_normal_bf16_kernel(uint64_t key, float stddev, uint16_t* out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f32_to_bf16_bits(__fmul_rn(normal_from_bits(rand_bits(key, (uint64_t)i)), stddev));
}

__global__ void gen_uniform_kernel(uint64_t key, float lo, float span, float* out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = uniform_from_bits(rand_bits(key, (uint64_t)i), lo, span);
}

__global__ void gen_int8_kernel(uint64_t key, int8_t* out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (int8_t)((int)(rand_bits(key, (uint64_t)i) % 255u) - 127);
}

static int grid_for(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  return (int)(g < 148 * 16 ? (g > 0 ? g : 1) : 148 * 16);
}

void gen_normal_bf16(uint64_t seed, uint64_t stream, float stddev, uint16_t* out, int64_t n, cudaStream_t s) {
  gen_normal_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(rand_key(seed, stream), stddev, out, n);
  XTG_CUDA(cudaGetLastError());
}

void gen_uniform(uint64_t seed, uint64_t stream, float lo, float hi, float* out, int64_t n, cudaStream_t s) {
  const float span = hi - lo;   // the oracle rounds the span on the host the same way
  gen_uniform_kernel<<<grid_for(n, 256), 256, 0, s>>>(rand_key(seed, stream), lo, span, out, n);
  XTG_CUDA(cudaGetLastError());
}

void gen_int8(uint64_t seed, uint64_t stream, int8_t* out, int64_t n, cudaStream_t s) {
  gen_int8_kernel<<<grid_for(n, 256), 256, 0, s>>>(rand_key(seed, stream), out, n);
  XTG_CUDA(cudaGetLastError());
}

// ---- NVFP4 quantizer: global = amax / (6 * 448); block scale = E4M3(amax_block / (6 * global)); codes = nearest
// E2M1 of w / (scale * global), ties to the even code ----

__global__ void amax_bf16_kernel(const uint16_t* w, int64_t n, unsigned int* amax_bits) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(bf16_bits_to_f32(w[i])));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));   // non-negative floats order as ints
}

__global__ void quantize_nvfp4_kernel(const uint16_t* w, int n_out, int k, const unsigned int* amax_bits,
                                      uint8_t* codes, uint8_t* scales, float* global_out) {
  const float amax = __uint_as_float(*amax_bits);
  float global = __fdiv_rn(amax, 2688.f);
  if (global == 0.f) global = 1.f;
  const int groups = k / 16;
  const int64_t total = (int64_t)n_out * groups;
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_out = global;
  const float six_g = __fmul_rn(6.f, global);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = i / groups, g = i % groups;
    const uint16_t* src = w + n * k + g * 16;
    float v[16];
    float bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = bf16_bits_to_f32(src[j]);
      bmax = fmaxf(bmax, fabsf(v[j]));
    }
    float sc = __fdiv_rn(bmax, six_g);
    if (sc == 0.f) sc = 1.f;
    const uint8_t sc_code = f32_to_e4m3(sc);
    scales[i] = sc_code;
    const float denom = __fmul_rn(e4m3_to_f32(sc_code), global);
    uint8_t* dst = codes + n * (k / 2) + g * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      dst[j] = (uint8_t)(e2m1_code(__fdiv_rn(v[2 * j], denom)) | (e2m1_code(__fdiv_rn(v[2 * j + 1], denom)) << 4));
  }
}

void quantize_nvfp4(const uint16_t* w, int n_out, int k, uint8_t* codes, uint8_t* scales, float* global_out,
                    unsigned int* amax_scratch, cudaStream_t s) {
  XTG_REQUIRE(k % 16 == 0, "quantize_nvfp4: k must be a multiple of 16");
  XTG_CUDA(cudaMemsetAsync(amax_scratch, 0, sizeof(unsigned int), s));
  const int64_t n = (int64_t)n_out * k;
  amax_bf16_kernel<<<grid_for(n, 256), 256, 0, s>>>(w, n, amax_scratch);
  XTG_CUDA(cudaGetLastError());
  const int64_t groups = (int64_t)n_out * (k / 16);
  quantize_nvfp4_kernel<<<grid_for(groups, 256), 256, 0, s>>>(w, n_out, k, amax_scratch, codes, scales, global_out);
  XTG_CUDA(cudaGetLastError());
}

// ---- repack ModelOpt rows -> tensor-core units ----

// One thread per (tile, K block, tile row): the row's 32 code bytes (two 16-byte halves of the A layout) and its 4
// scale bytes in the scale-factor atom.
__global__ void pack_nvfp4_kernel(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b,
                                  const uint8_t* scales_b, int n_out, int k, int interleave, int tiles, int kblocks,
                                  uint8_t* dst) {
  const int64_t total = (int64_t)tiles * kblocks * kTileRows;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i % kTileRows);
    const int64_t tb = i / kTileRows;
    const int t = (int)(tb / kblocks), b = (int)(tb % kblocks);
    const uint8_t* c = codes_a;
    const uint8_t* sc = scales_a;
    int row = t * kTileRows + r;
    if (interleave) {
      row = t * 64 + (r & 63);
      if (r >= 64) {
        c = codes_b;
        sc = scales_b;
      }
    }
    uint8_t* unit = dst + tb * kUnitBytes;
    uint8_t bytes[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int kk = b * kKBlock + 2 * q;
      bytes[q] = (row < n_out && kk < k) ? c[(int64_t)row * (k / 2) + kk / 2] : 0;
    }
    *reinterpret_cast<uint4*>(unit + a_code_offset(r, 0)) = *reinterpret_cast<const uint4*>(bytes);
    *reinterpret_cast<uint4*>(unit + a_code_offset(r, 32)) = *reinterpret_cast<const uint4*>(bytes + 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int grp = b * 4 + j;
      unit[kUnitCodeBytes + sf_offset(r, j)] = (row < n_out && grp * 16 < k) ? sc[(int64_t)row * (k / 16) + grp] : 0;
    }
  }
}

void pack_nvfp4(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b, const uint8_t* scales_b,
                int n_out, int k, bool interleave, uint8_t* dst, cudaStream_t s) {
  XTG_REQUIRE(k % 16 == 0, "pack_nvfp4: k must be a multiple of 16");
  const int tiles = packed_tiles(n_out, interleave), kblocks = packed_kblocks(k);
  const int64_t total = (int64_t)tiles * kblocks * kTileRows;
  pack_nvfp4_kernel<<<grid_for(total, 256), 256, 0, s>>>(codes_a, scales_a, codes_b, scales_b, n_out, k,
                                                         interleave ? 1 : 0, tiles, kblocks, dst);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg
