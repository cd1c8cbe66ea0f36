// NVFP4 weights on the device: the seeded synthetic generators, the NVFP4 quantizer, and the repack from ModelOpt's
// row layout (engine/include/xtg/kernels.h:13-20) into the GEMV's streaming layout.
//
// Streaming layout. A weight [n_out][k] is cut into tiles of 16 output rows and blocks of 64 inputs; block (t, b)
// is 576 contiguous bytes, blocks in tile-major order, so that any run of blocks is one contiguous byte range:
//   bytes   0..511  codes, 16 per lane of a warp: lane L = 4 g + tq holds, for each k16 step j = 0..3 of the block,
//                   [row g byte tq, row g+8 byte tq, row g byte tq+4, row g+8 byte tq+4] of that step's 8 code bytes
//                   (byte q of a step holds inputs 2q (low nibble) and 2q+1), i.e. exactly the A fragment of
//                   mma.m16n8k16 after an e2m1x2 -> f16x2 conversion per byte;
//   bytes 512..575  E4M3 scales, 8 per lane group g: for j = 0..3, [scale(row g, step j), scale(row g+8, step j)].
// Rows past n_out and inputs past k are zero codes with zero scales. An interleaved pack puts 8 rows of weight A
// (gate) in tile rows 0-7 and the same 8 rows of weight B (up) in rows 8-15, so that one lane holds gate and up of
// the same feature after the MMA.
#include "common.cuh"
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

// ---- repack ModelOpt rows -> streaming layout ----

// One thread per (tile, block, lane): 16 code bytes, and for lanes 0..7 the 8 scale bytes of row group `lane`.
__global__ void pack_nvfp4_kernel(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b,
                                  const uint8_t* scales_b, int n_out, int k, int interleave, int tiles, int blocks,
                                  uint8_t* dst) {
  const int64_t total = (int64_t)tiles * blocks * 32;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int lane = (int)(i & 31);
    const int64_t tb = i >> 5;
    const int t = (int)(tb / blocks), b = (int)(tb % blocks);
    uint8_t* out = dst + tb * kBlockBytes;
    // the source of tile row r
    auto src = [&](int r, const uint8_t*& c, const uint8_t*& s, int& row) {
      if (interleave) {
        row = t * 8 + (r & 7);
        c = r < 8 ? codes_a : codes_b;
        s = r < 8 ? scales_a : scales_b;
      } else {
        row = t * 16 + r;
        c = codes_a;
        s = scales_a;
      }
    };
    const int g = lane >> 2, tq = lane & 3;
    uint8_t bytes[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = b * 64 + j * 16;   // first input of the step
#pragma unroll
      for (int part = 0; part < 4; ++part) {
        const int r = g + ((part & 1) ? 8 : 0);
        const int q = tq + ((part & 2) ? 4 : 0);
        const uint8_t* c;
        const uint8_t* s;
        int row;
        src(r, c, s, row);
        uint8_t v = 0;
        if (row < n_out && kk + 2 * q < k) v = c[(int64_t)row * (k / 2) + kk / 2 + q];
        (void)s;
        bytes[4 * j + part] = v;
      }
    }
    *reinterpret_cast<uint4*>(out + lane * 16) = *reinterpret_cast<const uint4*>(bytes);
    if (lane < 8) {
      uint8_t sb[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int grp = b * 4 + j;
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const uint8_t* c;
          const uint8_t* s;
          int row;
          src(lane + 8 * hi, c, s, row);
          (void)c;
          sb[2 * j + hi] = (row < n_out && grp * 16 < k) ? s[(int64_t)row * (k / 16) + grp] : 0;
        }
      }
      *reinterpret_cast<uint2*>(out + 512 + lane * 8) = *reinterpret_cast<const uint2*>(sb);
    }
  }
}

void pack_nvfp4(const uint8_t* codes_a, const uint8_t* scales_a, const uint8_t* codes_b, const uint8_t* scales_b,
                int n_out, int k, bool interleave, uint8_t* dst, cudaStream_t s) {
  const int tiles = packed_tiles(n_out, interleave), blocks = packed_blocks(k);
  const int64_t total = (int64_t)tiles * blocks * 32;
  pack_nvfp4_kernel<<<grid_for(total, 256), 256, 0, s>>>(codes_a, scales_a, codes_b, scales_b, n_out, k,
                                                         interleave ? 1 : 0, tiles, blocks, dst);
  XTG_CUDA(cudaGetLastError());
}

// The inverse: tile rows back to ModelOpt codes / scales (debug exports, tests).
__global__ void unpack_nvfp4_kernel(const uint8_t* src, int n_out, int k, int tiles, int blocks, uint8_t* codes,
                                    uint8_t* scales) {
  const int64_t total = (int64_t)n_out * (k / 16);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(i / (k / 16)), grp = (int)(i % (k / 16));
    const int t = row / 16, r = row % 16, g = r & 7, hi = r >> 3;
    const int b = grp / 4, j = grp % 4;
    const uint8_t* blk = src + ((int64_t)t * blocks + b) * kBlockBytes;
    scales[i] = blk[512 + g * 8 + 2 * j + hi];
    for (int q = 0; q < 8; ++q) {
      const int tq = q & 3, part = hi + ((q >> 2) << 1);
      codes[(int64_t)row * (k / 2) + grp * 8 + q] = blk[(g * 4 + tq) * 16 + 4 * j + part];
    }
  }
  (void)tiles;
}

void unpack_nvfp4(const uint8_t* src, int n_out, int k, uint8_t* codes, uint8_t* scales, cudaStream_t s) {
  const int tiles = packed_tiles(n_out, false), blocks = packed_blocks(k);
  const int64_t total = (int64_t)n_out * (k / 16);
  unpack_nvfp4_kernel<<<grid_for(total, 256), 256, 0, s>>>(src, n_out, k, tiles, blocks, codes, scales);
  XTG_CUDA(cudaGetLastError());
}

}  // namespace xtg
