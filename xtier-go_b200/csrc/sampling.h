// Internal interface of the sampling kernels (sampling.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xtg {

constexpr int kMaxTopK = 1024;   // the sorted head Sampler::sample keeps for top_p / min_p (sampler.cpp:60)

// For rows x vocab f32 logits (vocab <= 131072): idx / val [rows][k] the k most likely entries, most likely first
// (ties: lowest index first), row_max [rows], total [rows] = sum_i exp((l_i - row_max) / T) (T <= 0: 1).
void launch_topk(const float* logits, int rows, int vocab, int k, float temperature, int32_t* idx, float* val,
                 float* row_max, double* total, cudaStream_t s);

}  // namespace xtg
