// Host interface of the sampling kernels (sampling.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

// Per-row sampling parameters (32 bytes, mirrored by a numpy structured dtype on the host).
struct SampleParams {
  float temperature;       // <= 0: greedy
  int32_t top_k;           // <= 0: disabled
  float top_p;             // >= 1: disabled
  float min_p;             // <= 0: disabled
  float repetition_penalty;
  float frequency_penalty;
  float presence_penalty;
  int32_t step;            // per-request RNG step counter
  uint64_t seed;
};
static_assert(sizeof(SampleParams) == 40, "SampleParams layout");

void sample(const float* logits, int S, int V, int64_t ld, const SampleParams* params, int32_t* out_tok, float* out_lp,
            cudaStream_t st);
void apply_penalties(float* logits, int64_t ld, const int32_t* row_of, const int32_t* tok, const int32_t* out_count,
                     const SampleParams* params, int n, cudaStream_t st);

}  // namespace vmc
