// Per-row sampling parameters shared by the sampling kernels (csrc/kernels/sampling.h) and the host
// code that fills them (the native serving loop); no CUDA dependency.
#pragma once
#include <stdint.h>

namespace vmc {

// 40 bytes, mirrored by a numpy structured dtype on the host (vm_c_b200/core/engine.py SAMPLE_DTYPE).
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

}  // namespace vmc
