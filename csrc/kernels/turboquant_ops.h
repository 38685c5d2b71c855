// Host interface of the TurboQuant store kernel (turboquant.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "turboquant_types.h"

namespace vmc {

// RoPE on Q/K, then: Q heads rotated (the same per-KV-head rotation as their keys) and written
// bf16 to q_out [T, Hq, D]; K / V heads quantised into the TurboQuant slots of the token's cache
// slot (skipped when slot < 0). qkv as in rope_store (bf16, or fp32 split-K partials).
void rope_store_tq(const void* qkv, bool qkv_f32, int nsplit, int64_t split_stride, int T, int Hq, int Hkv, int D,
                   const int32_t* pos, const int32_t* slots, const float* cos_sin, bool neox, void* q_out,
                   const TqDev& tq, cudaStream_t st);

}  // namespace vmc
