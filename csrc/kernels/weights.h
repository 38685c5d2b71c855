// Host interface of the load-time weight kernels (weights.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

// Bytes of a tiled weight [N, K] in format `wf` (N padded to 128, K to the format's chunk).
int64_t tiled_weight_bytes(int wf, int N, int K);
// Convert GGUF rows (`src_type` = GGUF type id: 0 F32, 1 F16, 30 BF16, 8 Q8_0, 12 Q4_K, 14 Q6_K)
// into the tiled format `wf`.
void repack_weight(int wf, int src_type, const void* src, int N, int K, void* dst, cudaStream_t st);
// Inverse of the bf16 tiling (tests / diagnostics).
void untile_bf16(const void* tiles, int N, int K, void* out, cudaStream_t st);
// Quantise n floats into GGUF blocks of type gtype (8 Q8_0, 12 Q4_K, 14 Q6_K) on the device.
void quantize_blocks(int gtype, const float* x, int64_t n, void* out, cudaStream_t st);

}  // namespace vmc
