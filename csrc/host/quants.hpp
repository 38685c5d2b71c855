// CPU codecs for GGUF block-quantised tensors.
//
// Dequantisers cover the same formats as the reference's CPU dequant
// (src/core/ggml_dequant.cpp: dequantize_row_q4_0/q4_1/q5_0/q5_1/q8_0 at :109, q2_K..q6_K at
// :199/:252, q8_K, iq4_xs). They are the numerical oracle for the GPU kernels and the load-time
// path for formats that have no native GPU GEMM. The quantisers (Q8_0, Q4_0, Q4_K, Q6_K) build
// the seeded random-init checkpoints; they use plain min/max rounding, not llama.cpp's search.
#pragma once
#include <cstddef>
#include <cstdint>

#include "ggml_types.hpp"

namespace vmc {

// Dequantise `n` elements (a multiple of the block size) of type `t` from `src` into `dst`.
void dequantize_row(GType t, const void* src, float* dst, int64_t n);
// Quantise `n` floats into blocks of type `t` (Q8_0, Q4_0, Q4_K, Q6_K, F16, BF16, F32).
void quantize_row(GType t, const float* src, void* dst, int64_t n);
bool can_quantize(GType t);

// Multi-threaded helpers over a 2-D tensor with `rows` rows of `row_elems` elements.
void dequantize_tensor(GType t, const void* src, float* dst, int64_t rows, int64_t row_elems, int threads);
void quantize_tensor(GType t, const float* src, void* dst, int64_t rows, int64_t row_elems, int threads);

// The non-linear 4-bit codebook of the IQ4_NL / IQ4_XS formats (part of the file format).
extern const int8_t kIQ4NLValues[16];

}  // namespace vmc
