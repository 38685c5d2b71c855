// Host interface of the per-layer elementwise kernels (layers.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

// resid[t, :] (fp32) and/or out_bf16[t, :] = dequantised GGUF row ids[t] of `table`.
void embed(const int32_t* ids, int T, const void* table, int gtype, int64_t row_bytes, int H, float* resid,
           void* out_bf16, cudaStream_t st);
// resid += sum_j delta[j] (ndelta slices delta_stride elements apart); out = rmsnorm(resid) * w.
void add_rmsnorm(float* resid, const void* delta, bool delta_f32, int ndelta, int64_t delta_stride, const float* w,
                 int T, int H, float eps, void* out, cudaStream_t st);
// RoPE on Q/K heads of qkv [T, (Hq+2Hkv)*D]; Q -> q_out, K/V -> paged cache at slots[t].
// qkv may be nsplit fp32 per-split partials `split_stride` elements apart (split-K GEMM output).
void rope_store(const void* qkv, bool qkv_f32, int nsplit, int64_t split_stride, int T, int Hq, int Hkv, int D,
                const int32_t* pos, const int32_t* slots, const float* cos_sin, bool neox, void* q_out, void* kv,
                cudaStream_t st);
void swiglu(const void* gu, bool f32, int nsplit, int64_t split_stride, int64_t T, int F, bool interleaved, void* out,
            cudaStream_t st);
void gather_rows(const void* src, const int32_t* idx, int n, int H, void* dst, cudaStream_t st);
void f32_to_bf16(const float* x, int64_t n, void* y, cudaStream_t st);

}  // namespace vmc
