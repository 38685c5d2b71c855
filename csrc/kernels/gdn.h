// Host interface of the gated delta-net kernels (gdn.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

// Causal depthwise conv (kernel K along time, per channel) + SiLU over x [T, C] (row stride
// x_stride) for nseq sequences of tokens [q_start[s], q_start[s+1]); conv_state [slots, K-1, C]
// holds each sequence's last K-1 inputs (read when has_state[s], always written back).
void gdn_conv(const float* x, int64_t x_stride, const float* w, int C, int K, const int32_t* q_start,
              const int32_t* slot, const int32_t* has_state, int nseq, float* conv_state, float* y, int64_t y_stride,
              cudaStream_t st);

struct GdnArgs {
  const float* qkv;  // conv output [T, 2*Hk*D + Hv*D]: q heads | k heads | v heads
  int64_t qkv_stride;
  const float* alpha;  // [T, Hv] raw gate projection
  const float* beta;   // [T, Hv] raw beta projection
  int64_t ab_stride;
  const float* z;  // [T, Hv*D] output gate
  int64_t z_stride;
  const float* a_neg;    // [Hv] = -exp(A_log)
  const float* dt_bias;  // [Hv]
  const float* norm_w;   // [D]
  float* state;          // [slots, Hv, D, D] fp32, key index major
  const int32_t* slot;
  const int32_t* has_state;
  const int32_t* q_start;
  __nv_bfloat16* out;  // [T, Hv*D] rmsnorm(o) * norm_w * silu(z)
  int64_t out_stride;
  int Hk, Hv, D;
  float eps;  // l2-norm floor of q/k and RMSNorm epsilon
};

void gdn_recurrent(const GdnArgs& a, int nseq, cudaStream_t st);

}  // namespace vmc
