// Gated delta-net (GDN) linear attention of hybrid Qwen3.5-MoE layers: causal depthwise conv + SiLU
// over the mixed q|k|v channels, and the gated delta-rule recurrence with its gated RMSNorm.
//
// Reference behaviour: src/official/llama/models/qwen35moe.cpp:398-530 (build_layer_attn_linear:
// conv state, ssm_conv, SiLU, q/k l2 norms, key heads tiled over value heads by ggml_repeat_4d,
// gate = ssm_a * softplus(alpha + dt_bias), beta = sigmoid, gated norm, ssm_out) and
// src/official/llama/models/delta-net-base.cpp:289-363 (one recurrence step: S *= exp(g);
// d = beta * (v - S^T k); S += k d^T; o = S^T q with q scaled by 1/sqrt(Dk)).
//
// Design. Every value column j of a head's state S[Dk][Dv] evolves on its own once q and k are
// known, so one CTA owns one (sequence, value head) with 4 threads per column: a thread keeps
// Dk/4 entries of its column in registers for the whole sequence, the two column dot products are
// reduced with two warp shuffles, and the state crosses HBM once per call (read at the start,
// written at the end) instead of once per token. The next token's inputs are loaded into
// registers while the current token is computed. The gated RMSNorm over the head's Dv outputs
// (rmsnorm(o) * w * silu(z)) is the epilogue of each token. Prefill runs the same recurrence
// token by token (a chunked tensor-core form is a separate kernel).
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "gdn.h"

namespace vmc {
namespace {

constexpr int kConvMaxK = 8;

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

// y[t, c] = silu(sum_j w[c, j] * xin[t - K + 1 + j, c]), where rows before the sequence's first
// token come from its conv state (the last K-1 inputs of earlier calls; zeros for a new sequence).
// The state then holds the last K-1 inputs. One thread per (sequence, channel).
__global__ void gdn_conv_kernel(const float* __restrict__ x, int64_t x_stride, const float* __restrict__ w, int C,
                                int K, const int32_t* __restrict__ q_start, const int32_t* __restrict__ slot,
                                const int32_t* __restrict__ has_state, float* __restrict__ conv_state,
                                float* __restrict__ y, int64_t y_stride) {
  pdl_wait();
  const int s = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int t0 = q_start[s], t1 = q_start[s + 1];
  float* st = conv_state + static_cast<int64_t>(slot[s]) * (K - 1) * C;
  float hist[kConvMaxK];  // hist[0..K-2]: oldest .. newest
  float wc[kConvMaxK];
#pragma unroll
  for (int j = 0; j < kConvMaxK; ++j) {
    wc[j] = j < K ? w[static_cast<int64_t>(c) * K + j] : 0.f;
    hist[j] = (j < K - 1 && has_state[s]) ? st[static_cast<int64_t>(j) * C + c] : 0.f;
  }
  for (int t = t0; t < t1; ++t) {
    const float xt = x[static_cast<int64_t>(t) * x_stride + c];
    float acc = wc[K - 1] * xt;
#pragma unroll
    for (int j = 0; j < kConvMaxK - 1; ++j)
      if (j < K - 1) acc += wc[j] * hist[j];
    y[static_cast<int64_t>(t) * y_stride + c] = silu(acc);
#pragma unroll
    for (int j = 0; j < kConvMaxK - 1; ++j)
      if (j < K - 2) hist[j] = hist[j + 1];
    if (K >= 2) hist[K - 2] = xt;
  }
#pragma unroll
  for (int j = 0; j < kConvMaxK - 1; ++j)
    if (j < K - 1) st[static_cast<int64_t>(j) * C + c] = hist[j];
  pdl_trigger();
}

struct TokIn {
  float q, k, v, z, alpha, beta;
};

template <int DK>
__global__ void __launch_bounds__(4 * DK, 1)
    gdn_recurrent_kernel(GdnArgs a) {
  constexpr int DV = DK;
  constexpr int NT = 4 * DV;
  constexpr int RPT = DK / 4;  // state rows per thread
  constexpr int NW = NT / 32;
  __shared__ float sq[DK], sk[DK];
  __shared__ float red[3][NW];

  pdl_wait();
  const int h = blockIdx.x, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = lane >> 3;                // row phase 0..3: rows r, r + 4, ...
  const int j = warp * 8 + (lane & 7);    // value column
  const int kh = h % a.Hk;                // key head tiled over value heads (ggml_repeat_4d)
  const int t0 = a.q_start[s], t1 = a.q_start[s + 1];
  float* S = a.state + (static_cast<int64_t>(a.slot[s]) * a.Hv + h) * DK * DV;
  float st[RPT];
  const bool init = a.has_state[s] != 0;
#pragma unroll
  for (int ii = 0; ii < RPT; ++ii) st[ii] = init ? S[(ii * 4 + r) * DV + j] : 0.f;

  const float a_neg = a.a_neg[h], dt_bias = a.dt_bias[h], nw = a.norm_w[j];
  const float qscale = rsqrtf(static_cast<float>(DK));
  const int64_t qoff = static_cast<int64_t>(kh) * DK, koff = static_cast<int64_t>(a.Hk + kh) * DK,
                voff = static_cast<int64_t>(2 * a.Hk) * DK + static_cast<int64_t>(h) * DV;
  auto load = [&](int t) {
    TokIn in;
    const float* row = a.qkv + static_cast<int64_t>(t) * a.qkv_stride;
    in.q = tid < DK ? row[qoff + tid] : 0.f;
    in.k = (tid >= DK && tid < 2 * DK) ? row[koff + tid - DK] : 0.f;
    in.v = row[voff + j];
    in.z = a.z[static_cast<int64_t>(t) * a.z_stride + static_cast<int64_t>(h) * DV + j];
    in.alpha = a.alpha[static_cast<int64_t>(t) * a.ab_stride + h];
    in.beta = a.beta[static_cast<int64_t>(t) * a.ab_stride + h];
    return in;
  };
  TokIn cur = t0 < t1 ? load(t0) : TokIn{};
  for (int t = t0; t < t1; ++t) {
    TokIn nxt = t + 1 < t1 ? load(t + 1) : TokIn{};
    // l2 norms of q (threads 0..DK-1) and k (threads DK..2DK-1): one value per thread.
    float qq = cur.q * cur.q, kk = cur.k * cur.k;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      qq += __shfl_xor_sync(0xffffffffu, qq, o);
      kk += __shfl_xor_sync(0xffffffffu, kk, o);
    }
    if (lane == 0) {
      red[0][warp] = qq;
      red[1][warp] = kk;
    }
    __syncthreads();
    float qs = 0.f, ks = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      qs += red[0][w];
      ks += red[1][w];
    }
    if (tid < DK) sq[tid] = cur.q * qscale / fmaxf(sqrtf(qs), a.eps);
    else if (tid < 2 * DK) sk[tid - DK] = cur.k / fmaxf(sqrtf(ks), a.eps);
    __syncthreads();
    const float g = __expf(a_neg * softplus(cur.alpha + dt_bias));
    const float beta = 1.f / (1.f + __expf(-cur.beta));
    float p = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPT; ++ii) p += st[ii] * sk[ii * 4 + r];
    p += __shfl_xor_sync(0xffffffffu, p, 8);
    p += __shfl_xor_sync(0xffffffffu, p, 16);
    const float d = beta * (cur.v - g * p);
    float o = 0.f;
#pragma unroll
    for (int ii = 0; ii < RPT; ++ii) {
      st[ii] = g * st[ii] + sk[ii * 4 + r] * d;
      o += st[ii] * sq[ii * 4 + r];
    }
    o += __shfl_xor_sync(0xffffffffu, o, 8);
    o += __shfl_xor_sync(0xffffffffu, o, 16);
    // Gated RMSNorm over the head's DV outputs (each column counted once: lanes with r == 0).
    float oo = r == 0 ? o * o : 0.f;
#pragma unroll
    for (int off = 16; off; off >>= 1) oo += __shfl_xor_sync(0xffffffffu, oo, off);
    if (lane == 0) red[2][warp] = oo;
    __syncthreads();
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) ss += red[2][w];
    if (r == 0) {
      const float y = o * rsqrtf(ss / DV + a.eps) * nw * silu(cur.z);
      a.out[static_cast<int64_t>(t) * a.out_stride + static_cast<int64_t>(h) * DV + j] = __float2bfloat16(y);
    }
    cur = nxt;
    // red[] and sq/sk are rewritten by the next token only after its first barrier.
  }
#pragma unroll
  for (int ii = 0; ii < RPT; ++ii) S[(ii * 4 + r) * DV + j] = st[ii];
  pdl_trigger();
}

}  // namespace

void gdn_conv(const float* x, int64_t x_stride, const float* w, int C, int K, const int32_t* q_start,
              const int32_t* slot, const int32_t* has_state, int nseq, float* conv_state, float* y, int64_t y_stride,
              cudaStream_t st) {
  VMC_CHECK(K >= 2 && K <= kConvMaxK, "gdn_conv: kernel size must be in [2, 8]");
  if (nseq <= 0) return;
  launch_k(gdn_conv_kernel, dim3((C + 127) / 128, nseq), dim3(128), 0, st, x, x_stride, w, C, K, q_start, slot,
           has_state, conv_state, y, y_stride);
}

void gdn_recurrent(const GdnArgs& a, int nseq, cudaStream_t st) {
  VMC_CHECK(a.Hv % a.Hk == 0, "gdn_recurrent: value heads must be a multiple of key heads");
  if (nseq <= 0) return;
  switch (a.D) {
    case 64: launch_k(gdn_recurrent_kernel<64>, dim3(a.Hv, nseq), dim3(256), 0, st, a); break;
    case 128: launch_k(gdn_recurrent_kernel<128>, dim3(a.Hv, nseq), dim3(512), 0, st, a); break;
    default: VMC_CHECK(false, "gdn_recurrent: head dim must be 64 or 128");
  }
}

}  // namespace vmc
