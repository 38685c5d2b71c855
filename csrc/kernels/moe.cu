// Mixture-of-experts routing and combine (Mixtral), around the grouped tcgen05 GEMM.
//
// Replaces the reference's MoE path: llama.cpp's build_moe_ffn (softmax router, top-k,
// renormalised weights, ggml_mul_mat_id per expert and a weighted sum; vendored
// src/llama-graph.cpp build_moe_ffn) followed by vm_c's TP all-reduce of the expert output
// (src/official/llama/models/llama.cpp:196). Here:
//
//  * moe_route_kernel (one CTA): per token, softmax over the E router logits, top-k experts
//    (ties -> lower id), weights renormalised to sum 1 when requested; then, for the experts this
//    rank holds ([e0, e0 + e_local): all of them with TP-sliced experts, a 1/ep share with expert
//    parallelism), a stable counting sort of the (token, slot) pairs by expert: per-expert row
//    counts and offsets, the source token of every sorted row, and each pair's sorted row (-1 when
//    its expert lives on another rank). Stable order keeps every rank's sums bit-identical.
//  * the caller gathers the token rows in sorted order and runs the grouped GEMMs
//    (gate/up with the fused SwiGLU epilogue, then down) over all local experts in one launch each;
//  * moe_combine_kernel: out[t] = sum_j w[t, j] * y[row(t, j)] over this rank's experts (fp32).
//    With TP attention the hidden states are replicated on every rank, so dispatch needs no
//    communication and the combine's cross-rank sum is the all-reduce that follows (fused with
//    the residual add and RMSNorm on the peer-memory path).
#include "common.cuh"
#include "moe.h"

namespace vmc {
namespace {

constexpr int kRouteThreads = 1024;
constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(MoeRouteArgs a) {
  __shared__ int s_warp[kRouteThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  // 1) softmax + top-k per token.
  for (int t = tid; t < a.T; t += blockDim.x) {
    const float* lg = a.logits + static_cast<int64_t>(t) * a.ld_logits;
    float mx = -INFINITY;
    for (int e = 0; e < a.E; ++e) mx = fmaxf(mx, lg[e]);
    float sum = 0.f;
    for (int e = 0; e < a.E; ++e) sum += __expf(lg[e] - mx);
    uint64_t taken = 0;
    float wsel[kMaxTopK];
    int isel[kMaxTopK];
    float wsum = 0.f;
    for (int j = 0; j < a.k; ++j) {
      int best = -1;
      float bv = -INFINITY;
      for (int e = 0; e < a.E; ++e) {
        if ((taken >> e) & 1ull) continue;
        if (best < 0 || lg[e] > bv) {
          best = e;
          bv = lg[e];
        }
      }
      taken |= 1ull << best;
      isel[j] = best;
      wsel[j] = __expf(bv - mx) / sum;
      wsum += wsel[j];
    }
    for (int j = 0; j < a.k; ++j) {
      a.topk_id[t * a.k + j] = isel[j];
      a.topk_w[t * a.k + j] = a.norm_topk ? wsel[j] / wsum : wsel[j];
    }
  }
  __syncthreads();
  // 2) stable counting sort of the local (token, slot) pairs by expert.
  const int n = a.T * a.k;
  const int lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x / 32;
  int base = 0;
  for (int el = 0; el < a.e_local; ++el) {
    const int e = a.e0 + el;
    int run = 0;  // rows of expert e so far
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
      const int i = i0 + tid;
      const bool mine = i < n && a.topk_id[i] == e;
      const unsigned bal = __ballot_sync(0xffffffffu, mine);
      if (lane == 0) s_warp[warp] = __popc(bal);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < nwarps; ++w) {
        const int c = s_warp[w];
        before += w < warp ? c : 0;
        total += c;
      }
      if (mine) {
        const int pos = base + run + before + __popc(bal & ((1u << lane) - 1u));
        a.sorted_src[pos] = i / a.k;
        a.slot_row[i] = pos;
      }
      run += total;
      __syncthreads();
    }
    if (tid == 0) {
      a.counts[el] = run;
      a.offsets[el] = base;
    }
    base += run;
  }
  // Pairs routed to other ranks, and the unused tail of the sorted rows (gathered but ignored).
  for (int i = tid; i < n; i += blockDim.x) {
    const int e = a.topk_id[i];
    if (e < a.e0 || e >= a.e0 + a.e_local) a.slot_row[i] = -1;
    if (i >= base) a.sorted_src[i] = 0;
  }
  if (tid == 0) *a.total_rows = base;
}

__global__ void moe_combine_kernel(const float* __restrict__ y, int ldy, const int32_t* __restrict__ slot_row,
                                   const float* __restrict__ topk_w, int T, int k, int H, float* __restrict__ out,
                                   int ldo) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  int rows[kMaxTopK];
  float ws[kMaxTopK];
  for (int j = 0; j < k; ++j) {
    rows[j] = slot_row[t * k + j];
    ws[j] = topk_w[t * k + j];
  }
  for (int h = threadIdx.x * 4; h < H; h += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      if (rows[j] < 0) continue;
      const float4 v = *reinterpret_cast<const float4*>(y + static_cast<int64_t>(rows[j]) * ldy + h);
      acc.x += ws[j] * v.x;
      acc.y += ws[j] * v.y;
      acc.z += ws[j] * v.z;
      acc.w += ws[j] * v.w;
    }
    *reinterpret_cast<float4*>(out + static_cast<int64_t>(t) * ldo + h) = acc;
  }
}

}  // namespace

void moe_route(const MoeRouteArgs& a, cudaStream_t st) {
  VMC_CHECK(a.E >= 1 && a.E <= kMaxExperts, "moe_route: 1..64 experts");
  VMC_CHECK(a.k >= 1 && a.k <= kMaxTopK && a.k <= a.E, "moe_route: top-k must be in 1..min(8, E)");
  VMC_CHECK(a.e0 >= 0 && a.e_local >= 1 && a.e0 + a.e_local <= a.E, "moe_route: bad local expert range");
  if (a.T <= 0) return;
  launch_k(moe_route_kernel, dim3(1), dim3(kRouteThreads), 0, st, a);
}

void moe_combine(const float* y, int ldy, const int32_t* slot_row, const float* topk_w, int T, int k, int H,
                 float* out, int ldo, cudaStream_t st) {
  VMC_CHECK(H % 4 == 0 && ldy % 4 == 0 && ldo % 4 == 0, "moe_combine: hidden size must be a multiple of 4");
  VMC_CHECK(k >= 1 && k <= kMaxTopK, "moe_combine: top-k must be in 1..8");
  if (T <= 0) return;
  launch_k(moe_combine_kernel, dim3(T), dim3(256), 0, st, y, ldy, slot_row, topk_w, T, k, H, out, ldo);
}


// ---- expert-parallel dispatch ------------------------------------------------------------------

namespace {

__global__ void __launch_bounds__(256) moe_dispatch_kernel(MoeDispatchArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row < a.rows) {
    const float lg = lane < a.E ? a.logits[static_cast<size_t>(row) * a.ld_logits + lane] : -INFINITY;
    const float mx = warp_max(lg);
    const float ex = lane < a.E ? __expf(lg - mx) : 0.f;
    const float sum = warp_sum(ex);
    uint32_t taken = 0;
    int isel[kMaxTopK];
    float wsel[kMaxTopK];
    float wsum = 0.f;
    for (int j = 0; j < a.k; ++j) {
      // warp argmax over the untaken experts, ties to the lower id (as moe_route)
      float v = (lane < a.E && !((taken >> lane) & 1u)) ? lg : -INFINITY;
      int id = lane < a.E && !((taken >> lane) & 1u) ? lane : 0x7fffffff;
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, id, o);
        if (v2 > v || (v2 == v && i2 < id)) {
          v = v2;
          id = i2;
        }
      }
      isel[j] = id;
      wsel[j] = __shfl_sync(0xffffffffu, ex, id) / sum;
      wsum += wsel[j];
      taken |= 1u << id;
    }
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.x) + static_cast<size_t>(row) * a.H);
    for (int j = 0; j < a.k; ++j) {
      const int e = isel[j];
      const int o = e / a.e_local, le = e - o * a.e_local;
      uint32_t slot = 0;
      if (lane == 0) slot = atomicAdd_system(a.cnt[o] + le, 1u);
      slot = __shfl_sync(0xffffffffu, slot, 0);
      if (slot < static_cast<uint32_t>(a.cap)) {
        const size_t dst_row = static_cast<size_t>(le) * a.cap + slot;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.recv_x[o]) + dst_row * a.H);
        for (int i = lane; i < a.H / 8; i += 32) dst[i] = src[i];
        if (lane == 0) a.recv_ret[o][dst_row] = (a.rank << 24) | (row << 3) | j;
      } else if (lane == 0) {
        atomicCAS(a.err, 0u, static_cast<uint32_t>(kErrCommWait));
      }
      if (lane == 0) a.topk_w[static_cast<size_t>(row) * a.k + j] = a.norm_topk ? wsel[j] / wsum : wsel[j];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    sys_fence();
    for (int q = 0; q < a.nranks; ++q) sys_count(a.arrive[q], 1u);
    const uint32_t G = gridDim.x;
    if (blockIdx.x == 0) sys_wait(a.arrive[a.rank], a.state[0] + a.nranks * G, a.err, kErrCommWait);
    if (atomicAdd(a.state + 1, 1u) == G - 1) {
      a.state[0] += a.nranks * G;
      a.state[1] = 0;
      __threadfence();
    }
  }
}

}  // namespace

void moe_dispatch(const MoeDispatchArgs& a, cudaStream_t st) {
  VMC_CHECK(a.E >= 1 && a.E <= 32, "moe_dispatch: at most 32 experts (one lane each)");
  VMC_CHECK(a.k >= 1 && a.k <= kMaxTopK && a.k <= a.E, "moe_dispatch: bad top-k");
  VMC_CHECK(a.H % 8 == 0 && a.nranks >= 1 && a.nranks <= 8 && a.e_local >= 1, "moe_dispatch: bad shape");
  VMC_CHECK(a.rpr < (1 << 21), "moe_dispatch: too many rows per rank for the return word");
  launch_k(moe_dispatch_kernel, dim3(moe_dispatch_ctas(a.rpr)), dim3(256), 0, st, a);
}

}  // namespace vmc
