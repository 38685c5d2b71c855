// GPU sampling: penalties, greedy argmax, and seeded top-k / top-p / min-p / temperature sampling.
//
// Covers the reference's sampler kernels (src/cuda/sampler_kernels.cu: apply_penalties_kernel :193,
// greedy_sampling_kernel :237, full_multinomial_sampling_kernel :256, filtered_sampling_kernel
// :280) with per-request seeds instead of the reference's fixed seed 0 (src/core/engine.cpp:1146).
//
//  * greedy rows: block-wide argmax and log-softmax of the chosen token.
//  * unrestricted rows (top_k = 0, top_p = 1, min_p = 0): exact softmax sampling by the Gumbel-max
//    trick, argmax(x/T + G_i), with G_i from a counter-based Philox4x32-10 stream (Salmon et al.,
//    "Parallel Random Numbers: As Easy as 1, 2, 3", SC 2011) keyed by the request seed and its step.
//  * restricted rows: exact k-th largest threshold by a 3-pass radix select (12+12+8 bits of the
//    order-preserving key), candidate gather (<= 1024), bitonic sort in shared memory, then
//    top-p / min-p cut-offs on the sorted candidates and inverse-CDF sampling with one uniform.
#include "common.cuh"
#include "sampling.h"

namespace vmc {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxCand = 1024;

__device__ __forceinline__ uint32_t mulhi32(uint32_t a, uint32_t b) { return __umulhi(a, b); }

// Philox4x32 with 10 rounds.
__device__ __forceinline__ uint4 philox(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = mulhi32(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = mulhi32(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}
__device__ __forceinline__ float u01_open(uint32_t x) { return (static_cast<float>(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ ArgMax block_argmax(ArgMax a, ArgMax* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = a;
  __syncthreads();
  if (w == 0) {
    a = (threadIdx.x < nw) ? sh[threadIdx.x] : ArgMax{-INFINITY, 0x7fffffff};
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
      a = better(a, b);
    }
    if (threadIdx.x == 0) sh[0] = a;
  }
  __syncthreads();
  return sh[0];
}

__device__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (threadIdx.x < nw) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

// Find the k-th largest order key among x[0..V) (1-based k <= V).
__device__ uint32_t radix_kth_largest(const float* x, int V, int k, uint32_t* hist) {
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  const int shifts[3] = {20, 8, 0};
  const int widths[3] = {12, 12, 8};
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass], nb = 1 << widths[pass];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const uint32_t key = order_key(x[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> sh) & (nb - 1)], 1u);
    }
    __syncthreads();
    // Scan bins from the top (one thread; at most 4096 bins).
    __shared__ int sel_bin, sel_rem;
    if (threadIdx.x == 0) {
      int rem = remaining, b = nb - 1;
      for (; b > 0; --b) {
        const int c = static_cast<int>(hist[b]);
        if (c >= rem) break;
        rem -= c;
      }
      sel_bin = b;
      sel_rem = rem;
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(sel_bin) << sh;
    mask |= static_cast<uint32_t>(nb - 1) << sh;
    remaining = sel_rem;
    __syncthreads();
  }
  return prefix;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const float* __restrict__ logits, int V, int64_t ld,
                                                          const SampleParams* __restrict__ params,
                                                          int32_t* __restrict__ out_tok, float* __restrict__ out_lp) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float* x = logits + row * ld;
  const SampleParams sp = params[row];
  __shared__ ArgMax sh_am[32];
  __shared__ float sh_f[32];
  __shared__ uint32_t hist[4096];
  __shared__ float cand_v[kMaxCand];
  __shared__ int cand_i[kMaxCand];
  __shared__ int n_cand;

  // Two passes over the row (the second hits L1/L2): the argmax (independent compares, four
  // running maxima per thread), then the sum of exponentials against the row maximum, giving the
  // raw log-softmax normaliser (the reported logprob) and the greedy choice.
  const bool vec = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  ArgMax b4[4] = {{-INFINITY, 0x7fffffff}, {-INFINITY, 0x7fffffff}, {-INFINITY, 0x7fffffff}, {-INFINITY, 0x7fffffff}};
  if (vec) {
    // eight loads in flight per thread: one outstanding 16-byte load per thread left a 64-row
    // batch latency-bound at ~15 GB/s per SM
    const int step = blockDim.x * 4;
    int i = threadIdx.x * 4;
    for (; i + 7 * step < V; i += 8 * step) {
      float4 q[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) q[u] = __ldg(reinterpret_cast<const float4*>(x + i + u * step));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = i + u * step;
        if (q[u].x > b4[0].v) b4[0] = ArgMax{q[u].x, j};
        if (q[u].y > b4[1].v) b4[1] = ArgMax{q[u].y, j + 1};
        if (q[u].z > b4[2].v) b4[2] = ArgMax{q[u].z, j + 2};
        if (q[u].w > b4[3].v) b4[3] = ArgMax{q[u].w, j + 3};
      }
    }
    for (; i < V; i += step) {
      const float4 q = *reinterpret_cast<const float4*>(x + i);
      if (q.x > b4[0].v) b4[0] = ArgMax{q.x, i};
      if (q.y > b4[1].v) b4[1] = ArgMax{q.y, i + 1};
      if (q.z > b4[2].v) b4[2] = ArgMax{q.z, i + 2};
      if (q.w > b4[3].v) b4[3] = ArgMax{q.w, i + 3};
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x)
      if (x[i] > b4[0].v) b4[0] = ArgMax{x[i], i};
  }
  const ArgMax am = block_argmax(better(better(b4[0], b4[1]), better(b4[2], b4[3])), sh_am);
  const float lmax = am.v;
  float lsum = 0.f;
  if (lmax != -INFINITY) {
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec) {
      const int step = blockDim.x * 4;
      int i = threadIdx.x * 4;
      for (; i + 3 * step < V; i += 4 * step) {
        float4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = __ldg(reinterpret_cast<const float4*>(x + i + u * step));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          s4[0] += __expf(q[u].x - lmax);
          s4[1] += __expf(q[u].y - lmax);
          s4[2] += __expf(q[u].z - lmax);
          s4[3] += __expf(q[u].w - lmax);
        }
      }
      for (; i < V; i += step) {
        const float4 q = *reinterpret_cast<const float4*>(x + i);
        s4[0] += __expf(q.x - lmax);
        s4[1] += __expf(q.y - lmax);
        s4[2] += __expf(q.z - lmax);
        s4[3] += __expf(q.w - lmax);
      }
    } else {
      for (int i = threadIdx.x; i < V; i += blockDim.x) s4[0] += __expf(x[i] - lmax);
    }
    lsum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  }
  lsum = block_sum(lsum, sh_f);
  const float log_z = lmax + __logf(lsum);

  const bool greedy = sp.temperature <= 0.f || sp.top_k == 1;
  int chosen;
  if (greedy) {
    chosen = am.i;
  } else {
    const float inv_t = 1.f / sp.temperature;
    const uint2 key = make_uint2(static_cast<uint32_t>(sp.seed), static_cast<uint32_t>(sp.seed >> 32));
    const bool unrestricted = sp.top_k <= 0 && sp.top_p >= 1.f && sp.min_p <= 0.f;
    if (unrestricted) {
      ArgMax a{-INFINITY, 0x7fffffff};
      for (int base = threadIdx.x * 4; base < V; base += blockDim.x * 4) {
        const uint4 rnd = philox(make_uint4(static_cast<uint32_t>(base), static_cast<uint32_t>(sp.step), 0x5a4d1u, 0u), key);
        const uint32_t rr[4] = {rnd.x, rnd.y, rnd.z, rnd.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = base + j;
          if (i < V) {
            const float g = -__logf(-__logf(u01_open(rr[j])));
            a = better(a, ArgMax{x[i] * inv_t + g, i});
          }
        }
      }
      chosen = block_argmax(a, sh_am).i;
    } else {
      int k = sp.top_k > 0 ? min(sp.top_k, kMaxCand) : kMaxCand;
      k = min(k, V);
      const uint32_t thr = radix_kth_largest(x, V, k, hist);
      if (threadIdx.x == 0) n_cand = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        if (order_key(x[i]) >= thr) {
          const int slot = atomicAdd(&n_cand, 1);
          if (slot < kMaxCand) {
            cand_v[slot] = x[i];
            cand_i[slot] = i;
          }
        }
      }
      __syncthreads();
      const int n = min(n_cand, kMaxCand);
      for (int i = n + threadIdx.x; i < kMaxCand; i += blockDim.x) {
        cand_v[i] = -INFINITY;
        cand_i[i] = 0x7fffffff;
      }
      __syncthreads();
      // Bitonic sort, descending by value (ties: lower index first).
      for (int size = 2; size <= kMaxCand; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          const int i = threadIdx.x;
          const int j = i ^ stride;
          if (j > i) {
            const bool desc = (i & size) == 0;
            const float vi = cand_v[i], vj = cand_v[j];
            const int ii = cand_i[i], ij = cand_i[j];
            const bool i_first = vi > vj || (vi == vj && ii < ij);
            if (desc != i_first) {
              cand_v[i] = vj; cand_v[j] = vi;
              cand_i[i] = ij; cand_i[j] = ii;
            }
          }
          __syncthreads();
        }
      }
      if (threadIdx.x == 0) {
        // Softmax over the top-k set at temperature T, then top-p and min-p cut-offs.
        const float m0 = cand_v[0] * inv_t;
        float z = 0.f;
        for (int i = 0; i < min(n, k); ++i) z += __expf(cand_v[i] * inv_t - m0);
        int keep = min(n, k);
        if (sp.top_p < 1.f) {
          float c = 0.f;
          for (int i = 0; i < keep; ++i) {
            c += __expf(cand_v[i] * inv_t - m0) / z;
            if (c >= sp.top_p) { keep = i + 1; break; }
          }
        }
        if (sp.min_p > 0.f) {
          const float cut = logf(sp.min_p);  // p_i / p_max >= min_p
          int kk = 1;
          while (kk < keep && cand_v[kk] * inv_t - m0 >= cut) ++kk;
          keep = kk;
        }
        float zz = 0.f;
        for (int i = 0; i < keep; ++i) zz += __expf(cand_v[i] * inv_t - m0);
        const uint4 rnd = philox(make_uint4(0xffffffffu, static_cast<uint32_t>(sp.step), 0x5a4d2u, 0u), key);
        const float u = u01_open(rnd.x) * zz;
        float c = 0.f;
        int pick = keep - 1;
        for (int i = 0; i < keep; ++i) {
          c += __expf(cand_v[i] * inv_t - m0);
          if (c >= u) { pick = i; break; }
        }
        n_cand = cand_i[pick];
      }
      __syncthreads();
      chosen = n_cand;
    }
  }
  if (threadIdx.x == 0) {
    out_tok[row] = chosen;
    if (out_lp) out_lp[row] = x[chosen] - log_z;
  }
}

// One thread per (row, token) penalty entry.
__global__ void penalties_kernel(float* __restrict__ logits, int64_t ld, const int32_t* __restrict__ row_of,
                                 const int32_t* __restrict__ tok, const int32_t* __restrict__ out_count,
                                 const SampleParams* __restrict__ params, int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = row_of[i];
  const SampleParams sp = params[r];
  float* p = logits + r * ld + tok[i];
  float v = *p;
  if (sp.repetition_penalty != 1.f) v = v > 0.f ? v / sp.repetition_penalty : v * sp.repetition_penalty;
  const int c = out_count[i];
  if (c > 0) v -= sp.frequency_penalty * c + sp.presence_penalty;
  *p = v;
}

}  // namespace

void sample(const float* logits, int S, int V, int64_t ld, const SampleParams* params, int32_t* out_tok, float* out_lp,
            cudaStream_t st) {
  if (S <= 0) return;
  launch_k(sample_kernel, dim3(S), dim3(kThreads), 0, st, logits, V, ld, params, out_tok, out_lp);
}

void apply_penalties(float* logits, int64_t ld, const int32_t* row_of, const int32_t* tok, const int32_t* out_count,
                     const SampleParams* params, int n, cudaStream_t st) {
  if (n <= 0) return;
  launch_k(penalties_kernel, dim3((n + 255) / 256), dim3(256), 0, st, logits, ld, row_of, tok, out_count, params, n);
}

}  // namespace vmc
