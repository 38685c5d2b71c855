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

// Restricted sampling over n candidates (cand_v / cand_i in shared memory, unsorted, n <= kMaxCand):
// pad, bitonic sort (descending value, ties by lower index), keep the top k, softmax over them at
// temperature 1/inv_t, top-p then min-p cut-offs, inverse-CDF draw with the row's Philox uniform.
// Every thread of the block must call it; returns the chosen token id.
__device__ int pick_restricted(float* cand_v, int* cand_i, int n, int k, const SampleParams& sp, float inv_t,
                               uint2 key, int* sh_out) {
  for (int i = n + threadIdx.x; i < kMaxCand; i += blockDim.x) {
    cand_v[i] = -INFINITY;
    cand_i[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= kMaxCand; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const int i = threadIdx.x;
      const int j = i ^ stride;
      if (i < kMaxCand && j > i) {
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
    *sh_out = cand_i[pick];
  }
  __syncthreads();
  return *sh_out;
}

// Gumbel noise of vocabulary entry i (global index) for a row: the same value on every rank.
__device__ __forceinline__ float gumbel_at(int i, int step, uint2 key) {
  const uint4 rnd = philox(make_uint4(static_cast<uint32_t>(i & ~3), static_cast<uint32_t>(step), 0x5a4d1u, 0u), key);
  const uint32_t rr[4] = {rnd.x, rnd.y, rnd.z, rnd.w};
  return -__logf(-__logf(u01_open(rr[i & 3])));
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
      chosen = pick_restricted(cand_v, cand_i, min(n_cand, kMaxCand), k, sp, inv_t, key, &n_cand);
    }
  }
  if (threadIdx.x == 0) {
    out_tok[row] = chosen;
    if (out_lp) out_lp[row] = x[chosen] - log_z;
  }
}

// ---- vocabulary-parallel sampling ----------------------------------------------------------------
//
// Each rank holds logits of vocabulary entries [v0, v0 + V_local). tp_sample_local reduces its shard
// of every sampled row to: the row maximum and sum of exp(x - max) (for the log-probability), and a
// candidate list - the argmax (greedy rows), the Gumbel-perturbed argmax with noise drawn at the
// global index (unrestricted rows), or the local top-k by radix select (restricted rows, k capped at
// kMaxCand as in the single-GPU kernel) - and stores it into every rank's exchange buffer (peer
// memory), then releases it (system-scope fence) and counts one arrival at every rank.
// tp_sample_merge waits for all ranks' rows, merges the lists and picks exactly as sample_kernel
// would on the whole vocabulary (the global top-k is contained in the union of the local ones), so
// all ranks draw the same token without exchanging the logits themselves.

struct XHeader {   // per (source rank, row)
  float lmax;      // shard maximum
  float lsum;      // sum of exp(x - lmax) over the shard
  int n;           // candidates that follow
  float raw;       // unrestricted rows: raw logit of the perturbed winner
};
struct XCand {
  float v;
  int i;
};
constexpr int kXRowBytes = 16 + kMaxCand * 8;  // one (rank, row) slot of the exchange buffer

__device__ __forceinline__ void fence_acq_rel_sys_s() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_sys_s(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_s(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct TpSampleArgs {
  const float* logits;
  int V_local, v0;
  int64_t ld;
  const SampleParams* params;
  int S, rank, nranks;
  uint8_t* xbuf[8];      // every rank's exchange buffer [nranks][max_rows][kXRowBytes]
  int max_rows;
  uint32_t* count[8];    // every rank's arrival counter
  uint32_t* state;       // this rank's [0] target, [1] CTAs done
  int32_t* out_tok;
  float* out_lp;
  uint32_t* err;
};

__global__ void __launch_bounds__(kThreads) tp_sample_local_kernel(TpSampleArgs a) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float* x = a.logits + row * a.ld;
  const int V = a.V_local;
  const SampleParams sp = a.params[row];
  __shared__ ArgMax sh_am[32];
  __shared__ float sh_f[32];
  __shared__ uint32_t hist[4096];
  __shared__ int n_cand;
  ArgMax b{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x)
    if (x[i] > b.v) b = ArgMax{x[i], i};
  const ArgMax am = block_argmax(b, sh_am);
  float ls = 0.f;
  if (am.v != -INFINITY)
    for (int i = threadIdx.x; i < V; i += blockDim.x) ls += __expf(x[i] - am.v);
  ls = block_sum(ls, sh_f);
  const size_t slot = static_cast<size_t>(a.rank) * a.max_rows + row;
  const bool greedy = sp.temperature <= 0.f || sp.top_k == 1;
  const bool unrestricted = sp.top_k <= 0 && sp.top_p >= 1.f && sp.min_p <= 0.f;
  XHeader hd{am.v, ls, 1, am.v};
  if (greedy) {
    if (threadIdx.x == 0)
      for (int q = 0; q < a.nranks; ++q) {
        uint8_t* base = a.xbuf[q] + slot * kXRowBytes;
        *reinterpret_cast<XCand*>(base + 16) = XCand{am.v, a.v0 + am.i};
      }
  } else if (unrestricted) {
    const float inv_t = 1.f / sp.temperature;
    const uint2 key = make_uint2(static_cast<uint32_t>(sp.seed), static_cast<uint32_t>(sp.seed >> 32));
    ArgMax g{-INFINITY, 0x7fffffff};
    for (int i = threadIdx.x; i < V; i += blockDim.x) g = better(g, ArgMax{x[i] * inv_t + gumbel_at(a.v0 + i, sp.step, key), i});
    g = block_argmax(g, sh_am);
    hd.raw = x[g.i];
    if (threadIdx.x == 0)
      for (int q = 0; q < a.nranks; ++q)
        *reinterpret_cast<XCand*>(a.xbuf[q] + slot * kXRowBytes + 16) = XCand{g.v, a.v0 + g.i};
  } else {
    int k = sp.top_k > 0 ? min(sp.top_k, kMaxCand) : kMaxCand;
    k = min(k, V);
    const uint32_t thr = radix_kth_largest(x, V, k, hist);
    if (threadIdx.x == 0) n_cand = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      if (order_key(x[i]) >= thr) {
        const int c = atomicAdd(&n_cand, 1);
        if (c < kMaxCand)
          for (int q = 0; q < a.nranks; ++q)
            *reinterpret_cast<XCand*>(a.xbuf[q] + slot * kXRowBytes + 16 + 8 * c) = XCand{x[i], a.v0 + i};
      }
    }
    __syncthreads();
    hd.n = min(n_cand, kMaxCand);
  }
  if (threadIdx.x == 0)
    for (int q = 0; q < a.nranks; ++q) *reinterpret_cast<XHeader*>(a.xbuf[q] + slot * kXRowBytes) = hd;
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys_s();
    for (int q = 0; q < a.nranks; ++q) red_add_sys_s(a.count[q], 1u);
  }
}

__global__ void __launch_bounds__(kThreads) tp_sample_merge_kernel(TpSampleArgs a) {
  extern __shared__ __align__(16) uint8_t dyn[];
  float* all_v = reinterpret_cast<float*>(dyn);                 // [nranks * kMaxCand]
  int* all_i = reinterpret_cast<int*>(all_v + 8 * kMaxCand);
  __shared__ ArgMax sh_am[32];
  __shared__ uint32_t hist[4096];
  __shared__ float cand_v[kMaxCand];
  __shared__ int cand_i[kMaxCand];
  __shared__ int n_cand, ok;
  __shared__ XHeader hdr[8];
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, NR = a.nranks;
  const uint32_t target = a.state[0] + static_cast<uint32_t>(NR * a.S);
  if (threadIdx.x == 0) {
    int good = 0;
    const long long t0 = clock64();  // time bound (about 2 s of SM clock)
    for (uint32_t i = 0;; ++i) {
      if (static_cast<int32_t>(ld_acquire_sys_s(a.count[a.rank]) - target) >= 0) { good = 1; break; }
      if (clock64() - t0 > (4ll << 30)) { atomicCAS(a.err, 0u, static_cast<uint32_t>(kErrCommWait)); break; }
      if (i > 32) __nanosleep(64);
    }
    ok = good;
  }
  __syncthreads();
  const uint8_t* mine = a.xbuf[a.rank];
  if (ok) {
    if (threadIdx.x < NR)
      hdr[threadIdx.x] = *reinterpret_cast<const XHeader*>(mine + (static_cast<size_t>(threadIdx.x) * a.max_rows + row) * kXRowBytes);
    __syncthreads();
    float M = -INFINITY;
    for (int q = 0; q < NR; ++q) M = fmaxf(M, hdr[q].lmax);
    float Z = 0.f;
    for (int q = 0; q < NR; ++q)
      if (hdr[q].lmax != -INFINITY) Z += hdr[q].lsum * __expf(hdr[q].lmax - M);
    const float log_z = M + __logf(Z);
    const SampleParams sp = a.params[row];
    const bool greedy = sp.temperature <= 0.f || sp.top_k == 1;
    const bool unrestricted = sp.top_k <= 0 && sp.top_p >= 1.f && sp.min_p <= 0.f;
    int chosen = 0;
    float raw = 0.f;
    if (greedy || unrestricted) {
      if (threadIdx.x == 0) {
        ArgMax best{-INFINITY, 0x7fffffff};
        int from = 0;
        for (int q = 0; q < NR; ++q) {
          const XCand c = *reinterpret_cast<const XCand*>(mine + (static_cast<size_t>(q) * a.max_rows + row) * kXRowBytes + 16);
          const ArgMax nb = better(best, ArgMax{c.v, c.i});
          if (nb.i != best.i || nb.v != best.v) from = q;
          best = nb;
        }
        n_cand = best.i;
        cand_v[0] = greedy ? best.v : hdr[from].raw;
      }
      __syncthreads();
      chosen = n_cand;
      raw = cand_v[0];
    } else {
      // gather every rank's candidates, then the global top-k by radix select
      int total = 0;
      for (int q = 0; q < NR; ++q) {
        const int nq = hdr[q].n;
        const XCand* c = reinterpret_cast<const XCand*>(mine + (static_cast<size_t>(q) * a.max_rows + row) * kXRowBytes + 16);
        for (int j = threadIdx.x; j < nq; j += blockDim.x) {
          const XCand e = c[j];
          all_v[total + j] = e.v;
          all_i[total + j] = e.i;
        }
        total += nq;
      }
      __syncthreads();
      int k = sp.top_k > 0 ? min(sp.top_k, kMaxCand) : kMaxCand;
      k = min(k, total);
      const uint32_t thr = radix_kth_largest(all_v, total, k, hist);
      if (threadIdx.x == 0) n_cand = 0;
      __syncthreads();
      for (int j = threadIdx.x; j < total; j += blockDim.x) {
        if (order_key(all_v[j]) >= thr) {
          const int c = atomicAdd(&n_cand, 1);
          if (c < kMaxCand) {
            cand_v[c] = all_v[j];
            cand_i[c] = all_i[j];
          }
        }
      }
      __syncthreads();
      const float inv_t = 1.f / sp.temperature;
      const uint2 key = make_uint2(static_cast<uint32_t>(sp.seed), static_cast<uint32_t>(sp.seed >> 32));
      const int n = min(n_cand, kMaxCand);
      chosen = pick_restricted(cand_v, cand_i, n, k, sp, inv_t, key, &n_cand);
      // raw logit of the chosen token: it is among the sorted candidates
      if (threadIdx.x < kMaxCand && cand_i[threadIdx.x] == chosen) hdr[0].raw = cand_v[threadIdx.x];
      __syncthreads();
      raw = hdr[0].raw;
    }
    if (threadIdx.x == 0) {
      a.out_tok[row] = chosen;
      if (a.out_lp) a.out_lp[row] = raw - log_z;
    }
  }
  if (threadIdx.x == 0) {
    if (atomicAdd(a.state + 1, 1u) == static_cast<uint32_t>(a.S - 1)) {
      a.state[0] = target;
      a.state[1] = 0;
      __threadfence();
    }
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


void tp_sample(const TpSample& t, const float* logits, int S, int V_local, int64_t ld, const SampleParams* params,
               int32_t* out_tok, float* out_lp, cudaStream_t st) {
  if (S <= 0) return;
  VMC_CHECK(t.nranks >= 1 && t.nranks <= 8, "tp_sample: 1..8 ranks");
  VMC_CHECK(S <= t.max_rows, "tp_sample: more rows than the exchange buffer holds");
  TpSampleArgs a{};
  a.logits = logits;
  a.V_local = V_local;
  a.v0 = t.rank * V_local;
  a.ld = ld;
  a.params = params;
  a.S = S;
  a.rank = t.rank;
  a.nranks = t.nranks;
  for (int q = 0; q < 8; ++q) {
    a.xbuf[q] = q < t.nranks ? static_cast<uint8_t*>(t.xbuf[q]) : nullptr;
    a.count[q] = q < t.nranks ? t.count[q] : nullptr;
  }
  a.max_rows = t.max_rows;
  a.state = t.state;
  a.out_tok = out_tok;
  a.out_lp = out_lp;
  a.err = t.err;
  launch_k(tp_sample_local_kernel, dim3(S), dim3(kThreads), 0, st, a);
  const int dyn = 8 * kMaxCand * 8;
  static bool configured = false;
  if (!configured) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(tp_sample_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn));
    configured = true;
  }
  launch_k(tp_sample_merge_kernel, dim3(S), dim3(kThreads), dyn, st, a);
}

size_t tp_sample_row_bytes() { return kXRowBytes; }

}  // namespace vmc
