// Peer-memory tensor-parallel collectives fused with the adjacent compute (one process per GPU,
// NVLink 5 / NVSwitch peer access through CUDA IPC mappings).
//
// Replaces the reference's NCCL all-reduce at its two per-layer sites (after Wo and after the FFN /
// MoE down projection: src/distributed/nccl_comm.cu:259-327 via the GGML_OP_VM_C_TP_ALLREDUCE graph
// op, src/official/llama/models/llama.cpp:171,196,221), which is followed by a separate residual add
// and RMSNorm in the ggml graph.
//
//  * ar_add_rmsnorm_kernel: the row-parallel GEMM of every rank writes its fp32 split-K partials
//    into its own symmetric buffer; this kernel then (1) sums this rank's splits locally into split
//    slice 0, (2) signals every peer and waits for every peer's signal (epoch flags,
//    release/acquire at system scope, bounded spin), (3) reads slice 0 of all ranks over NVLink and
//    adds them in rank order (bit-identical result on every rank), (4) adds the residual stream,
//    (5) applies RMSNorm and writes the normalised bf16 activations for the next GEMM. One-shot
//    all-reduce + residual + norm in a single kernel.
//
// Synchronisation: CTA b of every rank owns flag slot b; its participation count (epoch) advances
// identically on all ranks because every rank launches the same sequence of calls with the same
// grid. The partial buffers alternate between two sites, and a rank rewrites a site only after its
// next all-reduce has seen every peer start that next all-reduce, so no reader can still be reading.
#include <cstdlib>
#include <cstring>

#include "comm.h"
#include "common.cuh"

namespace vmc {
namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Flag protocol. 0 (default): system-scope fence + release store / acquire loads, the PTX memory
// model's guarantee that a peer which sees the flag sees the partial rows. 1: GPU-scope fences around
// relaxed system-scope flag accesses, which relies on a peer reading this GPU's partial through this
// GPU's L2 over NVLink rather than on the memory model; kept as a measurement option. Measured on 2
// B200s inside CUDA graphs (64 x 4096 fp32, 4 split-K partials): 24.5 us for 0, 14.5 us for 1, 17.9 us
// for NCCL all-reduce + a separate residual/RMSNorm kernel. The default serving path uses rs_norm_ag
// (below), not this kernel.
#ifndef VMC_AR_SYNC
#define VMC_AR_SYNC 0
#endif
// Peer data: bypass L1 so that a line cached by an earlier call is never reused.
__device__ __forceinline__ float4 ld_cg_f4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

constexpr int kMaxRanks = 8;
constexpr int kArThreads = 256;
constexpr int kMaxPer = 32;  // floats per thread held in registers (H <= 256 * 4 * 8 = 8192)

// NR = number of ranks (compile-time, so that the loads of all ranks' partials are issued
// back to back before the first add).
//
// Two phases around one flag exchange. (1) Each CTA sums this rank's split-K partials of its rows
// (local memory) into split slice 0 of its own symmetric buffer, then publishes with a system-scope
// release. (2) After every peer's CTA b has published, it reads slice 0 of every rank for its rows
// (one fp32 partial per rank crosses NVLink, whatever the split count), adds them in rank order
// (the same sum on every rank), adds the residual and applies RMSNorm. Rows are assigned to CTAs
// identically on every rank (row = b + k * grid), so CTA b only ever waits for the CTAs b of its
// peers, which wrote exactly the rows it reads.
template <int NR>
__global__ void __launch_bounds__(kArThreads) ar_add_rmsnorm_kernel(ArArgs a) {
  const int b = blockIdx.x;
  __shared__ float red[32];
  __shared__ int ok;
  pdl_trigger();
  pdl_wait();
  const int H = a.H;
  const int nvec = H / 4;
  float* mine = const_cast<float*>(a.data[a.rank]);
  if (a.nsplit > 1) {
    for (int row = b; row < a.T; row += gridDim.x) {
      const size_t base = static_cast<size_t>(row) * H;
      for (int vi = threadIdx.x; vi < nvec; vi += kArThreads) {
        float4 p[8];  // splits 0..7 loaded together, then added in split order
#pragma unroll
        for (int sp = 0; sp < 8; ++sp)
          if (sp < a.nsplit) p[sp] = *reinterpret_cast<const float4*>(mine + sp * a.split_stride + base + 4 * vi);
        float4 acc = p[0];
#pragma unroll
        for (int sp = 1; sp < 8; ++sp) {
          if (sp < a.nsplit) {
            acc.x += p[sp].x;
            acc.y += p[sp].y;
            acc.z += p[sp].z;
            acc.w += p[sp].w;
          }
        }
        for (int sp = 8; sp < a.nsplit; ++sp) {
          const float4 q = *reinterpret_cast<const float4*>(mine + sp * a.split_stride + base + 4 * vi);
          acc.x += q.x;
          acc.y += q.y;
          acc.z += q.z;
          acc.w += q.w;
        }
        *reinterpret_cast<float4*>(mine + base + 4 * vi) = acc;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const uint32_t e = a.epochs[b] + 1;
    a.epochs[b] = e;
    // Publish: the partial rows this CTA's peers will read are in this GPU's memory (written by the
    // previous kernel or by phase 1 above); then one flag store per rank.
    if constexpr (VMC_AR_SYNC == 0) {
      __threadfence_system();
      for (int q = 0; q < NR; ++q) st_release_sys(a.flags[q] + b * kMaxRanks + a.rank, e);
    } else {
      __threadfence();
      for (int q = 0; q < NR; ++q) st_relaxed_sys(a.flags[q] + b * kMaxRanks + a.rank, e);
    }
    // Bounded by time (about 2 s of SM clock for all peers together), not by a poll count, so the
    // bound does not depend on how long one system-scope load takes.
    int good = 1;
    const long long t0 = clock64();
    for (int q = 0; q < NR && good; ++q) {
      while ((VMC_AR_SYNC == 0 ? ld_acquire_sys(a.flags[a.rank] + b * kMaxRanks + q)
                               : ld_relaxed_sys(a.flags[a.rank] + b * kMaxRanks + q)) < e) {
        if (clock64() - t0 > (4ll << 30)) {
          atomicCAS(a.err, 0u, static_cast<uint32_t>(kErrCommWait));
          good = 0;
          break;
        }
      }
    }
    if constexpr (VMC_AR_SYNC != 0) __threadfence();
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  for (int row = b; row < a.T; row += gridDim.x) {
    float v[kMaxPer];
    float ss = 0.f;
    const size_t base = static_cast<size_t>(row) * H;
#pragma unroll
    for (int j = 0; j < kMaxPer / 4; ++j) {
      const int vi = threadIdx.x + j * kArThreads;
      if (vi < nvec) {
        float4 acc = *reinterpret_cast<const float4*>(a.resid + base + 4 * vi);
        float4 p[NR];
#pragma unroll
        for (int q = 0; q < NR; ++q) p[q] = ld_cg_f4(a.data[q] + base + 4 * vi);
#pragma unroll
        for (int q = 0; q < NR; ++q) {  // rank order: the same sum on every rank
          acc.x += p[q].x;
          acc.y += p[q].y;
          acc.z += p[q].z;
          acc.w += p[q].w;
        }
        *reinterpret_cast<float4*>(a.resid + base + 4 * vi) = acc;
        v[4 * j] = acc.x;
        v[4 * j + 1] = acc.y;
        v[4 * j + 2] = acc.z;
        v[4 * j + 3] = acc.w;
        ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < kArThreads / 32 ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / H + a.eps);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kMaxPer / 4; ++j) {
      const int vi = threadIdx.x + j * kArThreads;
      if (vi < nvec) {
        const float4 w = *reinterpret_cast<const float4*>(a.w + 4 * vi);
        uint2 o;
        o.x = pack_bf16x2(v[4 * j] * inv * w.x, v[4 * j + 1] * inv * w.y);
        o.y = pack_bf16x2(v[4 * j + 2] * inv * w.z, v[4 * j + 3] * inv * w.w);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.out) + base + 4 * vi) = o;
      }
    }
  }
}

// ---- reduce-scatter + residual + RMSNorm + all-gather ------------------------------------------
//
// Memory-model protocol (PTX scopes): every producer of remote data (a source GEMM CTA storing its
// partial tile into the owner's receive buffer, or an owner CTA pushing its normalised rows into a
// peer's h) finishes its stores, synchronises its threads (bar.sync), and one thread issues a
// system-scope acq_rel fence followed by a relaxed system-scope add on the consumer's arrival
// counter: a release pattern, so a consumer that reads the counter with a system-scope acquire load
// observes every store made before the barrier. Counters only grow; the expected value of the next
// call lives in the consumer's private `state` and advances by the number of arrivals per call.
// Waits are bounded and record kErrCommWait.

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void red_add_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *p >= target (wrap-safe comparison), system-scope acquire. The bound is time
// (about 2 s of SM clock), not an iteration count, so sleeping between polls cannot stretch it.
__device__ __forceinline__ bool wait_count_sys(const uint32_t* p, uint32_t target, uint32_t* err) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (static_cast<int32_t>(ld_acquire_sys(p) - target) >= 0) return true;
    if (clock64() - t0 > (4ll << 30)) {
      atomicCAS(err, 0u, static_cast<uint32_t>(kErrCommWait));
      return false;
    }
    if (i > 32) __nanosleep(64);
  }
}

struct RsArgs {
  const __nv_bfloat16* recv;  // this rank's receive buffer of the site: [slots][rpr][H]
                              // (expert-parallel combine: [rpr][k][H], the k expert outputs per row)
  uint32_t* rs_count;         // this rank's reduce-scatter arrival counter of the site
  uint32_t* ag_count[kMaxRanks];  // every rank's all-gather arrival counter of the site
  __nv_bfloat16* h[kMaxRanks];    // every rank's h buffer [max_tokens][H]
  uint32_t* state;            // this site's bookkeeping: [0] rs target, [1] ag target, [2] CTAs done
  float* resid;
  const float* w;
  float eps;
  int T, H, rpr, slots, rank;
  uint32_t rs_inc;
  uint32_t* err;
  int gather;                 // 0: write this rank's rows of h only (no all-gather)
  const float* topk_w;        // expert-parallel combine: router weights [rpr][slots]
  uint32_t* reset;            // expert-parallel combine: counters to zero once the rows are read
  int reset_n;
  int two_level;              // 1: the all-gather is signalled once per rank (last CTA), else per CTA
};

constexpr int kRsThreads = 256;
constexpr int kRsMaxVec = 4;  // 8-element vectors per thread (H <= 256 * 8 * 4 = 8192)

// MOE = false: sum of the slots (source rank, K split) of each owned row. MOE = true: the router-
// weighted sum of the k expert outputs returned for each owned row (expert-parallel combine).
template <int NR, bool MOE>
__global__ void __launch_bounds__(kRsThreads) rs_norm_ag_kernel(RsArgs a) {
  __shared__ float red[32];
  __shared__ int ok;
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, G = gridDim.x;
  if (threadIdx.x == 0) ok = wait_count_sys(a.rs_count, a.state[0] + a.rs_inc, a.err) ? 1 : 0;
  __syncthreads();
  const int H = a.H, nvec = H / 8;
  if (ok) {
    for (int lr = b; lr < a.rpr; lr += G) {
      const int m = a.rank * a.rpr + lr;
      if (m >= a.T) break;
      const size_t row = static_cast<size_t>(m) * H;
      float v[kRsMaxVec][8];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kRsMaxVec; ++j) {
        const int vi = threadIdx.x + j * kRsThreads;
        if (vi >= nvec) continue;
        const float4 r0 = *reinterpret_cast<const float4*>(a.resid + row + 8 * vi);
        const float4 r1 = *reinterpret_cast<const float4*>(a.resid + row + 8 * vi + 4);
        float acc[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
        if constexpr (MOE) {
          for (int sl = 0; sl < a.slots; ++sl) {  // expert outputs in top-k order
            const float wt = a.topk_w[static_cast<size_t>(lr) * a.slots + sl];
            const uint4 p = __ldcg(reinterpret_cast<const uint4*>(a.recv + (static_cast<size_t>(lr) * a.slots + sl) * H) + vi);
            const uint32_t q[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[2 * e] += wt * bf16_lo(q[e]);
              acc[2 * e + 1] += wt * bf16_hi(q[e]);
            }
          }
        }
        // partial slots in (source rank, split) order: the same sum on every owner
        int sl = MOE ? a.slots : 0;
        for (; sl + 4 <= a.slots; sl += 4) {
          uint4 p[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            p[u] = __ldcg(reinterpret_cast<const uint4*>(a.recv + (static_cast<size_t>(sl + u) * a.rpr + lr) * H) + vi);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t q[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[2 * e] += bf16_lo(q[e]);
              acc[2 * e + 1] += bf16_hi(q[e]);
            }
          }
        }
        for (; sl < a.slots; ++sl) {
          const uint4 p = __ldcg(reinterpret_cast<const uint4*>(a.recv + (static_cast<size_t>(sl) * a.rpr + lr) * H) + vi);
          const uint32_t q[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] += bf16_lo(q[e]);
            acc[2 * e + 1] += bf16_hi(q[e]);
          }
        }
        *reinterpret_cast<float4*>(a.resid + row + 8 * vi) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(a.resid + row + 8 * vi + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          v[j][e] = acc[e];
          ss += acc[e] * acc[e];
        }
      }
      ss = warp_sum(ss);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
      __syncthreads();
      if (threadIdx.x < 32) {
        float t = threadIdx.x < kRsThreads / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
      }
      __syncthreads();
      const float inv = rsqrtf(red[0] / H + a.eps);
      __syncthreads();
#pragma unroll
      for (int j = 0; j < kRsMaxVec; ++j) {
        const int vi = threadIdx.x + j * kRsThreads;
        if (vi >= nvec) continue;
        const float4 w0 = *reinterpret_cast<const float4*>(a.w + 8 * vi);
        const float4 w1 = *reinterpret_cast<const float4*>(a.w + 8 * vi + 4);
        uint4 o;
        o.x = pack_bf16x2(v[j][0] * inv * w0.x, v[j][1] * inv * w0.y);
        o.y = pack_bf16x2(v[j][2] * inv * w0.z, v[j][3] * inv * w0.w);
        o.z = pack_bf16x2(v[j][4] * inv * w1.x, v[j][5] * inv * w1.y);
        o.w = pack_bf16x2(v[j][6] * inv * w1.z, v[j][7] * inv * w1.w);
        if (a.gather) {
#pragma unroll
          for (int q = 0; q < NR; ++q) {  // own rank first is not required: the order is irrelevant
            const int dst = (a.rank + q) % NR;
            *reinterpret_cast<uint4*>(a.h[dst] + row + 8 * vi) = o;
          }
        } else {
          *reinterpret_cast<uint4*>(a.h[a.rank] + row + 8 * vi) = o;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Every CTA makes its all-gather stores complete at system scope and counts itself on this
    // site's CTA counter (GPU-scope acq_rel). The CTA that completes the grid advances the targets of
    // the next call (every CTA has read them by then), clears the expert row counters this combine
    // consumed, and signals the all-gather once at every rank: its system-scope fence orders all the
    // grid's stores, acquired through the CTA counter, before that one arrival. CTA 0 returns only
    // after every rank's signal has arrived here.
    const uint32_t ag_inc = static_cast<uint32_t>(a.two_level ? NR : NR * G);
    const uint32_t ag_target = a.state[1] + ag_inc;  // read before this CTA counts itself
    if (a.gather) {
      fence_acq_rel_sys();
      if (!a.two_level) {
#pragma unroll
        for (int q = 0; q < NR; ++q) red_add_sys(a.ag_count[q], 1u);
      }
    }
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(a.state + 2) : "memory");
    if (old == static_cast<uint32_t>(G - 1)) {
      a.state[0] += a.rs_inc;
      if (a.gather) a.state[1] += ag_inc;
      a.state[2] = 0;
      for (int i = 0; i < a.reset_n; ++i) a.reset[i] = 0;
      if (a.gather && a.two_level) {
        fence_acq_rel_sys();
#pragma unroll
        for (int q = 0; q < NR; ++q) red_add_sys(a.ag_count[q], 1u);
      } else {
        __threadfence();
      }
    }
    if (a.gather && b == 0) wait_count_sys(a.ag_count[a.rank], ag_target, a.err);
  }
}

}  // namespace

void ar_add_rmsnorm(const ArArgs& a, int max_ctas, cudaStream_t st) {
  VMC_CHECK(a.nranks >= 1 && a.nranks <= kMaxRanks, "ar_add_rmsnorm: 1..8 ranks");
  VMC_CHECK(a.H % 4 == 0 && a.H <= kArThreads * kMaxPer, "ar_add_rmsnorm: hidden size unsupported");
  if (a.T <= 0) return;
  const int grid = a.T < max_ctas ? a.T : max_ctas;
  switch (a.nranks) {
    case 1: launch_k(ar_add_rmsnorm_kernel<1>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 2: launch_k(ar_add_rmsnorm_kernel<2>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 3: launch_k(ar_add_rmsnorm_kernel<3>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 4: launch_k(ar_add_rmsnorm_kernel<4>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 5: launch_k(ar_add_rmsnorm_kernel<5>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 6: launch_k(ar_add_rmsnorm_kernel<6>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    case 7: launch_k(ar_add_rmsnorm_kernel<7>, dim3(grid), dim3(kArThreads), 0, st, a); break;
    default: launch_k(ar_add_rmsnorm_kernel<8>, dim3(grid), dim3(kArThreads), 0, st, a); break;
  }
}

bool tp_two_level() {
  static const bool on = [] {
    const char* e = std::getenv("VMC_TP_TWO_LEVEL");
    return e && std::strcmp(e, "1") == 0;
  }();
  return on;
}

namespace {
template <bool MOE>
void launch_rs(const RsArgs& a, int nranks, int grid, cudaStream_t st) {
  switch (nranks) {
    case 1: launch_k(rs_norm_ag_kernel<1, MOE>, dim3(grid), dim3(kRsThreads), 0, st, a); break;
    case 2: launch_k(rs_norm_ag_kernel<2, MOE>, dim3(grid), dim3(kRsThreads), 0, st, a); break;
    case 4: launch_k(rs_norm_ag_kernel<4, MOE>, dim3(grid), dim3(kRsThreads), 0, st, a); break;
    case 8: launch_k(rs_norm_ag_kernel<8, MOE>, dim3(grid), dim3(kRsThreads), 0, st, a); break;
    default: throw std::runtime_error("rs_norm_ag: 1, 2, 4 or 8 ranks");
  }
}

RsArgs rs_common(const TpComm& c, int site, int T, int H, float* resid, const float* w, float eps, int gather) {
  VMC_CHECK(c.nranks >= 1 && c.nranks <= kMaxRanks && site >= 0 && site < 4, "rs_norm_ag: bad ranks / site");
  VMC_CHECK(H % 8 == 0 && H <= kRsThreads * 8 * kRsMaxVec, "rs_norm_ag: hidden size unsupported");
  RsArgs a{};
  for (int q = 0; q < kMaxRanks; ++q) {
    a.ag_count[q] = q < c.nranks ? c.ag_count[site][q] : nullptr;
    a.h[q] = q < c.nranks ? static_cast<__nv_bfloat16*>(c.h[q]) : nullptr;
  }
  a.state = c.state + 4 * site;
  a.resid = resid;
  a.w = w;
  a.eps = eps;
  a.T = T;
  a.H = H;
  a.rpr = tp_rows_per_rank(T, c.nranks);
  a.rank = c.rank;
  a.err = c.err;
  a.gather = gather;
  a.two_level = tp_two_level() ? 1 : 0;
  return a;
}
}  // namespace

void rs_norm_ag(const TpComm& c, int site, int T, int H, int splits, int rs_inc, float* resid, const float* w,
                float eps, cudaStream_t st, int gather) {
  RsArgs a = rs_common(c, site, T, H, resid, w, eps, gather);
  VMC_CHECK(static_cast<int64_t>(c.nranks) * splits * a.rpr <= c.recv_rows, "rs_norm_ag: receive buffer too small");
  a.recv = static_cast<const __nv_bfloat16*>(c.recv[site & 1][c.rank]);
  a.rs_count = c.rs_count[site & 1][c.rank];
  a.slots = c.nranks * splits;
  a.rs_inc = static_cast<uint32_t>(rs_inc);
  launch_rs<false>(a, c.nranks, tp_norm_ctas(a.rpr, c.max_ctas), st);
}

void moe_combine_norm_ag(const TpComm& c, const void* comb, uint32_t* comb_count, int comb_inc, const float* topk_w,
                         int k, uint32_t* reset, int reset_n, int T, int H, float* resid, const float* w, float eps,
                         cudaStream_t st) {
  RsArgs a = rs_common(c, 2, T, H, resid, w, eps, 1);
  a.recv = static_cast<const __nv_bfloat16*>(comb);
  a.rs_count = comb_count;
  a.slots = k;
  a.rs_inc = static_cast<uint32_t>(comb_inc);
  a.topk_w = topk_w;
  a.reset = reset;
  a.reset_n = reset_n;
  launch_rs<true>(a, c.nranks, tp_norm_ctas(a.rpr, c.max_ctas), st);
}

// ---- symmetric memory through CUDA IPC ----------------------------------------------------------

uint64_t sym_alloc(size_t bytes, void* handle_out) {
  void* p = nullptr;
  VMC_CUDA_CHECK(cudaMalloc(&p, bytes));
  VMC_CUDA_CHECK(cudaMemset(p, 0, bytes));
  VMC_CUDA_CHECK(cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), p));
  return reinterpret_cast<uint64_t>(p);
}

uint64_t sym_open(const void* handle) {
  void* p = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  VMC_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<uint64_t>(p);
}

void sym_close(uint64_t peer_ptr) { VMC_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(peer_ptr))); }
void sym_free(uint64_t ptr) { VMC_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

}  // namespace vmc
