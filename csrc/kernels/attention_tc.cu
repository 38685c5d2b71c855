// Paged prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), head dim 128.
//
// Replaces, for the prefill chunks of bf16 caches, the role of ggml-cuda's flash_attn_ext_f16
// (fattn-mma-f16.cuh:1707), which runs on mma.sync; the mma.sync prefill kernel in attention.cu
// stays the path for other head dims, TurboQuant caches and token-tree masks.
//
// One CTA owns 128 GQA-packed query rows (packed row = token * G + head of one KV head, so the G
// heads that share a KV head read each K/V byte once) and walks the request's paged KV in tiles of
// 128 keys (8 pages of 16 tokens):
//
//   warp 0     TMA producer: per tile, 8 pages x (K, V) x two 64-column halves, loaded through a
//              3-D tensor map over the layer's pages ([pages][16 rows][128] bf16, 128-byte swizzle)
//              into a 3-stage ring; pages past the needed range repeat the last needed page (finite
//              data under a zero softmax weight).
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM S buffers (A = Q and
//              B = K both K-major in shared memory), then O += P_j V_j with A = P_j read from TMEM
//              (bf16, written by the softmax warps) and B = V_j in shared memory as an MN-major
//              operand (V pages are key-major with D contiguous). S_{j+1} is issued before P_j is
//              waited on, so the tensor pipe computes the next scores while softmax runs.
//   warps 2-5  softmax, one packed row per thread (TMEM lane = row): causal mask against the row's
//              absolute position, online softmax in base 2 with a lazy base (moved only when a
//              row's maximum grows by more than 2^8, then O is rescaled in TMEM after PV_{j-1}
//              completed), P_j (bf16) into TMEM once PV_{j-2} released its buffer, and the final
//              O / l epilogue to global memory.
//
// TMEM (512 columns): S0 [0,128), S1 [128,256), O [256,384), P0 [384,448), P1 [448,512).
// Every wait is bounded; an expired wait records its code in the device error word, and the CTA
// drains its in-flight copies and frees its TMEM before returning.
#include <cuda.h>

#include <cstdlib>
#include <cstring>

#include "attention.h"
#include "common.cuh"

namespace vmc {
namespace {

constexpr int kD = 128;       // head dim
constexpr int kRows = 128;    // packed query rows per CTA (UMMA M)
constexpr int kKeys = 128;    // keys per KV tile (UMMA N of S, K of PV)
constexpr int kStages = 3;    // K/V tiles in flight
constexpr int kThreads = 192;
constexpr uint32_t kHalf = 128 * 128;                 // 128 rows x 64 bf16 (one swizzled half)
constexpr uint32_t kTile = 2 * kHalf;                 // 128 rows x 128 bf16
constexpr uint32_t kSmemData = kTile + kStages * 2 * kTile;
constexpr uint32_t kSmem = kSmemData + 1024 + 256;   // + alignment slack + barriers
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256, kColP0 = 384, kColP1 = 448;
constexpr float kRescaleLog2 = 8.f;                   // lazy-rescale threshold (factor 256)
// Error word on an expired wait: kErrAttnWait | (n << 8), n = 1..8 naming the wait.
__device__ __forceinline__ uint32_t tc_err(uint32_t n) { return static_cast<uint32_t>(kErrAttnWait) | (n << 8); }

struct TcParams {
  const __nv_bfloat16* q;       // [T, Hq, 128]
  const int32_t* q_start;
  const int32_t* ctx_len;
  const int32_t* block_tables;
  int max_blocks;
  int Hq, Hkv, G;
  float scale_log2;
  __nv_bfloat16* out;           // [T, Hq, 128]
  int req_offset;
  uint32_t* err;
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Shared-memory descriptor of an MN-major operand with 128-byte swizzle: each 128-byte row holds 64
// consecutive MN elements of one K index, 8 K rows form a 1024-byte atom (stride byte offset), and
// the next 64 MN elements start `lbo` bytes further (leading byte offset).
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3fff);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fff) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ bool warp_all(bool v) { return __all_sync(0xffffffffu, v); }

__global__ void __launch_bounds__(kThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap kv_map, TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.z + p.req_offset;
  const int kvh = blockIdx.y;
  const int qs = p.q_start[r], qlen = p.q_start[r + 1] - qs;
  const int rows = qlen * p.G;
  // Heaviest row tiles (latest positions, most keys) first.
  const int prow0 = (gridDim.x - 1 - blockIdx.x) * kRows;
  if (prow0 >= rows) return;
  const int ctx = p.ctx_len[r];
  const int last_row = min(rows, prow0 + kRows) - 1;
  const int kmax = ctx - qlen + last_row / p.G + 1;    // keys any row of this CTA may see
  const int ntiles = (kmax + kKeys - 1) / kKeys;
  const int npages = (kmax + 15) / 16;
  const int32_t* bt = p.block_tables + static_cast<int64_t>(r) * p.max_blocks;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  auto sK = [&](int s) { return smem + kTile + s * 2 * kTile; };
  auto sV = [&](int s) { return smem + kTile + s * 2 * kTile + kTile; };
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kSmemData);
  uint64_t* kv_full = bars;                 // [kStages]
  uint64_t* kv_empty = bars + kStages;      // [kStages]
  uint64_t* s_full = bars + 2 * kStages;    // [2]
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* p_free = p_full + 2;            // [2] PV of the buffer's last P completed
  uint64_t* o_done = p_free + 2;
  uint64_t* q_full = o_done + 1;
  uint64_t* mma_fin = q_full + 1;           // every MMA of the CTA completed (before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_fin + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&p_free[b], 1);
    }
    mbar_init(o_done, 1);
    mbar_init(q_full, 128);
    mbar_init(mma_fin, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, p.err, tc_err(1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * kTile);
        for (int pg = 0; pg < 8; ++pg) {
          const int blk = bt[min(j * 8 + pg, npages - 1)];
          const int pk = blk * 2 * p.Hkv + kvh, pv = pk + p.Hkv;  // page ids of K and V
          tma_load_3d(sK(s) + pg * 2048, &kv_map, &kv_full[s], 0, 0, pk);
          tma_load_3d(sK(s) + kHalf + pg * 2048, &kv_map, &kv_full[s], 64, 0, pk);
          tma_load_3d(sV(s) + pg * 2048, &kv_map, &kv_full[s], 0, 0, pv);
          tma_load_3d(sV(s) + kHalf + pg * 2048, &kv_map, &kv_full[s], 64, 0, pv);
        }
        issued = j + 1;
      }
      if (!ok) {  // drain: the copies of the last issued tiles land before the CTA exits
        for (int j = max(0, issued - kStages); j < issued; ++j)
          mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kRows, kKeys);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kRows, kD) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(q_full, 0, p.err, tc_err(2));
      tc_fence_after();
      const uint64_t qd[2] = {umma_sdesc_sw128(smem_u32(sQ)), umma_sdesc_sw128(smem_u32(sQ + kHalf))};
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&kv_full[s], (j / kStages) & 1, p.err, tc_err(3))) return false;
        tc_fence_after();
        const uint64_t kd[2] = {umma_sdesc_sw128(smem_u32(sK(s))), umma_sdesc_sw128(smem_u32(sK(s) + kHalf))};
        const uint32_t d = tmem + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
        for (int ks = 0; ks < kD / 16; ++ks)
          umma_bf16(d, qd[ks >> 2] + 2 * (ks & 3), kd[ks >> 2] + 2 * (ks & 3), idesc_s, ks > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, p.err, tc_err(4))) break;
        tc_fence_after();
        const int s = j % kStages;
        const uint32_t pa = tmem + ((j & 1) ? kColP1 : kColP0);
        const uint32_t va = smem_u32(sV(s));
#pragma unroll
        for (int ks = 0; ks < kKeys / 16; ++ks)
          umma_bf16_ts(tmem + kColO, pa + 8 * ks, sdesc_mn_sw128(va + ks * 16 * 128, kHalf), idesc_pv,
                       (j > 0 || ks > 0) ? 1u : 0u);
        umma_commit(&kv_empty[s]);
        umma_commit(&p_free[j & 1]);
        umma_commit(o_done);
      }
      umma_commit(mma_fin);
      mbar_wait(mma_fin, 0, nullptr, 0);
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;           // the TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;    // packed row within the tile = TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int prow = prow0 + row;
    const bool valid = prow < rows;
    const int t = valid ? prow / p.G : 0, g = valid ? prow % p.G : 0;
    const int64_t qoff = (static_cast<int64_t>(qs + t) * p.Hq + kvh * p.G + g) * kD;
    {
      const uint4* src = reinterpret_cast<const uint4*>(p.q + qoff);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = valid ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(sQ + (c >> 3) * kHalf + sw128_offset(row, c & 7)) = v;
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(q_full);
    const int qpos = valid ? ctx - qlen + t : -1;
    float m = -INFINITY, l = 0.f;  // m: the exponent base of this row's P values (log2 domain)
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = warp_all(mbar_wait(&s_full[j & 1], (j >> 1) & 1, p.err, tc_err(5)));
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[kKeys];
      const uint32_t scol = tmem + lane_addr + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
      for (int c = 0; c < kKeys / 16; ++c) tmem_ld16(scol + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(sv + 16 * c));
      tmem_ld_wait();
      const int lim = qpos - j * kKeys;  // keys 0..lim of this tile are visible to the row
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kKeys; ++i) {
        const float x = i <= lim ? __uint_as_float(sv[i]) * p.scale_log2 : -INFINITY;
        sv[i] = __float_as_uint(x);
        mx = fmaxf(mx, x);
      }
      // Lazy rescale: the base moves only when the tile's maximum exceeds it by more than
      // kRescaleLog2, so P stays <= 2^kRescaleLog2 (exact enough in bf16, no overflow in the fp32
      // O and l) and most tiles skip the O round trip and the wait for the previous PV.
      const bool move = mx > m + kRescaleLog2;   // m = -inf: the row's first visible key
      const float m_new = move ? mx : m;
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = move ? exp2f(m - base) : 1.f;  // 0 when the base is first set
      float sum = 0.f;
      uint32_t pk[kKeys / 2];
#pragma unroll
      for (int i = 0; i < kKeys / 2; ++i) {
        const float e0 = exp2f(__uint_as_float(sv[2 * i]) - base);
        const float e1 = exp2f(__uint_as_float(sv[2 * i + 1]) - base);
        sum += e0 + e1;
        pk[i] = pack_bf16x2(e0, e1);
      }
      l = l * alpha + sum;
      m = m_new;
      if (j >= 2) {  // P buffer j & 1 is free once PV_{j-2} completed
        ok = warp_all(mbar_wait(&p_free[j & 1], ((j >> 1) - 1) & 1, p.err, tc_err(7)));
        if (!ok) break;
        tc_fence_after();
      }
      const uint32_t pcol = tmem + lane_addr + ((j & 1) ? kColP1 : kColP0);
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c) tmem_st16(pcol + 16 * c, pk + 16 * c);
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // O holds the sum through tile j-1 once PV_{j-1} completed; rescale it to the new base.
        // (PV_{j-2} completed above, so phase j-1 is the oldest incomplete phase of o_done.)
        ok = warp_all(mbar_wait(o_done, (j - 1) & 1, p.err, tc_err(6)));
        if (!ok) break;
        tc_fence_after();
        {
#pragma unroll 1
          for (int c = 0; c < kD / 16; ++c) {
            uint32_t ov[16];
            tmem_ld16(tmem + lane_addr + kColO + 16 * c, ov);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st16(tmem + lane_addr + kColO + 16 * c, ov);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    if (ok) ok = warp_all(mbar_wait(mma_fin, 0, p.err, tc_err(8)));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.out + qoff);
#pragma unroll 1
      for (int c = 0; c < kD / 16; ++c) {
        uint32_t ov[16];
        tmem_ld16(tmem + lane_addr + kColO + 16 * c, ov);
        tmem_ld_wait();
        if (valid) {
          uint32_t w[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            w[e] = pack_bf16x2(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
          dst[2 * c] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[2 * c + 1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    VMC_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
    VMC_CHECK(f != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(f);
  }
  return fn;
}

int g_tc_mode = -1;  // -1: from VMC_ATTN_TC (default on), 0: off, 1: on

}  // namespace

void attn_prefill_tc_enable(int on) { g_tc_mode = on; }

bool attn_prefill_tc_eligible(const AttnLaunch& a) {
  if (g_tc_mode < 0) {
    const char* e = std::getenv("VMC_ATTN_TC");
    g_tc_mode = (e && std::strcmp(e, "0") == 0) ? 0 : 1;
  }
  return g_tc_mode == 1 && !a.decode && a.tq == nullptr && a.tree_mask == nullptr && a.D == kD &&
         a.num_blocks > 0 && a.Hq % a.Hkv == 0 && reinterpret_cast<uintptr_t>(a.kv) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(a.q) % 16 == 0 && reinterpret_cast<uintptr_t>(a.out) % 16 == 0;
}

void attn_prefill_tc(const AttnLaunch& a, cudaStream_t st) {
  if (a.num_reqs <= 0) return;
  TcParams p;
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.q_start = a.q_start;
  p.ctx_len = a.ctx_len;
  p.block_tables = a.block_tables;
  p.max_blocks = a.max_blocks;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.G = a.Hq / a.Hkv;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.req_offset = a.req_offset;
  p.err = a.err;
  // The layer's pages as a 3-D tensor: [pages = blocks x (K, V) x Hkv][16 rows][128] bf16.
  const int64_t pages = a.num_blocks * 2 * a.Hkv;
  VMC_CHECK(pages > 0 && pages < (int64_t(1) << 31), "attention_tc: page count out of range");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), 16, static_cast<cuuint64_t>(pages)};
  cuuint64_t strides[2] = {kD * 2, 16 * kD * 2};
  cuuint32_t box[3] = {64, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  const CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a.kv), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VMC_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed for the KV page map");
  static bool configured = false;
  if (!configured) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    configured = true;
  }
  const int G = a.Hq / a.Hkv;
  const dim3 grid((a.max_qlen * G + kRows - 1) / kRows, a.Hkv, a.num_reqs);
  launch_k(attn_prefill_tc_kernel, grid, dim3(kThreads), kSmem, st, map, p);
}

}  // namespace vmc
