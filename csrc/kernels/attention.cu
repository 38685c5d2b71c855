// Paged flash attention over the block-table KV cache (prefill chunks, decode, split-KV combine).
//
// Replaces the reference's attention paths: ggml-cuda flash_attn_ext_f16 (fattn-mma-f16.cuh:1707,
// contiguous llama KV, used for prefill) and flash_attn_ext_vec (fattn-vec.cuh:21, decode), plus
// vm_c's unreachable paged kernels (src/cuda/attention_kernels.cu:37,140,271). Here the KV cache
// is vm_c's paged layout: per layer [num_blocks, 2 (K,V), Hkv, block_size=16, D] bf16, addressed
// through per-request block tables.
//
// GQA packing: all G = Hq/Hkv query heads that share a KV head are processed by one CTA as rows of
// one tile (packed row = token * G + head), so every K/V byte is loaded once per group. Tiles are
// 16 packed rows per warp and use mma.sync m16n8k16 (bf16 -> fp32): a decode tile has only
// G (4..8) real rows, below the 64/128-row minimum of a tcgen05 MMA, and decode attention is bound
// by HBM bandwidth, not by tensor throughput.
//
//  * attn_decode_kernel  : 16 packed rows per CTA (q_len * G <= 16), 4 warps walk disjoint KV pages
//                          (per-warp cp.async double buffering) and merge through shared memory.
//                          grid.z splits the KV range across CTAs; partials (+LSE) are merged by
//                          attn_combine_kernel.
//  * attn_prefill_kernel : 64 packed rows per CTA (4 warps x 16), 64-key tiles shared by the warps,
//                          causal mask against each row's absolute position.
#include "attention.h"
#include "common.cuh"
#include "turboquant.cuh"

namespace vmc {
namespace {

constexpr int kBS = 16;  // tokens per KV block
#ifndef VMC_DEC_STAGES
#define VMC_DEC_STAGES 3
#endif
constexpr int kDecStages = VMC_DEC_STAGES;  // KV pages in flight per decode warp (ring depth)
#ifndef VMC_PRE_NS
#define VMC_PRE_NS 1
#endif
constexpr int kPreNS = VMC_PRE_NS;  // 16-key sub-blocks per softmax update on unmasked prefill tiles
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Frag {
  static constexpr int KD = D / 16;  // k-steps over the head dim
  static constexpr int ND = D / 8;   // n-tiles over the head dim
  static constexpr int RB = D * 2 + 16;  // padded smem row stride (bytes) -> conflict-free ldmatrix
};

struct AttnParams {
  const __nv_bfloat16* q;   // [T, Hq, D]
  const __nv_bfloat16* kv;  // [num_blocks, 2, Hkv, 16, D]
  const int32_t* q_start;   // [R + 1]
  const int32_t* ctx_len;   // [R]
  const int32_t* block_tables;  // [R, max_blocks]
  int max_blocks;
  int Hq, Hkv, G;
  float scale_log2;         // softmax scale * log2(e)
  __nv_bfloat16* out;       // [T, Hq, D]
  int splits;
  float* part_o;            // [splits, T, Hq, D] (split-KV only)
  float* part_lse;          // [splits, T, Hq]
  int req_offset;           // first request index handled by this launch
  TqDev tq;                 // TurboQuant cache of this layer (tq.cache == nullptr: bf16 pages in kv)
  // Token trees (prefill kernel): per query token, which of the request's last tree_span key
  // positions it may attend to (bit i = key at position ctx - tree_span + i); null = causal.
  const uint64_t* tree_mask;
  int tree_span;
};

// Copy one 16 x D page (K or V) into a padded smem tile (rows 16*slot .. 16*slot+15).
template <int D>
__device__ __forceinline__ void load_page_warp(uint8_t* smem_tile, int row0, const __nv_bfloat16* src, int lane) {
  constexpr int CH = D / 8;           // 16-byte chunks per row
  constexpr int TOTAL = kBS * CH;     // chunks per page
#pragma unroll
  for (int i = lane; i < TOTAL; i += 32) {
    const int r = i / CH, c = i % CH;
    cp_async16(smem_u32(smem_tile + (row0 + r) * Frag<D>::RB + c * 16), src + r * D + c * 8);
  }
}

// Load Q fragments for the 16 packed rows starting at `prow0` of request r.
template <int D>
__device__ __forceinline__ void load_q_frags(const AttnParams& p, int qs, int qlen, int kvh, int prow0, int lane,
                                             uint32_t (&qa)[Frag<D>::KD][4]) {
  const int rows = qlen * p.G;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int pr = prow0 + (lane >> 2) + 8 * half;
    const bool valid = pr < rows;
    const int t = valid ? pr / p.G : 0, g = valid ? pr % p.G : 0;
    const __nv_bfloat16* qrow = p.q + (static_cast<int64_t>(qs + t) * p.Hq + kvh * p.G + g) * D;
#pragma unroll
    for (int kd = 0; kd < Frag<D>::KD; ++kd) {
      const int d0 = 16 * kd + 2 * (lane & 3);
      qa[kd][half] = valid ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
      qa[kd][2 + half] = valid ? *reinterpret_cast<const uint32_t*>(qrow + d0 + 8) : 0u;
    }
  }
}

// One step of attention over NS x 16 keys for a warp's 16 rows: S = Q K^T for all NS sub-blocks,
// one online-softmax update (one rescale of O) for the whole step, then O += P V. K/V rows
// key0 .. key0 + 16 NS - 1 of the smem tiles. kpos0: absolute position of the first key;
// qpos_lo/hi: absolute positions of this thread's two rows (-1 for invalid rows); keys past a row's
// position are masked (and, with a tree mask, keys at or after tbase that are not its ancestors).
template <int D, int NS, bool MASK = true>
__device__ __forceinline__ void attn_step(const uint8_t* sK, const uint8_t* sV, int key0, int kpos0,
                                          const uint32_t (&qa)[Frag<D>::KD][4], int qpos_lo, int qpos_hi,
                                          float scale_log2, float (&o)[Frag<D>::ND][4], float (&m)[2], float (&l)[2],
                                          int lane, bool tree = false, int tbase = 0, uint64_t tm_lo = 0,
                                          uint64_t tm_hi = 0) {
  constexpr int RB = Frag<D>::RB;
  float s[2 * NS][4];
#pragma unroll
  for (int j = 0; j < 2 * NS; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
  // S = Q K^T: two n-tiles of 8 keys per sub-block.
#pragma unroll
  for (int sb = 0; sb < NS; ++sb) {
#pragma unroll
    for (int kd = 0; kd < Frag<D>::KD; ++kd) {
      uint32_t b[4];
      const int i = lane;
      const int key = key0 + 16 * sb + (i & 7) + 8 * (i >> 4);
      const int dim = 16 * kd + 8 * ((i >> 3) & 1);
      ldmatrix_x4(b, smem_u32(sK + key * RB + dim * 2));
      mma_bf16_16816(s[2 * sb], qa[kd], b[0], b[1]);
      mma_bf16_16816(s[2 * sb + 1], qa[kd], b[2], b[3]);
    }
  }
  // Mask + online softmax. Thread holds rows (lane/4) [e=0,1] and (lane/4 + 8) [e=2,3].
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < 2 * NS; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int kp = kpos0 + 8 * j + 2 * (lane & 3) + (e & 1);
      const int qp = (e < 2) ? qpos_lo : qpos_hi;
      float v = s[j][e] * scale_log2;
      if constexpr (MASK) {
        if (kp > qp) v = -INFINITY;
        else if (tree && kp >= tbase && !((((e < 2) ? tm_lo : tm_hi) >> (kp - tbase)) & 1ull)) v = -INFINITY;
      }
      s[j][e] = v;
      mx[e >> 1] = fmaxf(mx[e >> 1], v);
    }
  }
  float corr[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float mnew = fmaxf(m[h], mx[h]);
    corr[h] = (mnew == -INFINITY) ? 1.f : exp2f(m[h] - mnew);
    m[h] = mnew;
  }
  float rs[2] = {0.f, 0.f};
  uint32_t pa[NS][4];
#pragma unroll
  for (int j = 0; j < 2 * NS; ++j) {
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float mm = m[e >> 1];
      pv[e] = (mm == -INFINITY) ? 0.f : exp2f(s[j][e] - mm);
      rs[e >> 1] += pv[e];
    }
    // A fragment of P (16 rows x 16 keys) of sub-block j / 2: a0/a1 from its n-tile 0, a2/a3 from 1.
    pa[j >> 1][2 * (j & 1)] = pack_bf16x2(pv[0], pv[1]);
    pa[j >> 1][2 * (j & 1) + 1] = pack_bf16x2(pv[2], pv[3]);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
    rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
    l[h] = l[h] * corr[h] + rs[h];
  }
#pragma unroll
  for (int nd = 0; nd < Frag<D>::ND; ++nd) {
    o[nd][0] *= corr[0];
    o[nd][1] *= corr[0];
    o[nd][2] *= corr[1];
    o[nd][3] *= corr[1];
  }
  // O += P V, one k-step of 16 keys per sub-block.
#pragma unroll
  for (int sb = 0; sb < NS; ++sb) {
#pragma unroll
    for (int nd = 0; nd < Frag<D>::ND; nd += 2) {
      uint32_t b[4];
      const int i = lane;
      const int key = key0 + 16 * sb + (i & 7) + 8 * ((i >> 3) & 1);
      const int dim = 8 * nd + 8 * (i >> 4);
      ldmatrix_x4_trans(b, smem_u32(sV + key * RB + dim * 2));
      mma_bf16_16816(o[nd], pa[sb], b[0], b[1]);
      mma_bf16_16816(o[nd + 1], pa[sb], b[2], b[3]);
    }
  }
}

template <int D>
__device__ __forceinline__ void attn_step16(const uint8_t* sK, const uint8_t* sV, int key0, int kpos0,
                                            const uint32_t (&qa)[Frag<D>::KD][4], int qpos_lo, int qpos_hi,
                                            float scale_log2, float (&o)[Frag<D>::ND][4], float (&m)[2],
                                            float (&l)[2], int lane) {
  attn_step<D, 1>(sK, sV, key0, kpos0, qa, qpos_lo, qpos_hi, scale_log2, o, m, l, lane);
}

// TurboQuant: dequantise half (dims [half * D/2, (half + 1) * D/2)) of one key's K and V slot into
// bf16 rows of the padded smem tiles. Lanes 2k and 2k+1 of a warp hold the two halves of one key
// (the norm correction needs the squared norm over all D dims). KB: key bits (3, 4; 8 = fp8 e4m3),
// VB: value bits. Invalid keys (past the context) get zero rows.
template <int D, int KB, int VB>
__device__ __forceinline__ void tq_dequant_half(const AttnParams& p, int blk, int off, int kvh, int half, bool valid,
                                                uint8_t* k_row, uint8_t* v_row, const float* s_cent) {
  constexpr int HD = D / 2;
  const TqDev& t = p.tq;
  const uint16_t* sp = reinterpret_cast<const uint16_t*>(t.cache + tq_slot_offset(t, valid ? blk : 0, off, kvh, p.Hkv));
  uint32_t* kr = reinterpret_cast<uint32_t*>(k_row + half * HD * 2);
  if constexpr (KB == 8) {
#pragma unroll
    for (int w = 0; w < HD / 2; ++w) {
      const uint16_t b2 = valid ? __ldg(sp + half * (HD / 2) + w) : 0;
      uint32_t h2;
      asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(b2));
      const __half2 hv = *reinterpret_cast<const __half2*>(&h2);
      kr[w] = valid ? pack_bf16x2(__low2float(hv), __high2float(hv)) : 0u;
    }
  } else {
    // Packed indices stay in registers: one pass for the squared norm of the reconstruction (norm
    // correction), one to write the scaled centroids.
    constexpr int NW = KB == 4 ? HD / 4 : HD / 16;  // 16-bit words (4-bit) or 48-bit groups (3-bit)
    uint64_t pk[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if constexpr (KB == 4) {
        pk[w] = valid ? __ldg(sp + half * (HD / 4) + w) : 0;
      } else {
        const uint16_t* gp = sp + half * (HD / 16) * 3 + w * 3;
        pk[w] = valid ? (static_cast<uint64_t>(__ldg(gp)) | (static_cast<uint64_t>(__ldg(gp + 1)) << 16) |
                         (static_cast<uint64_t>(__ldg(gp + 2)) << 32))
                      : 0ull;
      }
    }
    constexpr int PER = KB == 4 ? 4 : 16;
    constexpr uint32_t MASK = (1u << KB) - 1u;
    float ss = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int n = 0; n < PER; ++n) {
        const float c = s_cent[(pk[w] >> (KB * n)) & MASK];
        ss += c * c;
      }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    const float norm = valid ? bf16_bits_to_float(__ldg(sp + t.mse_bytes / 2)) : 0.f;
    const float factor = t.norm_correction ? norm * rsqrtf(ss + 1e-16f) : norm;
#pragma unroll
    for (int w = 0; w < NW; ++w)
#pragma unroll
      for (int n = 0; n < PER; n += 2) {
        const float c0 = s_cent[(pk[w] >> (KB * n)) & MASK], c1 = s_cent[(pk[w] >> (KB * (n + 1))) & MASK];
        kr[(w * PER + n) / 2] = valid ? pack_bf16x2(c0 * factor, c1 * factor) : 0u;
      }
  }
  // V
  const uint16_t* vp = sp + t.key_packed / 2;
  const float vs = valid ? bf16_bits_to_float(__ldg(vp + t.val_bytes / 2)) : 0.f;
  const float vm = valid ? bf16_bits_to_float(__ldg(vp + t.val_bytes / 2 + 1)) : 0.f;
  uint32_t* vr = reinterpret_cast<uint32_t*>(v_row + half * HD * 2);
  if constexpr (VB == 4) {
#pragma unroll
    for (int w = 0; w < HD / 4; ++w) {
      const uint32_t b2 = valid ? __ldg(vp + half * (HD / 4) + w) : 0;
      const float a0 = static_cast<float>(b2 & 15u) * vs + vm, a1 = static_cast<float>((b2 >> 4) & 15u) * vs + vm;
      const float a2 = static_cast<float>((b2 >> 8) & 15u) * vs + vm, a3 = static_cast<float>((b2 >> 12) & 15u) * vs + vm;
      vr[2 * w] = valid ? pack_bf16x2(a0, a1) : 0u;
      vr[2 * w + 1] = valid ? pack_bf16x2(a2, a3) : 0u;
    }
  } else {
#pragma unroll
    for (int g = 0; g < HD / 16; ++g) {
      const uint16_t* gp = vp + half * (HD / 16) * 3 + g * 3;
      const uint64_t bits = valid ? (static_cast<uint64_t>(__ldg(gp)) | (static_cast<uint64_t>(__ldg(gp + 1)) << 16) |
                                     (static_cast<uint64_t>(__ldg(gp + 2)) << 32))
                                  : 0ull;
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        const float a0 = static_cast<float>((bits >> (3 * n)) & 7u) * vs + vm;
        const float a1 = static_cast<float>((bits >> (3 * n + 3)) & 7u) * vs + vm;
        vr[8 * g + n / 2] = valid ? pack_bf16x2(a0, a1) : 0u;
      }
    }
  }
}

// Centroid table of the TurboQuant keys into shared memory (all threads; followed by a barrier).
__device__ __forceinline__ void tq_load_centroids(const AttnParams& p, float* s_cent) {
  const int n = p.tq.key_fp8 ? 0 : (1 << p.tq.key_bits);
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_cent[i] = p.tq.centroids[i];
  __syncthreads();
}

// Merge the 4 warps of a decode CTA (each holds o, m, l for the same 16 packed rows over disjoint
// keys) through shared memory and write the output rows, or this split's partial O and LSE.
template <int D>
__device__ __forceinline__ void decode_merge_store(const AttnParams& p, uint8_t* smem, const float (&o)[Frag<D>::ND][4],
                                                   const float (&m)[2], const float (&l)[2], int rows, int qs, int kvh,
                                                   int split, int total_tokens) {
  constexpr int ND = Frag<D>::ND;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Merge the 4 warps: each writes (m, l, o) for its 16 rows to smem; warp 0 combines.
  float* mo = reinterpret_cast<float*>(smem);           // [4][16][D]
  float* ml = mo + 4 * 16 * D;                          // [4][16][2]
  const int rlo = lane >> 2, rhi = rlo + 8;
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) {
    const int d = 8 * nd + 2 * (lane & 3);
    mo[(warp * 16 + rlo) * D + d] = o[nd][0];
    mo[(warp * 16 + rlo) * D + d + 1] = o[nd][1];
    mo[(warp * 16 + rhi) * D + d] = o[nd][2];
    mo[(warp * 16 + rhi) * D + d + 1] = o[nd][3];
  }
  if ((lane & 3) == 0) {
    ml[(warp * 16 + rlo) * 2 + 0] = m[0];
    ml[(warp * 16 + rlo) * 2 + 1] = l[0];
    ml[(warp * 16 + rhi) * 2 + 0] = m[1];
    ml[(warp * 16 + rhi) * 2 + 1] = l[1];
  }
  __syncthreads();
  // 128 threads: thread -> (row = tid / 8, 8 dim-chunks of D/8 each)
  const int row = threadIdx.x >> 3;
  if (row < rows) {
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, ml[(w * 16 + row) * 2]);
    float L = 0.f, wsc[4];
    for (int w = 0; w < 4; ++w) {
      const float mw = ml[(w * 16 + row) * 2];
      wsc[w] = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      L += wsc[w] * ml[(w * 16 + row) * 2 + 1];
    }
    const int t = row / p.G, g = row % p.G;
    const int64_t orow = static_cast<int64_t>(qs + t) * p.Hq + kvh * p.G + g;
    constexpr int PER = D / 8;
    const int d0 = (threadIdx.x & 7) * PER;
    if (p.splits == 1) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      for (int d = d0; d < d0 + PER; d += 2) {
        float a0 = 0.f, a1 = 0.f;
        for (int w = 0; w < 4; ++w) {
          a0 += wsc[w] * mo[(w * 16 + row) * D + d];
          a1 += wsc[w] * mo[(w * 16 + row) * D + d + 1];
        }
        *reinterpret_cast<uint32_t*>(p.out + orow * D + d) = pack_bf16x2(a0 * inv, a1 * inv);
      }
    } else if (qs + t < total_tokens) {
      // Partial: normalised O and log2-sum-exp of this split. Rows past the partial buffers'
      // total_tokens rows (a q_start beyond the launch's token count) are not written.
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float* po = p.part_o + (static_cast<int64_t>(split) * total_tokens * p.Hq + orow) * D;
      for (int d = d0; d < d0 + PER; ++d) {
        float a = 0.f;
        for (int w = 0; w < 4; ++w) a += wsc[w] * mo[(w * 16 + row) * D + d];
        po[d] = a * inv;
      }
      if ((threadIdx.x & 7) == 0)
        p.part_lse[static_cast<int64_t>(split) * total_tokens * p.Hq + orow] = (L > 0.f) ? M + log2f(L) : -INFINITY;
    }
  }
}


// ---------------------------------------------------------------------------------------------
// Decode: one CTA = (request, kv head, split); 16 packed rows; 4 warps split the pages.

template <int D, int KQ>
__global__ void __launch_bounds__(128) attn_decode_kernel(AttnParams p, int total_tokens) {
  constexpr int RB = Frag<D>::RB;
  constexpr int ND = Frag<D>::ND;
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.y;
  const int r = blockIdx.x + p.req_offset;
  const int split = blockIdx.z;
  const int qs = p.q_start[r], qlen = p.q_start[r + 1] - qs;
  const int ctx = p.ctx_len[r];
  if (qlen <= 0) return;
  const int nblocks = (ctx + kBS - 1) / kBS;
  const int per_split = (nblocks + p.splits - 1) / p.splits;
  const int b0 = split * per_split, b1 = min(nblocks, b0 + per_split);
  const int32_t* bt = p.block_tables + static_cast<int64_t>(r) * p.max_blocks;

  uint32_t qa[Frag<D>::KD][4];
  load_q_frags<D>(p, qs, qlen, kvh, 0, lane, qa);
  const int rows = qlen * p.G;
  const int pr_lo = lane >> 2, pr_hi = pr_lo + 8;
  const int qpos_lo = pr_lo < rows ? ctx - qlen + pr_lo / p.G : -1;
  const int qpos_hi = pr_hi < rows ? ctx - qlen + pr_hi / p.G : -1;

  float o[ND][4];
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  // Per-warp ring of kDecStages pages: stage s holds K rows [0,16) and V rows [0,16) of one page.
  uint8_t* wsm = smem + warp * (kDecStages * 2 * kBS * RB);
  auto sK = [&](int s) { return wsm + s * (2 * kBS * RB); };
  auto sV = [&](int s) { return wsm + s * (2 * kBS * RB) + kBS * RB; };
  const int64_t page_elems = static_cast<int64_t>(kBS) * D;
  // Block ids of this warp's pages (b0 + warp + 4j), 32 at a time in one coalesced load, so that a
  // page's copy never waits on its own dependent block-table load.
  int ids = 0;
  auto fetch_ids = [&](int j0) {
    const int bj = b0 + warp + 4 * (j0 + lane);
    ids = bj < b1 ? bt[bj] : 0;
  };
  __shared__ float s_cent[KQ ? 16 : 1];
  if constexpr (KQ != 0) tq_load_centroids(p, s_cent);
  auto issue = [&](int j, int s) {  // j = index of the page among this warp's pages
    if ((j & 31) == 0) fetch_ids(j);
    const int blk = __shfl_sync(0xffffffffu, ids, j & 31);
    if constexpr (KQ == 0) {
      const __nv_bfloat16* kp = p.kv + (static_cast<int64_t>(blk) * 2 * p.Hkv + kvh) * page_elems;
      const __nv_bfloat16* vp = p.kv + (static_cast<int64_t>(blk) * 2 * p.Hkv + p.Hkv + kvh) * page_elems;
      load_page_warp<D>(sK(s), 0, kp, lane);
      load_page_warp<D>(sV(s), 0, vp, lane);
    } else {
      const int key = lane >> 1;
      const bool valid = (b0 + warp + 4 * j) * kBS + key < ctx;
      tq_dequant_half<D, KQ / 10, KQ % 10>(p, blk, key, kvh, lane & 1, valid, sK(s) + key * RB, sV(s) + key * RB,
                                           s_cent);
    }
  };
  int b = b0 + warp;
  int j = 0;
#pragma unroll
  for (int s = 0; s < kDecStages - 1; ++s) {
    if (b + 4 * s < b1) issue(s, s);
    cp_async_commit();
  }
  for (; b < b1; b += 4, ++j) {
    const int ahead = j + kDecStages - 1;
    if (b + 4 * (kDecStages - 1) < b1) issue(ahead, ahead % kDecStages);
    cp_async_commit();
    cp_async_wait<kDecStages - 1>();
    __syncwarp();
    const int stage = j % kDecStages;
    attn_step16<D>(sK(stage), sV(stage), 0, b * kBS, qa, qpos_lo, qpos_hi, p.scale_log2, o, m, l, lane);
    __syncwarp();
  }
  cp_async_wait<0>();
  __syncthreads();
  decode_merge_store<D>(p, smem, o, m, l, rows, qs, kvh, split, total_tokens);
}

// Merge split-KV partials: one warp per (token, head).
template <int D>
__global__ void attn_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse, int splits,
                                    int64_t rows, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_lse[s * rows + row]);
  float wsum = 0.f;
  float acc[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) acc[i] = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float lse = part_lse[s * rows + row];
    const float w = (lse == -INFINITY) ? 0.f : exp2f(lse - M);
    wsum += w;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) acc[i] += w * part_o[(s * rows + row) * D + lane + 32 * i];
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
  for (int i = 0; i < D / 32; ++i) out[row * D + lane + 32 * i] = __float2bfloat16(acc[i] * inv);
}

// ---------------------------------------------------------------------------------------------
// Prefill / extend: one CTA = (64 packed rows, kv head, request). 64-key tiles shared by warps.

template <int D, int KQ>
__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnParams p) {
  constexpr int RB = Frag<D>::RB;
  constexpr int ND = Frag<D>::ND;
  constexpr int TK = 64;  // keys per tile (4 pages)
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.z + p.req_offset;
  const int kvh = blockIdx.y;
  const int qs = p.q_start[r], qlen = p.q_start[r + 1] - qs;
  const int rows = qlen * p.G;
  const int prow_cta = blockIdx.x * 64;
  if (prow_cta >= rows) return;
  const int ctx = p.ctx_len[r];
  const int32_t* bt = p.block_tables + static_cast<int64_t>(r) * p.max_blocks;
  const int prow0 = prow_cta + 16 * warp;

  uint32_t qa[Frag<D>::KD][4];
  load_q_frags<D>(p, qs, qlen, kvh, prow0, lane, qa);
  const int pr_lo = prow0 + (lane >> 2), pr_hi = pr_lo + 8;
  const int qpos_lo = pr_lo < rows ? ctx - qlen + pr_lo / p.G : -1;
  const int qpos_hi = pr_hi < rows ? ctx - qlen + pr_hi / p.G : -1;
  const bool tree = p.tree_mask != nullptr;
  const uint64_t tm_lo = (tree && pr_lo < rows) ? p.tree_mask[qs + pr_lo / p.G] : 0ull;
  const uint64_t tm_hi = (tree && pr_hi < rows) ? p.tree_mask[qs + pr_hi / p.G] : 0ull;
  // Keys needed by this CTA: up to the largest query position among its rows.
  const int last_row = min(rows, prow_cta + 64) - 1;
  const int kmax = ctx - qlen + last_row / p.G + 1;  // exclusive
  const int ntiles = (kmax + TK - 1) / TK;
  // Rows of this warp that exist at all (skip compute for fully invalid warps).
  const bool warp_active = prow0 < rows;
  const int warp_qmax = warp_active ? (ctx - qlen + (min(rows, prow0 + 16) - 1) / p.G) : -1;
  const int warp_qmin = ctx - qlen + prow0 / p.G;  // position of the warp's first row

  float o[ND][4];
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  auto sK = [&](int s) { return smem + s * (2 * TK * RB); };
  auto sV = [&](int s) { return smem + s * (2 * TK * RB) + TK * RB; };
  const int64_t page_elems = static_cast<int64_t>(kBS) * D;
  constexpr int CH = D / 8;
  __shared__ float s_cent[KQ ? 16 : 1];
  if constexpr (KQ != 0) tq_load_centroids(p, s_cent);
  auto issue = [&](int tile, int s) {
    if constexpr (KQ != 0) {
      // One thread per (key, half) of the 64-key tile: dequantise into the bf16 tiles.
      const int key = threadIdx.x >> 1;
      const int b = tile * 4 + (key >> 4);
      const bool valid = tile * TK + key < kmax;
      const int blk = valid ? bt[b] : 0;
      tq_dequant_half<D, KQ / 10, KQ % 10>(p, blk, key & 15, kvh, threadIdx.x & 1, valid, sK(s) + key * RB,
                                           sV(s) + key * RB, s_cent);
      return;
    }
    // 4 pages x (K, V) x 16 rows x CH chunks, spread over 128 threads.
    constexpr int TOTAL = 4 * 2 * kBS * CH;
    for (int i = threadIdx.x; i < TOTAL; i += 128) {
      const int c = i % CH;
      const int rr = (i / CH) % kBS;
      const int kvsel = (i / (CH * kBS)) % 2;
      const int pg = i / (CH * kBS * 2);
      const int b = tile * 4 + pg;
      const bool valid = b * kBS < kmax;
      const int blk = valid ? bt[b] : 0;
      const __nv_bfloat16* src =
          p.kv + (static_cast<int64_t>(blk) * 2 * p.Hkv + kvsel * p.Hkv + kvh) * page_elems + rr * D + c * 8;
      uint8_t* dst = (kvsel ? sV(s) : sK(s)) + (pg * kBS + rr) * RB + c * 16;
      cp_async16_zfill(smem_u32(dst), src, valid);
    }
  };
  issue(0, 0);
  cp_async_commit();
  for (int tile = 0; tile < ntiles; ++tile) {
    const int s = tile & 1;
    if (tile + 1 < ntiles) issue(tile + 1, s ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (warp_active) {
      const int kpos0 = tile * TK;
      if (!tree && kpos0 + TK - 1 <= warp_qmin) {
        // every key of the tile precedes every row of the warp: no mask, one softmax update per
        // kPreNS x 16 keys
#pragma unroll
        for (int sub = 0; sub < TK / 16; sub += kPreNS)
          attn_step<D, kPreNS, false>(sK(s), sV(s), sub * 16, kpos0 + sub * 16, qa, qpos_lo, qpos_hi, p.scale_log2,
                                      o, m, l, lane);
      } else {
#pragma unroll
        for (int sub = 0; sub < TK / 16; ++sub) {
          const int kp0 = kpos0 + sub * 16;
          if (kp0 <= warp_qmax && kp0 < kmax)
            attn_step<D, 1>(sK(s), sV(s), sub * 16, kp0, qa, qpos_lo, qpos_hi, p.scale_log2, o, m, l, lane, tree,
                            ctx - p.tree_span, tm_lo, tm_hi);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  if (!warp_active) return;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int pr = (half ? pr_hi : pr_lo);
    if (pr >= rows) continue;
    const int t = pr / p.G, g = pr % p.G;
    const int64_t row = static_cast<int64_t>(qs + t) * p.Hq + kvh * p.G + g;
    const float inv = l[half] > 0.f ? 1.f / l[half] : 0.f;
    __nv_bfloat16* dst = p.out + row * D;
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      const int d = 8 * nd + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(dst + d) = pack_bf16x2(o[nd][2 * half] * inv, o[nd][2 * half + 1] * inv);
    }
  }
}

template <int D>
constexpr int decode_smem() {
  constexpr int RB = Frag<D>::RB;
  constexpr int smem_pipe = 4 * kDecStages * 2 * kBS * RB;
  constexpr int smem_merge = 4 * 16 * D * 4 + 4 * 16 * 2 * 4;
  return smem_pipe > smem_merge ? smem_pipe : smem_merge;
}

template <int D, int KQ>
void config_decode() {
  static bool cfg = false;
  if (!cfg) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(attn_decode_kernel<D, KQ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        decode_smem<D>()));
    cfg = true;
  }
}

template <int D>
int decode_ctas_per_sm() {
  config_decode<D, 0>();
  int n = 0;
  VMC_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_decode_kernel<D, 0>, 128, decode_smem<D>()));
  return n;
}

template <int D, int KQ>
void launch_decode(const AttnParams& p, int num_reqs, int total_tokens, cudaStream_t st) {
  const int smem = decode_smem<D>();
  config_decode<D, KQ>();
  dim3 grid(num_reqs, p.Hkv, p.splits);
  launch_k(attn_decode_kernel<D, KQ>, grid, dim3(128), smem, st, p, total_tokens);
  if (p.splits > 1) {
    const int64_t rows = static_cast<int64_t>(total_tokens) * p.Hq;
    launch_k(attn_combine_kernel<D>, dim3(static_cast<int>((rows + 3) / 4)), dim3(128), 0, st,
             static_cast<const float*>(p.part_o), static_cast<const float*>(p.part_lse), p.splits, rows, p.out);
  }
}

template <int D, int KQ>
void launch_prefill(const AttnParams& p, int num_reqs, int max_qlen, cudaStream_t st) {
  constexpr int RB = Frag<D>::RB;
  const int smem = 2 * 2 * 64 * RB;
  static bool cfg = false;
  if (!cfg) {
    VMC_CUDA_CHECK(cudaFuncSetAttribute(attn_prefill_kernel<D, KQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cfg = true;
  }
  dim3 grid((max_qlen * p.G + 63) / 64, p.Hkv, num_reqs);
  launch_k(attn_prefill_kernel<D, KQ>, grid, dim3(128), smem, st, p);
}

// KV format code: 0 = bf16 pages; TurboQuant: 10 * key bits + value bits (fp8 keys: 8).
template <int D, int KQ>
void launch_any(const AttnParams& p, const AttnLaunch& a, cudaStream_t st) {
  if (a.decode) launch_decode<D, KQ>(p, a.num_reqs, a.total_tokens, st);
  else launch_prefill<D, KQ>(p, a.num_reqs, a.max_qlen, st);
}

template <int D>
void dispatch_kv(const AttnParams& p, const AttnLaunch& a, cudaStream_t st) {
  if (!a.tq) {
    launch_any<D, 0>(p, a, st);
    return;
  }
  const int kb = a.tq->key_fp8 ? 8 : a.tq->key_bits, vb = a.tq->value_bits;
  switch (kb * 10 + vb) {
    case 44: launch_any<D, 44>(p, a, st); break;
    case 34: launch_any<D, 34>(p, a, st); break;
    case 33: launch_any<D, 33>(p, a, st); break;
    case 84: launch_any<D, 84>(p, a, st); break;
    default: throw std::runtime_error("attention: unsupported TurboQuant variant");
  }
}

// One warp per (request, layer, K/V, kv head): the lanes hold the request's rows (16-byte pieces,
// lane-strided) in registers, then write them, so sources and destinations may overlap.
constexpr int kMoveMax = 16;
template <int D>
__global__ void kv_move_kernel(__nv_bfloat16* cache, int L, int64_t layer_elems, int Hkv, const int32_t* src,
                               const int32_t* dst, const int32_t* cnt, int num_reqs, int max_moves) {
  pdl_trigger();
  pdl_wait();
  constexpr int kVec = D / 8;                      // 16-byte pieces per row
  constexpr int kPer = (kVec + 31) / 32;           // pieces per lane
  const int lane = threadIdx.x & 31;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t per_req = static_cast<int64_t>(L) * 2 * Hkv;
  if (w >= per_req * num_reqs) return;
  const int r = static_cast<int>(w / per_req);
  int rest = static_cast<int>(w % per_req);
  const int l = rest / (2 * Hkv);
  rest %= 2 * Hkv;
  const int kvsel = rest / Hkv, h = rest % Hkv;
  const int n = min(cnt[r], kMoveMax);
  __nv_bfloat16* base = cache + l * layer_elems;
  auto row = [&](int slot) {
    const int blk = slot / 16, off = slot % 16;
    return reinterpret_cast<uint4*>(base + ((static_cast<int64_t>(blk) * 2 + kvsel) * Hkv + h) * 16 * D +
                                    static_cast<int64_t>(off) * D);
  };
  uint4 v[kMoveMax][kPer];
#pragma unroll
  for (int i = 0; i < kMoveMax; ++i) {
    if (i < n) {
      const uint4* s = row(src[r * max_moves + i]);
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (lane + 32 * j < kVec) v[i][j] = s[lane + 32 * j];
    }
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kMoveMax; ++i) {
    if (i < n) {
      uint4* d = row(dst[r * max_moves + i]);
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (lane + 32 * j < kVec) d[lane + 32 * j] = v[i][j];
    }
  }
}

}  // namespace

void kv_move(void* cache, int L, int64_t layer_elems, int Hkv, int D, const int32_t* src, const int32_t* dst,
             const int32_t* cnt, int num_reqs, int max_moves, cudaStream_t st) {
  VMC_CHECK(max_moves <= kMoveMax, "kv_move: at most 16 moves per request");
  if (num_reqs <= 0) return;
  const int64_t warps = static_cast<int64_t>(num_reqs) * L * 2 * Hkv;
  const dim3 grid(static_cast<unsigned>((warps + 7) / 8));
  auto* c = static_cast<__nv_bfloat16*>(cache);
  switch (D) {
    case 32: launch_k(kv_move_kernel<32>, grid, dim3(256), 0, st, c, L, layer_elems, Hkv, src, dst, cnt, num_reqs, max_moves); break;
    case 64: launch_k(kv_move_kernel<64>, grid, dim3(256), 0, st, c, L, layer_elems, Hkv, src, dst, cnt, num_reqs, max_moves); break;
    case 128: launch_k(kv_move_kernel<128>, grid, dim3(256), 0, st, c, L, layer_elems, Hkv, src, dst, cnt, num_reqs, max_moves); break;
    default: throw std::runtime_error("kv_move: unsupported head dim");
  }
}

void paged_attention(const AttnLaunch& a, cudaStream_t st) {
  VMC_CHECK(a.Hq % a.Hkv == 0, "attention: Hq must be a multiple of Hkv");
  AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(a.q);
  p.kv = static_cast<const __nv_bfloat16*>(a.kv);
  p.q_start = a.q_start;
  p.ctx_len = a.ctx_len;
  p.block_tables = a.block_tables;
  p.max_blocks = a.max_blocks;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.G = a.Hq / a.Hkv;
  p.scale_log2 = a.scale * kLog2e;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.splits = a.decode ? (a.splits < 1 ? 1 : a.splits) : 1;
  p.part_o = a.part_o;
  p.part_lse = a.part_lse;
  p.req_offset = a.req_offset;
  if (a.tq) p.tq = *a.tq;
  else p.tq.cache = nullptr;
  p.tree_mask = a.tree_mask;
  p.tree_span = a.tree_span;
  VMC_CHECK(!(a.decode && a.tree_mask), "attention: tree masks need the prefill path");
  VMC_CHECK(!a.tree_mask || (a.tree_span >= 1 && a.tree_span <= 64), "attention: tree span must be 1..64");
  if (a.num_reqs <= 0) return;
  if (attn_prefill_tc_eligible(a)) {
    attn_prefill_tc(a, st);
    return;
  }
  if (a.decode) {
    VMC_CHECK(a.max_qlen * p.G <= 16, "attention: decode path needs q_len * group <= 16");
    VMC_CHECK(p.splits == 1 || (a.part_o && a.part_lse), "attention: split-KV needs partial buffers");
  }
  switch (a.D) {
    case 32: dispatch_kv<32>(p, a, st); break;
    case 64: dispatch_kv<64>(p, a, st); break;
    case 128: dispatch_kv<128>(p, a, st); break;
    default: throw std::runtime_error("attention: unsupported head dim");
  }
}

int attn_decode_ctas_per_sm(int D) {
  switch (D) {
    case 32: return decode_ctas_per_sm<32>();
    case 64: return decode_ctas_per_sm<64>();
    case 128: return decode_ctas_per_sm<128>();
    default: throw std::runtime_error("attention: unsupported head dim");
  }
}

}  // namespace vmc
