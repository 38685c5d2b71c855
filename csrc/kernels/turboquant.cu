// TurboQuant store: RoPE + rotation + quantisation of K / V into the compressed paged cache, in one
// kernel on the QKV projection output.
//
// Replaces the reference's TQ store path (src/cuda/turboquant_kernels.cu:792 turboquant_store:
// fp16 copy, one-thread-per-vector norm kernel, a cuBLAS SGEMM with the dense d x d Hadamard
// matrix, then one thread per (token, head) quantising serially with a 256-float local array).
// Here one warp owns one (token, head) vector: RoPE in registers, the norm by a warp reduction, the
// rotation as an in-warp fast Walsh-Hadamard transform (O(d log d) shuffles, optionally after
// seeded random sign flips per layer and KV head: a random orthogonal rotation), the Lloyd-Max
// quantisation by binary search over the midpoints, and the packed slot bytes written with 16-bit
// stores (slots are only 2-byte aligned). Query heads get the same RoPE + rotation (written as the
// bf16 attention input), so q.k is preserved exactly by the orthogonal transform.
#include "common.cuh"
#include "turboquant.cuh"
#include "turboquant_ops.h"

namespace vmc {
namespace {

template <typename TI, int E>
__global__ void rope_store_tq_kernel(const TI* __restrict__ qkv, int nsplit, int64_t split_stride, int T, int Hq,
                                     int Hkv, const int32_t* __restrict__ pos, const int32_t* __restrict__ slots,
                                     const float2* __restrict__ cs, int neox, __nv_bfloat16* __restrict__ q_out,
                                     TqDev tq) {
  constexpr int D = 32 * E;
  __shared__ float s_mid[255];
  pdl_trigger();
  pdl_wait();
  const int nmid = tq.key_fp8 ? 0 : (1 << tq.key_bits) - 1;
  for (int i = threadIdx.x; i < nmid; i += blockDim.x) s_mid[i] = tq.midpoints[i];
  __syncthreads();
  const int warps = blockDim.x >> 5;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int H = Hq + 2 * Hkv;
  if (gw >= static_cast<int64_t>(T) * H) return;
  const int t = static_cast<int>(gw / H), h = static_cast<int>(gw % H);
  const TI* src = qkv + static_cast<int64_t>(t) * H * D + static_cast<int64_t>(h) * D;
  auto ld = [&](int i) -> float {
    if constexpr (sizeof(TI) == 2) {
      return __bfloat162float(src[i]);
    } else {
      float v = src[i];
      for (int sp = 1; sp < nsplit; ++sp) v += src[sp * split_stride + i];
      return v;
    }
  };
  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = ld(lane * E + j);
  const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv, is_v = h >= Hq + Hkv;
  // RoPE on Q and K. Pairs (i0, i1) may live in different lanes: fetch partners with shuffles.
  if (!is_v) {
    const float2* c = cs + static_cast<int64_t>(pos[t]) * (D / 2);
    float r[E];
    // Generic partner exchange: every lane publishes all E values, partners are read per element.
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const int i = lane * E + j;
      const int partner = neox ? (i < D / 2 ? i + D / 2 : i - D / 2) : (i ^ 1);
      float pv = 0.f;
#pragma unroll
      for (int jj = 0; jj < E; ++jj) {
        const float cand = __shfl_sync(0xffffffffu, v[jj], partner / E);
        if (jj == partner % E) pv = cand;
      }
      const bool first = neox ? (i < D / 2) : ((i & 1) == 0);
      const float2 cv = c[neox ? (first ? i : i - D / 2) : (i >> 1)];
      r[j] = first ? (v[j] * cv.x - pv * cv.y) : (pv * cv.y + v[j] * cv.x);
    }
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] = r[j];
  }
  const int kvh = is_q ? h / (Hq / Hkv) : (is_k ? h - Hq : h - Hq - Hkv);
  if (!tq.key_fp8 && !is_v) {
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] *= tq_sign(tq.rot_seed, tq.layer, kvh, lane * E + j);
  }
  if (is_q) {
    if (!tq.key_fp8) tq_fwht<E>(v, lane);
    __nv_bfloat16* dst = q_out + (static_cast<int64_t>(t) * Hq + h) * D + lane * E;
#pragma unroll
    for (int j = 0; j < E; ++j) dst[j] = __float2bfloat16(v[j]);
    return;
  }
  const int slot_idx = slots[t];
  if (slot_idx < 0) return;
  uint8_t* sp = tq.cache + tq_slot_offset(tq, slot_idx / 16, slot_idx % 16, kvh, Hkv);
  uint16_t* sp16 = reinterpret_cast<uint16_t*>(sp);  // slots are 2-byte aligned
  if (is_k) {
    if (tq.key_fp8) {
      // E bytes per lane, written as 16-bit words (pairs of lanes when E == 1).
      uint32_t b = 0;
#pragma unroll
      for (int j = 0; j < E; j += 2) {
        const float lo = v[j], hi = (j + 1 < E) ? v[j + 1] : 0.f;
        uint16_t w;
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(w) : "f"(hi), "f"(lo));
        b |= static_cast<uint32_t>(w) << (8 * j);
      }
      if constexpr (E >= 2) {
#pragma unroll
        for (int j = 0; j < E; j += 2) sp16[(lane * E + j) / 2] = static_cast<uint16_t>(b >> (8 * j));
      } else {
        const uint32_t other = __shfl_down_sync(0xffffffffu, b, 1);
        if ((lane & 1) == 0) sp16[lane / 2] = static_cast<uint16_t>((b & 0xffu) | ((other & 0xffu) << 8));
      }
      return;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    const float norm = sqrtf(ss);
    const float inv = norm > 0.f ? 1.f / norm : 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) v[j] *= inv;
    tq_fwht<E>(v, lane);
    // Lloyd-Max index: number of midpoints <= y (binary search).
    uint32_t idx[E];
#pragma unroll
    for (int j = 0; j < E; ++j) {
      int lo = 0, hi = nmid;  // answer in [0, nmid]
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (v[j] >= s_mid[mid]) lo = mid + 1;
        else hi = mid;
      }
      idx[j] = static_cast<uint32_t>(lo);
    }
    if (tq.key_bits == 4) {
      // 4 E bits per lane; a 16-bit word covers 4 dims = 4 / E lanes.
      uint32_t pk = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) pk |= (idx[j] & 0xfu) << (4 * j);
      constexpr int LPW = 4 / E > 0 ? 4 / E : 1;
      uint32_t word = pk;
#pragma unroll
      for (int r = 1; r < LPW; ++r) word |= __shfl_down_sync(0xffffffffu, pk, r) << (4 * E * r);
      if constexpr (E >= 4) {
#pragma unroll
        for (int w = 0; w < E / 4; ++w) sp16[(lane * E) / 4 + w] = static_cast<uint16_t>(pk >> (16 * w));
      } else {
        if (lane % LPW == 0) sp16[lane / LPW] = static_cast<uint16_t>(word);
      }
    } else {
      // 3-bit: 16 dims = 48 bits = three 16-bit words, gathered on the first lane of the group.
      uint64_t pk = 0;
#pragma unroll
      for (int j = 0; j < E; ++j) pk |= static_cast<uint64_t>(idx[j] & 7u) << (3 * j);
      constexpr int LPG = 16 / E;
      uint64_t g = pk;
#pragma unroll
      for (int r = 1; r < LPG; ++r) {
        const uint32_t lo = __shfl_down_sync(0xffffffffu, static_cast<uint32_t>(pk), r);
        g |= static_cast<uint64_t>(lo) << (3 * E * r);
      }
      if (lane % LPG == 0) {
        uint16_t* dst = sp16 + (lane / LPG) * 3;
        dst[0] = static_cast<uint16_t>(g);
        dst[1] = static_cast<uint16_t>(g >> 16);
        dst[2] = static_cast<uint16_t>(g >> 32);
      }
    }
    if (lane == 0) sp16[tq.mse_bytes / 2] = float_to_bf16_bits(norm);
    return;
  }
  // V: asymmetric min / max quantisation of the raw vector.
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int j = 1; j < E; ++j) {
    mn = fminf(mn, v[j]);
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int qmax = (1 << tq.value_bits) - 1;
  const float scale = fmaxf((mx - mn) / static_cast<float>(qmax), 1e-8f);
  uint32_t qv[E];
#pragma unroll
  for (int j = 0; j < E; ++j) qv[j] = static_cast<uint32_t>(min(max(static_cast<int>(roundf((v[j] - mn) / scale)), 0), qmax));
  uint16_t* vd = reinterpret_cast<uint16_t*>(sp + tq.key_packed);
  if (tq.value_bits == 4) {
    uint32_t pk = 0;
#pragma unroll
    for (int j = 0; j < E; ++j) pk |= (qv[j] & 0xfu) << (4 * j);
    constexpr int LPW = 4 / E > 0 ? 4 / E : 1;
    uint32_t word = pk;
#pragma unroll
    for (int r = 1; r < LPW; ++r) word |= __shfl_down_sync(0xffffffffu, pk, r) << (4 * E * r);
    if constexpr (E >= 4) {
#pragma unroll
      for (int w = 0; w < E / 4; ++w) vd[(lane * E) / 4 + w] = static_cast<uint16_t>(pk >> (16 * w));
    } else {
      if (lane % LPW == 0) vd[lane / LPW] = static_cast<uint16_t>(word);
    }
  } else {
    uint64_t pk = 0;
#pragma unroll
    for (int j = 0; j < E; ++j) pk |= static_cast<uint64_t>(qv[j] & 7u) << (3 * j);
    constexpr int LPG = 16 / E;
    uint64_t g = pk;
#pragma unroll
    for (int r = 1; r < LPG; ++r) {
      const uint32_t lo = __shfl_down_sync(0xffffffffu, static_cast<uint32_t>(pk), r);
      g |= static_cast<uint64_t>(lo) << (3 * E * r);
    }
    if (lane % LPG == 0) {
      uint16_t* dst = vd + (lane / LPG) * 3;
      dst[0] = static_cast<uint16_t>(g);
      dst[1] = static_cast<uint16_t>(g >> 16);
      dst[2] = static_cast<uint16_t>(g >> 32);
    }
  }
  if (lane == 0) {
    vd[tq.val_bytes / 2] = float_to_bf16_bits(scale);
    vd[tq.val_bytes / 2 + 1] = float_to_bf16_bits(mn);
  }
}

template <typename TI>
void launch_store(const TI* qkv, int nsplit, int64_t split_stride, int T, int Hq, int Hkv, int D, const int32_t* pos,
                  const int32_t* slots, const float* cos_sin, bool neox, void* q_out, const TqDev& tq,
                  cudaStream_t st) {
  const int64_t warps = static_cast<int64_t>(T) * (Hq + 2 * Hkv);
  const int wpb = 8;
  const dim3 grid(static_cast<unsigned>((warps + wpb - 1) / wpb));
  auto* qo = static_cast<__nv_bfloat16*>(q_out);
  auto* c2 = reinterpret_cast<const float2*>(cos_sin);
  switch (D) {
    case 32: launch_k(rope_store_tq_kernel<TI, 1>, grid, dim3(32 * wpb), 0, st, qkv, nsplit, split_stride, T, Hq, Hkv, pos, slots, c2, static_cast<int>(neox), qo, tq); break;
    case 64: launch_k(rope_store_tq_kernel<TI, 2>, grid, dim3(32 * wpb), 0, st, qkv, nsplit, split_stride, T, Hq, Hkv, pos, slots, c2, static_cast<int>(neox), qo, tq); break;
    case 128: launch_k(rope_store_tq_kernel<TI, 4>, grid, dim3(32 * wpb), 0, st, qkv, nsplit, split_stride, T, Hq, Hkv, pos, slots, c2, static_cast<int>(neox), qo, tq); break;
    default: throw std::runtime_error("turboquant: head dim must be 32, 64 or 128");
  }
}

}  // namespace

void rope_store_tq(const void* qkv, bool qkv_f32, int nsplit, int64_t split_stride, int T, int Hq, int Hkv, int D,
                   const int32_t* pos, const int32_t* slots, const float* cos_sin, bool neox, void* q_out,
                   const TqDev& tq, cudaStream_t st) {
  if (T <= 0) return;
  VMC_CHECK(tq.key_fp8 || tq.key_bits == 3 || tq.key_bits == 4, "turboquant: key bits must be 3, 4 or fp8");
  VMC_CHECK(tq.value_bits == 3 || tq.value_bits == 4, "turboquant: value bits must be 3 or 4");
  VMC_CHECK(tq.slot % 2 == 0 && tq.mse_bytes % 2 == 0 && tq.key_packed % 2 == 0 && tq.val_bytes % 2 == 0,
            "turboquant: slot fields must be 2-byte aligned");
  if (qkv_f32)
    launch_store(static_cast<const float*>(qkv), nsplit, split_stride, T, Hq, Hkv, D, pos, slots, cos_sin, neox, q_out,
                 tq, st);
  else
    launch_store(static_cast<const __nv_bfloat16*>(qkv), 1, int64_t{0}, T, Hq, Hkv, D, pos, slots, cos_sin, neox,
                 q_out, tq, st);
}

}  // namespace vmc
