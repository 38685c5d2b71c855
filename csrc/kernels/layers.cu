// Per-layer elementwise kernels: token embedding gather (dequantising GGUF rows), fused
// residual-add + RMSNorm, RoPE fused with the paged KV-cache store, standalone SwiGLU, row gather.
//
// Replaces ggml-cuda's get_rows (getrows.cu:6), rms_norm(+mul/+add) (norm.cu:77,502,562),
// rope(+set_rows) (rope.cu:44,116,670), set_rows (set-rows.cu:114) and unary swiglu (unary.cu:263),
// and vm_c's unreachable fused_qk_norm_rope_store_kernel (src/cuda/fused_attn_kernels.cu:40).
#include "common.cuh"
#include "layers.h"

namespace vmc {
namespace {

// ---- per-element GGUF dequant (row-major raw rows; used for embedding gathers) ----------------

// fp16 fields of the GGUF blocks sit at even offsets: one 16-bit load.
__device__ __forceinline__ float h2f(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}

__device__ float dq_elem(int type, const uint8_t* row, int k) {
  switch (type) {
    case 0: return reinterpret_cast<const float*>(row)[k];
    case 1: return __half2float(reinterpret_cast<const __half*>(row)[k]);
    case 30: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[k]);
    case 8: {
      const uint8_t* b = row + (k / 32) * 34;
      return h2f(b) * static_cast<float>(static_cast<int8_t>(b[2 + k % 32]));
    }
    case 12: {
      const uint8_t* b = row + (k / 256) * 144;
      const int e = k % 256, j = e / 32, l = e % 32, p = j / 2;
      const uint8_t* sc = b + 4;
      int s, m;
      if (j < 4) { s = sc[j] & 63; m = sc[j + 4] & 63; }
      else { s = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4); m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
      const int q = (b[16 + 32 * p + l] >> (4 * (j & 1))) & 15;
      return h2f(b) * s * q - h2f(b + 2) * m;
    }
    case 14: {
      const uint8_t* b = row + (k / 256) * 210;
      const int e = k % 256, h = e / 128, r = e % 128, kk = r / 32, l = r % 32;
      const int lo = (b[64 * h + l + 32 * (kk & 1)] >> (4 * (kk >> 1))) & 15;
      const int hi = (b[128 + 32 * h + l] >> (2 * kk)) & 3;
      return h2f(b + 208) * static_cast<float>(static_cast<int8_t>(b[192 + e / 16])) * ((lo | (hi << 4)) - 32);
    }
    default: return 0.f;
  }
}

__global__ void embed_kernel(const int32_t* __restrict__ ids, int T, const uint8_t* __restrict__ table, int type,
                             int64_t row_bytes, int H, float* __restrict__ resid, __nv_bfloat16* __restrict__ out_bf16) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  const uint8_t* row = table + static_cast<int64_t>(ids[t]) * row_bytes;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float v = dq_elem(type, row, k);
    if (resid) resid[static_cast<int64_t>(t) * H + k] = v;
    if (out_bf16) out_bf16[static_cast<int64_t>(t) * H + k] = __float2bfloat16(v);
  }
}

// ---- residual add + RMSNorm ------------------------------------------------------------------
// resid (fp32) += delta (bf16 or fp32, may be null); out = rmsnorm(resid) * w (bf16).
template <typename TD>
__global__ void add_rmsnorm_kernel(float* __restrict__ resid, const TD* __restrict__ delta, int ndelta,
                                   int64_t delta_stride, const float* __restrict__ w, int H, float eps,
                                   __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  float* x = resid + static_cast<int64_t>(t) * H;
  __shared__ float red[32];
  float ss = 0.f;
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    float v = x[k];
    for (int j = 0; j < ndelta; ++j) {
      const TD* dj = delta + j * delta_stride + static_cast<int64_t>(t) * H;
      if constexpr (sizeof(TD) == 2) v += __bfloat162float(dj[k]);
      else v += dj[k];
    }
    x[k] = v;
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / H + eps);
  if (out) {
    for (int k = threadIdx.x; k < H; k += blockDim.x)
      out[static_cast<int64_t>(t) * H + k] = __float2bfloat16(x[k] * inv * w[k]);
  }
}

// ---- RoPE + KV store -----------------------------------------------------------------------
// qkv: [T, (Hq + 2 Hkv) * D] (bf16 or fp32). One warp per (token, head). Q heads are rotated and
// written to q_out [T, Hq, D]; K heads rotated and V heads copied into the paged cache at the
// token's slot (skipped when slot < 0). neox = rotate halves (x_i, x_{i+D/2}) instead of pairs.
template <typename TI>
__global__ void rope_store_kernel(const TI* __restrict__ qkv, int nsplit, int64_t split_stride, int T, int Hq, int Hkv,
                                  int D, const int32_t* __restrict__ pos, const int32_t* __restrict__ slots,
                                  const float2* __restrict__ cs, int neox, __nv_bfloat16* __restrict__ q_out,
                                  __nv_bfloat16* __restrict__ kv) {
  pdl_trigger();
  pdl_wait();
  const int warps = blockDim.x >> 5;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int H = Hq + 2 * Hkv;
  if (gw >= static_cast<int64_t>(T) * H) return;
  const int t = static_cast<int>(gw / H), h = static_cast<int>(gw % H);
  const TI* src = qkv + static_cast<int64_t>(t) * H * D + static_cast<int64_t>(h) * D;
  const int p = pos[t];
  const float2* c = cs + static_cast<int64_t>(p) * (D / 2);
  auto ld = [&](int i) -> float {
    if constexpr (sizeof(TI) == 2) {
      return __bfloat162float(src[i]);
    } else {
      float v = src[i];
      for (int sp = 1; sp < nsplit; ++sp) v += src[sp * split_stride + i];
      return v;
    }
  };
  __nv_bfloat16* dst;
  if (h < Hq) {
    dst = q_out + (static_cast<int64_t>(t) * Hq + h) * D;
  } else {
    const int slot = slots[t];
    if (slot < 0) return;
    const int blk = slot / 16, off = slot % 16;
    const int kvsel = h < Hq + Hkv ? 0 : 1;
    const int kvh = h - Hq - kvsel * Hkv;
    dst = kv + ((static_cast<int64_t>(blk) * 2 + kvsel) * Hkv + kvh) * 16 * D + static_cast<int64_t>(off) * D;
    if (kvsel == 1) {
      for (int i = lane; i < D; i += 32) dst[i] = __float2bfloat16(ld(i));
      return;
    }
  }
  for (int i = lane; i < D / 2; i += 32) {
    const float2 cv = c[i];
    const int i0 = neox ? i : 2 * i;
    const int i1 = neox ? i + D / 2 : 2 * i + 1;
    const float x0 = ld(i0), x1 = ld(i1);
    dst[i0] = __float2bfloat16(x0 * cv.x - x1 * cv.y);
    dst[i1] = __float2bfloat16(x0 * cv.y + x1 * cv.x);
  }
}

// ---- SwiGLU on a [T, 2F] (gate | up) input ---------------------------------------------------
// interleaved: the row holds (gate_0, up_0, gate_1, up_1, ...) instead of (gate | up).
template <typename TI>
__global__ void swiglu_kernel(const TI* __restrict__ gu, int nsplit, int64_t split_stride, int64_t T, int F,
                              int interleaved, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= T * F) return;
  const int64_t t = i / F;
  const int f = static_cast<int>(i % F);
  const int64_t ig = interleaved ? t * 2 * F + 2 * f : t * 2 * F + f;
  const int64_t iu = interleaved ? ig + 1 : ig + F;
  float g, u;
  if constexpr (sizeof(TI) == 2) {
    g = __bfloat162float(gu[ig]);
    u = __bfloat162float(gu[iu]);
  } else {
    g = gu[ig];
    u = gu[iu];
    for (int sp = 1; sp < nsplit; ++sp) {
      g += gu[sp * split_stride + ig];
      u += gu[sp * split_stride + iu];
    }
  }
  out[i] = __float2bfloat16(__fdividef(g, 1.f + __expf(-g)) * u);
}

// ---- gather rows (bf16) --------------------------------------------------------------------
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int32_t* __restrict__ idx, int n,
                                   int H, __nv_bfloat16* __restrict__ dst) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  if (r >= n) return;
  const int64_t s = static_cast<int64_t>(idx[r]) * H;
  for (int k = threadIdx.x * 8; k < H; k += blockDim.x * 8) {
    if (k + 8 <= H && (H % 8) == 0) {
      *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * H + k) = *reinterpret_cast<const uint4*>(src + s + k);
    } else {
      for (int j = k; j < min(H, k + 8); ++j) dst[static_cast<int64_t>(r) * H + j] = src[s + j];
    }
  }
}

// ---- fp32 -> bf16 ----------------------------------------------------------------------------
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, int64_t n, __nv_bfloat16* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16(x[i]);
}

inline int nblk(int64_t n, int t) { return static_cast<int>((n + t - 1) / t); }

}  // namespace

void embed(const int32_t* ids, int T, const void* table, int gtype, int64_t row_bytes, int H, float* resid,
           void* out_bf16, cudaStream_t st) {
  if (T <= 0) return;
  launch_k(embed_kernel, dim3(T), dim3(256), 0, st, ids, T, static_cast<const uint8_t*>(table), gtype, row_bytes, H,
           resid, static_cast<__nv_bfloat16*>(out_bf16));
}

void add_rmsnorm(float* resid, const void* delta, bool delta_f32, int ndelta, int64_t delta_stride, const float* w,
                 int T, int H, float eps, void* out, cudaStream_t st) {
  if (T <= 0) return;
  const int threads = H >= 2048 ? 512 : 256;
  if (delta_f32 || delta == nullptr)
    launch_k(add_rmsnorm_kernel<float>, dim3(T), dim3(threads), 0, st, resid, static_cast<const float*>(delta),
             delta ? ndelta : 0, delta_stride, w, H, eps, static_cast<__nv_bfloat16*>(out));
  else
    launch_k(add_rmsnorm_kernel<__nv_bfloat16>, dim3(T), dim3(threads), 0, st, resid,
             static_cast<const __nv_bfloat16*>(delta), ndelta, delta_stride, w, H, eps, static_cast<__nv_bfloat16*>(out));
}

void rope_store(const void* qkv, bool qkv_f32, int nsplit, int64_t split_stride, int T, int Hq, int Hkv, int D,
                const int32_t* pos, const int32_t* slots, const float* cos_sin, bool neox, void* q_out, void* kv,
                cudaStream_t st) {
  if (T <= 0) return;
  const int64_t warps = static_cast<int64_t>(T) * (Hq + 2 * Hkv);
  const int wpb = 8;
  if (qkv_f32)
    launch_k(rope_store_kernel<float>, dim3(nblk(warps, wpb)), dim3(32 * wpb), 0, st, static_cast<const float*>(qkv),
             nsplit, split_stride, T, Hq, Hkv, D, pos, slots, reinterpret_cast<const float2*>(cos_sin),
             static_cast<int>(neox), static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(kv));
  else
    launch_k(rope_store_kernel<__nv_bfloat16>, dim3(nblk(warps, wpb)), dim3(32 * wpb), 0, st,
             static_cast<const __nv_bfloat16*>(qkv), 1, static_cast<int64_t>(0), T, Hq, Hkv, D, pos, slots,
             reinterpret_cast<const float2*>(cos_sin), static_cast<int>(neox), static_cast<__nv_bfloat16*>(q_out),
             static_cast<__nv_bfloat16*>(kv));
}

void swiglu(const void* gu, bool f32, int nsplit, int64_t split_stride, int64_t T, int F, bool interleaved, void* out,
            cudaStream_t st) {
  if (T <= 0) return;
  if (f32)
    launch_k(swiglu_kernel<float>, dim3(nblk(T * F, 256)), dim3(256), 0, st, static_cast<const float*>(gu), nsplit,
             split_stride, T, F, static_cast<int>(interleaved), static_cast<__nv_bfloat16*>(out));
  else
    launch_k(swiglu_kernel<__nv_bfloat16>, dim3(nblk(T * F, 256)), dim3(256), 0, st,
             static_cast<const __nv_bfloat16*>(gu), 1, static_cast<int64_t>(0), T, F, static_cast<int>(interleaved),
             static_cast<__nv_bfloat16*>(out));
}

void gather_rows(const void* src, const int32_t* idx, int n, int H, void* dst, cudaStream_t st) {
  if (n <= 0) return;
  launch_k(gather_rows_kernel, dim3(n), dim3(128), 0, st, static_cast<const __nv_bfloat16*>(src), idx, n, H,
           static_cast<__nv_bfloat16*>(dst));
}

void f32_to_bf16(const float* x, int64_t n, void* y, cudaStream_t st) {
  if (n <= 0) return;
  launch_k(f32_to_bf16_kernel, dim3(nblk(n, 256)), dim3(256), 0, st, x, n, static_cast<__nv_bfloat16*>(y));
}

}  // namespace vmc
