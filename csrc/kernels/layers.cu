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
// resid (fp32) += sum_j delta_j (bf16 or fp32, ndelta slices delta_stride apart; may be null);
// out = rmsnorm(resid) * w (bf16). One CTA per row. Vector path (H % 4 == 0, H <= 16 * threads):
// every load of the row (residual and all delta slices) is issued before the first add, and the
// row stays in registers between the sum of squares and the output, so a decode-sized call costs
// about one memory round trip.
constexpr int kNormMaxVec = 4;    // float4 per thread
constexpr int kNormMaxDelta = 8;  // delta slices summed with unrolled loads

template <typename TD>
__device__ __forceinline__ float4 ld_delta4(const TD* p, int64_t i4) {
  if constexpr (sizeof(TD) == 2) {
    const uint2 u = *reinterpret_cast<const uint2*>(p + 4 * i4);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
  } else {
    return *reinterpret_cast<const float4*>(p + 4 * i4);
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

template <typename TD>
__global__ void add_rmsnorm_vec_kernel(float* __restrict__ resid, const TD* __restrict__ delta, int ndelta,
                                       int64_t delta_stride, const float* __restrict__ w, int H, float eps,
                                       __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int nvec = H >> 2;
  float4* x = reinterpret_cast<float4*>(resid + static_cast<int64_t>(t) * H);
  __shared__ float red[32];
  float4 v[kNormMaxVec];
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int k = threadIdx.x + i * blockDim.x;
    v[i] = k < nvec ? x[k] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (delta != nullptr) {
#pragma unroll
    for (int j = 0; j < kNormMaxDelta; ++j) {
      if (j < ndelta) {
        const TD* dj = delta + j * delta_stride + static_cast<int64_t>(t) * H;
#pragma unroll
        for (int i = 0; i < kNormMaxVec; ++i) {
          const int k = threadIdx.x + i * blockDim.x;
          if (k < nvec) {
            const float4 d = ld_delta4(dj, k);
            v[i].x += d.x;
            v[i].y += d.y;
            v[i].z += d.z;
            v[i].w += d.w;
          }
        }
      }
    }
    for (int j = kNormMaxDelta; j < ndelta; ++j) {
      const TD* dj = delta + j * delta_stride + static_cast<int64_t>(t) * H;
      for (int i = 0; i < kNormMaxVec; ++i) {
        const int k = threadIdx.x + i * blockDim.x;
        if (k < nvec) {
          const float4 d = ld_delta4(dj, k);
          v[i].x += d.x;
          v[i].y += d.y;
          v[i].z += d.z;
          v[i].w += d.w;
        }
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxVec; ++i) {
    const int k = threadIdx.x + i * blockDim.x;
    if (k < nvec) {
      if (delta != nullptr) x[k] = v[i];
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / H + eps);
  if (out) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    uint2* o = reinterpret_cast<uint2*>(out + static_cast<int64_t>(t) * H);
#pragma unroll
    for (int i = 0; i < kNormMaxVec; ++i) {
      const int k = threadIdx.x + i * blockDim.x;
      if (k < nvec) {
        const float4 g = w4[k];
        o[k] = make_uint2(pack_bf16x2(v[i].x * inv * g.x, v[i].y * inv * g.y),
                          pack_bf16x2(v[i].z * inv * g.z, v[i].w * inv * g.w));
      }
    }
  }
}

// Scalar path for hidden sizes the vector path does not cover.
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
  const float inv = rsqrtf(block_sum(ss, red) / H + eps);
  if (out) {
    for (int k = threadIdx.x; k < H; k += blockDim.x)
      out[static_cast<int64_t>(t) * H + k] = __float2bfloat16(x[k] * inv * w[k]);
  }
}

// ---- RoPE + KV store -----------------------------------------------------------------------
// qkv: [T, (Hq + 2 Hkv) * D] (bf16 or fp32; fp32 input may be nsplit split-K partials
// split_stride apart). One warp per (token, head); each lane owns groups of 4 dimensions: 4
// consecutive ones (two adjacent rotation pairs), or with neox (pairs x_i, x_{i + D/2}) dimensions
// 2q, 2q+1 and their partners. Q heads are rotated into q_out [T, Hq, D]; K heads rotated and V
// heads copied into the paged cache at the token's slot (skipped when slot < 0). All partial loads
// of a lane are issued before the first add.
template <typename TI>
__device__ __forceinline__ void ld2(const TI* p, int64_t i, float& a, float& b) {
  if constexpr (sizeof(TI) == 2) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p + i);
    a = __uint_as_float(u << 16);
    b = __uint_as_float(u & 0xffff0000u);
  } else {
    const float2 f = *reinterpret_cast<const float2*>(p + i);
    a = f.x;
    b = f.y;
  }
}

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
  __nv_bfloat16* dst;
  bool rotate = true;
  if (h < Hq) {
    dst = q_out + (static_cast<int64_t>(t) * Hq + h) * D;
  } else {
    const int slot = slots[t];
    if (slot < 0) return;
    const int blk = slot / 16, off = slot % 16;
    const int kvsel = h < Hq + Hkv ? 0 : 1;
    const int kvh = h - Hq - kvsel * Hkv;
    dst = kv + ((static_cast<int64_t>(blk) * 2 + kvsel) * Hkv + kvh) * 16 * D + static_cast<int64_t>(off) * D;
    rotate = kvsel == 0;
  }
  const int half = D / 2;
  for (int q = lane; q < D / 4; q += 32) {
    // element indices of this lane's two rotation pairs: (a0, a1) and (b0, b1)
    const int a0 = neox ? 2 * q : 4 * q, a1 = neox ? 2 * q + half : 4 * q + 1;
    const int b0 = neox ? 2 * q + 1 : 4 * q + 2, b1 = neox ? 2 * q + 1 + half : 4 * q + 3;
    // two contiguous element pairs to load: neox (a0, b0) and (a1, b1); else (a0, a1) and (b0, b1)
    const int l0 = a0, l1 = neox ? a1 : b0;
    float x[4];  // values at a0, a1, b0, b1
    float u0, u1, u2, u3;
    ld2(src, l0, u0, u1);
    ld2(src, l1, u2, u3);
    if constexpr (sizeof(TI) == 4) {
#pragma unroll
      for (int sp = 1; sp < 8; ++sp) {
        if (sp < nsplit) {
          float w0, w1, w2, w3;
          ld2(src + sp * split_stride, l0, w0, w1);
          ld2(src + sp * split_stride, l1, w2, w3);
          u0 += w0;
          u1 += w1;
          u2 += w2;
          u3 += w3;
        }
      }
      for (int sp = 8; sp < nsplit; ++sp) {
        float w0, w1, w2, w3;
        ld2(src + sp * split_stride, l0, w0, w1);
        ld2(src + sp * split_stride, l1, w2, w3);
        u0 += w0;
        u1 += w1;
        u2 += w2;
        u3 += w3;
      }
    }
    if (neox) { x[0] = u0; x[2] = u1; x[1] = u2; x[3] = u3; }
    else { x[0] = u0; x[1] = u1; x[2] = u2; x[3] = u3; }
    float y[4];
    if (rotate) {
      const int ia = neox ? 2 * q : 2 * q, ib = ia + 1;  // rotation pair indices in the table
      const float2 ca = c[ia], cb = c[ib];
      y[0] = x[0] * ca.x - x[1] * ca.y;
      y[1] = x[0] * ca.y + x[1] * ca.x;
      y[2] = x[2] * cb.x - x[3] * cb.y;
      y[3] = x[2] * cb.y + x[3] * cb.x;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = x[i];
    }
    if (neox) {
      *reinterpret_cast<uint32_t*>(dst + a0) = pack_bf16x2(y[0], y[2]);
      *reinterpret_cast<uint32_t*>(dst + a1) = pack_bf16x2(y[1], y[3]);
    } else {
      *reinterpret_cast<uint2*>(dst + a0) = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    }
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
  if (H % 4 == 0 && H <= 4 * kNormMaxVec * threads) {
    if (delta_f32 || delta == nullptr)
      launch_k(add_rmsnorm_vec_kernel<float>, dim3(T), dim3(threads), 0, st, resid, static_cast<const float*>(delta),
               delta ? ndelta : 0, delta_stride, w, H, eps, static_cast<__nv_bfloat16*>(out));
    else
      launch_k(add_rmsnorm_vec_kernel<__nv_bfloat16>, dim3(T), dim3(threads), 0, st, resid,
               static_cast<const __nv_bfloat16*>(delta), ndelta, delta_stride, w, H, eps,
               static_cast<__nv_bfloat16*>(out));
    return;
  }
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
  VMC_CHECK(D % 8 == 0, "rope_store: head dim must be a multiple of 8");
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
