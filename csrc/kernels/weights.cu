// Load-time weight kernels: GGUF row data -> tiled on-device formats (weight_formats.cuh), and
// on-device quantisers used to build seeded random-init checkpoints directly in GGUF block format.
//
// The quantisers implement exactly the host quantisers of csrc/host/quants.cpp (same operations,
// round-to-nearest-even), so a tensor quantised here equals the same tensor quantised on the CPU.
#include "common.cuh"
#include "weight_formats.cuh"
#include "weights.h"

namespace vmc {
namespace {

// fp16 / bf16 fields of the block formats always sit at even offsets: use 16-bit accesses.
__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}
__device__ __forceinline__ void st_u16(uint8_t* p, unsigned short u) { *reinterpret_cast<unsigned short*>(p) = u; }

// ---- repack: GGUF rows -> tiles -------------------------------------------------------------

// One thread per (row, 256-element block).
__global__ void repack_q4k_kernel(const uint8_t* __restrict__ src, int N, int KB, uint8_t* __restrict__ dst) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int Np = (N + 127) / 128 * 128;
  if (idx >= static_cast<int64_t>(Np) * KB) return;
  const int n = static_cast<int>(idx / KB), kb = static_cast<int>(idx % KB);
  uint8_t* o = dst + ((static_cast<int64_t>(n / 128) * KB + kb) * 128 + (n % 128)) * 160;
  if (n >= N) {
    for (int i = 0; i < 160; ++i) o[i] = 0;
    return;
  }
  const uint8_t* s = src + (static_cast<int64_t>(n) * KB + kb) * 144;
  // GGUF Q4_K header: fp16 d, fp16 dmin, 12 bytes packing eight 6-bit (scale, min) pairs.
  const float d = ld_half(s), dmin = ld_half(s + 2);
  const uint8_t* sc = s + 4;
  for (int j = 0; j < 8; ++j) {
    int scv, mv;
    if (j < 4) {
      scv = sc[j] & 63;
      mv = sc[j + 4] & 63;
    } else {
      scv = (sc[j + 4] & 0x0f) | ((sc[j - 4] >> 6) << 4);
      mv = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    st_u16(o + 4 * j, __bfloat16_as_ushort(__float2bfloat16(d * static_cast<float>(scv))));
    st_u16(o + 4 * j + 2, __bfloat16_as_ushort(__float2bfloat16(-dmin * static_cast<float>(mv))));
  }
  for (int g = 0; g < 32; ++g) {  // nibble bytes, 4-byte groups reordered (0,2,1,3)
    const uint8_t* q = s + 16 + 4 * g;
    uint8_t* p = o + 32 + 4 * g;
    p[0] = q[0];
    p[1] = q[2];
    p[2] = q[1];
    p[3] = q[3];
  }
}

__global__ void repack_q6k_kernel(const uint8_t* __restrict__ src, int N, int KB, uint8_t* __restrict__ dst) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int Np = (N + 127) / 128 * 128;
  if (idx >= static_cast<int64_t>(Np) * KB) return;
  const int n = static_cast<int>(idx / KB), kb = static_cast<int>(idx % KB);
  uint8_t* o = dst + ((static_cast<int64_t>(n / 128) * KB + kb) * 128 + (n % 128)) * 224;
  if (n >= N) {
    for (int i = 0; i < 224; ++i) o[i] = 0;
    return;
  }
  const uint8_t* b = src + (static_cast<int64_t>(n) * KB + kb) * 210;
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  const float d = ld_half(b + 208);
  uint8_t q[256];
  for (int e = 0; e < 256; ++e) {
    const int h = e / 128, r = e % 128, k = r / 32, l = r % 32;
    const int lo = (ql[64 * h + l + 32 * (k & 1)] >> (4 * (k >> 1))) & 0x0f;
    const int hi = (qh[32 * h + l] >> (2 * k)) & 3;
    q[e] = static_cast<uint8_t>(lo | (hi << 4));
  }
  for (int g = 0; g < 32; ++g) {  // low nibbles, 8-element groups
    const uint8_t* e = q + 8 * g;
    o[4 * g + 0] = static_cast<uint8_t>((e[0] & 15) | ((e[4] & 15) << 4));
    o[4 * g + 1] = static_cast<uint8_t>((e[2] & 15) | ((e[6] & 15) << 4));
    o[4 * g + 2] = static_cast<uint8_t>((e[1] & 15) | ((e[5] & 15) << 4));
    o[4 * g + 3] = static_cast<uint8_t>((e[3] & 15) | ((e[7] & 15) << 4));
  }
  for (int g = 0; g < 16; ++g) {  // high 2-bit fields, 16-element groups
    const uint8_t* e = q + 16 * g;
    uint32_t V = 0;
    for (int k = 0; k < 8; ++k) {
      V |= static_cast<uint32_t>(e[2 * k] >> 4) << (2 * k);
      V |= static_cast<uint32_t>(e[2 * k + 1] >> 4) << (16 + 2 * k);
    }
    for (int i = 0; i < 4; ++i) o[128 + 4 * g + i] = static_cast<uint8_t>(V >> (8 * i));
  }
  for (int g = 0; g < 16; ++g) {
    st_u16(o + 192 + 2 * g, __bfloat16_as_ushort(__float2bfloat16(d * static_cast<float>(sc[g]))));
  }
}

// One thread per (row, 256-element chunk = 8 GGUF Q8_0 blocks). K32 = number of 32-blocks per row.
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ src, int N, int K32, int KC, uint8_t* __restrict__ dst) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int Np = (N + 127) / 128 * 128;
  if (idx >= static_cast<int64_t>(Np) * KC) return;
  const int n = static_cast<int>(idx / KC), kc = static_cast<int>(idx % KC);
  uint8_t* o = dst + ((static_cast<int64_t>(n / 128) * KC + kc) * 128 + (n % 128)) * 272;
  for (int j = 0; j < 8; ++j) {
    const int blk = kc * 8 + j;
    if (n >= N || blk >= K32) {
      st_u16(o + 2 * j, 0);
      for (int i = 0; i < 32; ++i) o[16 + 32 * j + i] = 0;
      continue;
    }
    const uint8_t* b = src + (static_cast<int64_t>(n) * K32 + blk) * 34;
    st_u16(o + 2 * j, __bfloat16_as_ushort(__float2bfloat16(ld_half(b))));
    for (int g = 0; g < 8; ++g) {
      const uint8_t* q = b + 2 + 4 * g;
      uint8_t* p = o + 16 + 32 * j + 4 * g;
      p[0] = q[0];
      p[1] = q[2];
      p[2] = q[1];
      p[3] = q[3];
    }
  }
}

// One thread per 16-byte output chunk (8 bf16 values). src_type: 0 f32, 1 f16, 30 bf16.
__global__ void repack_bf16_kernel(const void* __restrict__ src, int src_type, int N, int K, int KT,
                                   uint8_t* __restrict__ dst) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int Np = (N + 127) / 128 * 128;
  const int64_t total = static_cast<int64_t>(Np / 128) * KT * 128 * 8;
  if (idx >= total) return;
  const int c = static_cast<int>(idx % 8);
  const int r = static_cast<int>((idx / 8) % 128);
  const int64_t tile = idx / (8 * 128);
  const int kt = static_cast<int>(tile % KT);
  const int nt = static_cast<int>(tile / KT);
  const int n = nt * 128 + r;
  const int k0 = kt * 64 + c * 8;
  uint32_t w[4];
  for (int i = 0; i < 4; ++i) {
    float v[2];
    for (int j = 0; j < 2; ++j) {
      const int k = k0 + 2 * i + j;
      float x = 0.f;
      if (n < N && k < K) {
        const int64_t off = static_cast<int64_t>(n) * K + k;
        if (src_type == 0) x = static_cast<const float*>(src)[off];
        else if (src_type == 1) x = __half2float(static_cast<const __half*>(src)[off]);
        else x = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[off]);
      }
      v[j] = x;
    }
    w[i] = pack_bf16x2(v[0], v[1]);
  }
  uint8_t* o = dst + tile * 16384 + sw128_offset(r, c);
  *reinterpret_cast<uint4*>(o) = make_uint4(w[0], w[1], w[2], w[3]);
}

// ---- on-device quantisers (GGUF block formats) ------------------------------------------------

__device__ __forceinline__ void st_half(uint8_t* p, float f) { st_u16(p, __half_as_ushort(__float2half_rn(f))); }
__device__ __forceinline__ float rt_half(float f) { return __half2float(__float2half_rn(f)); }
__device__ __forceinline__ int rne(float x) { return __float2int_rn(x); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void quant_q8_0_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* v = x + b * 32;
  uint8_t* o = out + b * 34;
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
  const float d = rt_half(amax / 127.f);
  st_half(o, amax / 127.f);
  const float id = d > 0.f ? 1.f / d : 0.f;
  for (int j = 0; j < 32; ++j) o[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(clampi(rne(v[j] * id), -127, 127)));
}

__global__ void quant_q4k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* v = x + b * 256;
  uint8_t* o = out + b * 144;
  float scale[8], minv[8];
  float max_scale = 0.f, max_min = 0.f;
  for (int s = 0; s < 8; ++s) {
    float mn = v[32 * s], mx = v[32 * s];
    for (int l = 1; l < 32; ++l) {
      mn = fminf(mn, v[32 * s + l]);
      mx = fmaxf(mx, v[32 * s + l]);
    }
    if (mn > 0.f) mn = 0.f;
    scale[s] = (mx - mn) / 15.f;
    minv[s] = -mn;
    max_scale = fmaxf(max_scale, scale[s]);
    max_min = fmaxf(max_min, minv[s]);
  }
  st_half(o, max_scale / 63.f);
  st_half(o + 2, max_min / 63.f);
  const float d = rt_half(max_scale / 63.f), dmin = rt_half(max_min / 63.f);
  int sc[8], mq[8];
  for (int s = 0; s < 8; ++s) {
    sc[s] = d > 0.f ? clampi(rne(scale[s] / d), 0, 63) : 0;
    mq[s] = dmin > 0.f ? clampi(rne(minv[s] / dmin), 0, 63) : 0;
  }
  for (int j = 0; j < 4; ++j) {
    o[4 + j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    o[4 + j + 4] = static_cast<uint8_t>((mq[j] & 63) | ((mq[j + 4] >> 4) << 6));
    o[4 + j + 8] = static_cast<uint8_t>((sc[j + 4] & 15) | ((mq[j + 4] & 15) << 4));
  }
  for (int p = 0; p < 4; ++p) {
    const float ds0 = d * sc[2 * p], dm0 = dmin * mq[2 * p];
    const float ds1 = d * sc[2 * p + 1], dm1 = dmin * mq[2 * p + 1];
    const float i0 = ds0 > 0.f ? 1.f / ds0 : 0.f, i1 = ds1 > 0.f ? 1.f / ds1 : 0.f;
    for (int l = 0; l < 32; ++l) {
      const int q0 = clampi(rne((v[64 * p + l] + dm0) * i0), 0, 15);
      const int q1 = clampi(rne((v[64 * p + 32 + l] + dm1) * i1), 0, 15);
      o[16 + 32 * p + l] = static_cast<uint8_t>(q0 | (q1 << 4));
    }
  }
}

__global__ void quant_q6k_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* v = x + b * 256;
  uint8_t* o = out + b * 210;
  float gscale[16];
  float max_abs_scale = 0.f;
  for (int g = 0; g < 16; ++g) {
    float amax = 0.f;
    for (int l = 0; l < 16; ++l) amax = fmaxf(amax, fabsf(v[16 * g + l]));
    gscale[g] = amax / 31.f;
    max_abs_scale = fmaxf(max_abs_scale, gscale[g]);
  }
  const float d = rt_half(max_abs_scale / 127.f);
  uint8_t q[256];
  for (int g = 0; g < 16; ++g) {
    const int s = d > 0.f ? clampi(rne(gscale[g] / d), 0, 127) : 0;
    o[192 + g] = static_cast<uint8_t>(static_cast<int8_t>(s));
    const float eff = d * s;
    const float ie = eff > 0.f ? 1.f / eff : 0.f;
    for (int l = 0; l < 16; ++l) q[16 * g + l] = static_cast<uint8_t>(clampi(rne(v[16 * g + l] * ie), -32, 31) + 32);
  }
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      const int q1 = q[128 * h + l], q2 = q[128 * h + 32 + l], q3 = q[128 * h + 64 + l], q4 = q[128 * h + 96 + l];
      o[64 * h + l] = static_cast<uint8_t>((q1 & 15) | ((q3 & 15) << 4));
      o[64 * h + 32 + l] = static_cast<uint8_t>((q2 & 15) | ((q4 & 15) << 4));
      o[128 + 32 * h + l] = static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  st_half(o + 208, max_abs_scale / 127.f);
}

// Dequantise tiled formats back to bf16 rows (diagnostics / tests of the repack).
__global__ void untile_bf16_kernel(const uint8_t* __restrict__ tiles, int N, int K, int KT, __nv_bfloat16* __restrict__ out) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(N) * K) return;
  const int n = static_cast<int>(idx / K), k = static_cast<int>(idx % K);
  const int nt = n / 128, r = n % 128, kt = k / 64, kk = k % 64;
  const uint8_t* t = tiles + (static_cast<int64_t>(nt) * KT + kt) * 16384;
  const uint8_t* p = t + sw128_offset(r, kk / 8) + (kk % 8) * 2;
  out[idx] = *reinterpret_cast<const __nv_bfloat16*>(p);
}

inline int blocks_for(int64_t n, int t) { return static_cast<int>((n + t - 1) / t); }

}  // namespace

int64_t tiled_weight_bytes(int wf, int N, int K) {
  const int64_t NT = (N + 127) / 128;
  const int64_t KC = (K + wf_chunk(wf) - 1) / wf_chunk(wf);
  return NT * KC * wf_tile_bytes(wf);
}

void repack_weight(int wf, int src_type, const void* src, int N, int K, void* dst, cudaStream_t st) {
  const int Np = (N + 127) / 128 * 128;
  const int T = 128;
  switch (wf) {
    case kWfQ4K: {
      VMC_CHECK(src_type == 12 && K % 256 == 0, "repack: Q4_K needs K % 256 == 0");
      const int KB = K / 256;
      repack_q4k_kernel<<<blocks_for(static_cast<int64_t>(Np) * KB, T), T, 0, st>>>(static_cast<const uint8_t*>(src), N, KB, static_cast<uint8_t*>(dst));
      break;
    }
    case kWfQ6K: {
      VMC_CHECK(src_type == 14 && K % 256 == 0, "repack: Q6_K needs K % 256 == 0");
      const int KB = K / 256;
      repack_q6k_kernel<<<blocks_for(static_cast<int64_t>(Np) * KB, T), T, 0, st>>>(static_cast<const uint8_t*>(src), N, KB, static_cast<uint8_t*>(dst));
      break;
    }
    case kWfQ8_0: {
      VMC_CHECK(src_type == 8 && K % 32 == 0, "repack: Q8_0 needs K % 32 == 0");
      const int K32 = K / 32, KC = (K + 255) / 256;
      repack_q8_0_kernel<<<blocks_for(static_cast<int64_t>(Np) * KC, T), T, 0, st>>>(static_cast<const uint8_t*>(src), N, K32, KC, static_cast<uint8_t*>(dst));
      break;
    }
    case kWfBF16: {
      VMC_CHECK(src_type == 0 || src_type == 1 || src_type == 30, "repack: bf16 tiles need an F32/F16/BF16 source");
      const int KT = (K + 63) / 64;
      const int64_t total = static_cast<int64_t>(Np / 128) * KT * 128 * 8;
      repack_bf16_kernel<<<blocks_for(total, 256), 256, 0, st>>>(src, src_type, N, K, KT, static_cast<uint8_t*>(dst));
      break;
    }
    default: throw std::runtime_error("repack: unknown weight format");
  }
  VMC_CUDA_CHECK(cudaGetLastError());
}

void untile_bf16(const void* tiles, int N, int K, void* out, cudaStream_t st) {
  const int KT = (K + 63) / 64;
  untile_bf16_kernel<<<blocks_for(static_cast<int64_t>(N) * K, 256), 256, 0, st>>>(
      static_cast<const uint8_t*>(tiles), N, K, KT, static_cast<__nv_bfloat16*>(out));
  VMC_CUDA_CHECK(cudaGetLastError());
}

void quantize_blocks(int gtype, const float* x, int64_t n, void* out, cudaStream_t st) {
  switch (gtype) {
    case 8:
      VMC_CHECK(n % 32 == 0, "quantize: Q8_0 needs n % 32 == 0");
      quant_q8_0_kernel<<<blocks_for(n / 32, 128), 128, 0, st>>>(x, n / 32, static_cast<uint8_t*>(out));
      break;
    case 12:
      VMC_CHECK(n % 256 == 0, "quantize: Q4_K needs n % 256 == 0");
      quant_q4k_kernel<<<blocks_for(n / 256, 128), 128, 0, st>>>(x, n / 256, static_cast<uint8_t*>(out));
      break;
    case 14:
      VMC_CHECK(n % 256 == 0, "quantize: Q6_K needs n % 256 == 0");
      quant_q6k_kernel<<<blocks_for(n / 256, 128), 128, 0, st>>>(x, n / 256, static_cast<uint8_t*>(out));
      break;
    default: throw std::runtime_error("quantize: unsupported GGUF type on device");
  }
  VMC_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vmc
