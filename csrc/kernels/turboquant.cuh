// TurboQuant KV cache: device-side layout description and helpers shared by the store (RoPE + rotate
// + quantise, turboquant.cu) and the attention kernels that read the compressed cache
// (attention.cu). The byte layout of a slot is described in csrc/host/turboquant.hpp.
#pragma once
#include <stdint.h>

#include "common.cuh"
#include "turboquant_types.h"

namespace vmc {



// Byte offset of the slot of (block, offset, kv head): NHD order.
__device__ __forceinline__ int64_t tq_slot_offset(const TqDev& t, int blk, int off, int kvh, int Hkv) {
  return ((static_cast<int64_t>(blk) * 16 + off) * Hkv + kvh) * t.slot;
}

// +-1 sign of dimension d of the random rotation of (layer, kv head): a stateless integer hash.
__device__ __forceinline__ float tq_sign(uint32_t seed, int layer, int kvh, int d) {
  if (seed == 0) return 1.f;
  uint32_t x = seed ^ (static_cast<uint32_t>(layer) * 0x9E3779B1u) ^ (static_cast<uint32_t>(kvh) * 0x85EBCA77u) ^
               (static_cast<uint32_t>(d) * 0xC2B2AE3Du);
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return (x & 1u) ? -1.f : 1.f;
}

// In-warp normalised Walsh-Hadamard transform of a D-vector held as v[E] per lane (element index
// lane * E + j, E = D / 32): y = H x / sqrt(D) with H the Sylvester Hadamard matrix.
template <int E>
__device__ __forceinline__ void tq_fwht(float (&v)[E], int lane) {
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      if ((j & h) == 0) {
        const float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
      v[j] = (lane & m) ? (o - v[j]) : (v[j] + o);
    }
  }
  const float s = rsqrtf(static_cast<float>(32 * E));
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] *= s;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16(f));
}

}  // namespace vmc
