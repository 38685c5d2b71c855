// GGUF tensor type ids and block geometry.
//
// The numeric ids and the byte layout of every block are fixed by the GGUF file
// format (a checkpoint written by any GGUF producer must load here), so they match
// the reference's vendored ggml (ggml/include/ggml.h `enum ggml_type`) and the
// reference's own block structs (include/vm_c/core/ggml_dequant.hpp:43-115).
#pragma once
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace vmc {

enum class GType : uint32_t {
  F32 = 0, F16 = 1, Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q8_1 = 9,
  Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, Q8_K = 15,
  IQ4_NL = 20, IQ4_XS = 23, I8 = 24, I16 = 25, I32 = 26, I64 = 27, F64 = 28, BF16 = 30,
};

struct GTypeTraits {
  const char* name;
  int block_elems;   // elements per block
  int block_bytes;   // bytes per block
};

inline GTypeTraits gtype_traits(GType t) {
  switch (t) {
    case GType::F32: return {"F32", 1, 4};
    case GType::F16: return {"F16", 1, 2};
    case GType::BF16: return {"BF16", 1, 2};
    case GType::F64: return {"F64", 1, 8};
    case GType::I8: return {"I8", 1, 1};
    case GType::I16: return {"I16", 1, 2};
    case GType::I32: return {"I32", 1, 4};
    case GType::I64: return {"I64", 1, 8};
    case GType::Q4_0: return {"Q4_0", 32, 18};
    case GType::Q4_1: return {"Q4_1", 32, 20};
    case GType::Q5_0: return {"Q5_0", 32, 22};
    case GType::Q5_1: return {"Q5_1", 32, 24};
    case GType::Q8_0: return {"Q8_0", 32, 34};
    case GType::Q8_1: return {"Q8_1", 32, 36};
    case GType::Q2_K: return {"Q2_K", 256, 84};
    case GType::Q3_K: return {"Q3_K", 256, 110};
    case GType::Q4_K: return {"Q4_K", 256, 144};
    case GType::Q5_K: return {"Q5_K", 256, 176};
    case GType::Q6_K: return {"Q6_K", 256, 210};
    case GType::Q8_K: return {"Q8_K", 256, 292};
    case GType::IQ4_NL: return {"IQ4_NL", 32, 18};
    case GType::IQ4_XS: return {"IQ4_XS", 256, 136};
  }
  throw std::runtime_error("unknown GGUF tensor type " + std::to_string(static_cast<uint32_t>(t)));
}

inline bool gtype_known(uint32_t t) {
  switch (t) {
    case 0: case 1: case 2: case 3: case 6: case 7: case 8: case 9: case 10: case 11:
    case 12: case 13: case 14: case 15: case 20: case 23: case 24: case 25: case 26:
    case 27: case 28: case 30:
      return true;
    default:
      return false;
  }
}

inline size_t gtype_row_bytes(GType t, int64_t n_elems) {
  auto tr = gtype_traits(t);
  if (n_elems % tr.block_elems != 0)
    throw std::runtime_error(std::string("row length not a multiple of the ") + tr.name +
                             " block size");
  return static_cast<size_t>(n_elems / tr.block_elems) * tr.block_bytes;
}

// IEEE half <-> float without relying on compiler intrinsics (host code).
inline float half_to_float(uint16_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
      man &= 0x3ff;
      bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  __builtin_memcpy(&f, &bits, 4);
  return f;
}

// Round-to-nearest-even float -> half.
inline uint16_t float_to_half(float f) {
  uint32_t x;
  __builtin_memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) return static_cast<uint16_t>(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
  if (absx >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // overflow -> inf
  if (absx < 0x38800000u) {  // subnormal or zero in half
    if (absx < 0x33000000u) return static_cast<uint16_t>(sign);
    // value = m * 2^(e-150); the half subnormal unit is 2^-24, so q = m >> (126 - e).
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7fffff) | 0x800000;
    int s = 126 - static_cast<int>(e);
    uint32_t q = m >> s;
    uint32_t rem = m & ((1u << s) - 1);
    uint32_t half = 1u << (s - 1);
    if (rem > half || (rem == half && (q & 1))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t e = (absx >> 23) - 127 + 15;
  uint32_t m = absx & 0x7fffff;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (q & 1))) ++q;
  return static_cast<uint16_t>(sign | q);
}

inline float bf16_to_float(uint16_t h) {
  uint32_t bits = static_cast<uint32_t>(h) << 16;
  float f;
  __builtin_memcpy(&f, &bits, 4);
  return f;
}

inline uint16_t float_to_bf16(float f) {
  uint32_t x;
  __builtin_memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((x >> 16) | 0x40);
  uint32_t lsb = (x >> 16) & 1;
  x += 0x7fff + lsb;
  return static_cast<uint16_t>(x >> 16);
}

}  // namespace vmc
