#include "quants.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

namespace vmc {

const int8_t kIQ4NLValues[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                 1,    13,   25,  38,  53,  69,  89,  113};

namespace {

inline float rd_half(const uint8_t* p) {
  uint16_t h;
  std::memcpy(&h, p, 2);
  return half_to_float(h);
}
inline void wr_half(uint8_t* p, float f) {
  uint16_t h = float_to_half(f);
  std::memcpy(p, &h, 2);
}

// 6-bit scale/min pairs of the Q4_K / Q5_K super-block: eight scales and eight mins packed in
// 12 bytes. Sub-blocks 0-3 keep their low 6 bits in bytes 0-7; sub-blocks 4-7 keep their low
// nibble in bytes 8-11 and their top two bits in the spare top bits of bytes 0-7.
inline void k4_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}
inline void k4_pack_scale_min(const int* sc, const int* mn, uint8_t* s) {
  for (int j = 0; j < 4; ++j) {
    s[j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = static_cast<uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 0x0f) | ((mn[j + 4] & 0x0f) << 4));
  }
}

void deq_q4_0(const uint8_t* b, float* y) {
  float d = rd_half(b);
  const uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    y[j] = d * static_cast<float>((qs[j] & 0x0f) - 8);
    y[j + 16] = d * static_cast<float>((qs[j] >> 4) - 8);
  }
}
void deq_q4_1(const uint8_t* b, float* y) {
  float d = rd_half(b), m = rd_half(b + 2);
  const uint8_t* qs = b + 4;
  for (int j = 0; j < 16; ++j) {
    y[j] = d * static_cast<float>(qs[j] & 0x0f) + m;
    y[j + 16] = d * static_cast<float>(qs[j] >> 4) + m;
  }
}
void deq_q5(const uint8_t* b, float* y, bool has_min) {
  float d = rd_half(b);
  float m = has_min ? rd_half(b + 2) : 0.f;
  const uint8_t* p = b + (has_min ? 4 : 2);
  uint32_t qh;
  std::memcpy(&qh, p, 4);
  const uint8_t* qs = p + 4;
  for (int j = 0; j < 16; ++j) {
    int hi0 = (qh >> j) & 1;
    int hi1 = (qh >> (j + 16)) & 1;
    int q0 = (qs[j] & 0x0f) | (hi0 << 4);
    int q1 = (qs[j] >> 4) | (hi1 << 4);
    if (has_min) {
      y[j] = d * q0 + m;
      y[j + 16] = d * q1 + m;
    } else {
      y[j] = d * (q0 - 16);
      y[j + 16] = d * (q1 - 16);
    }
  }
}
void deq_q8_0(const uint8_t* b, float* y) {
  float d = rd_half(b);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 2);
  for (int j = 0; j < 32; ++j) y[j] = d * qs[j];
}
void deq_q8_1(const uint8_t* b, float* y) {
  float d = rd_half(b);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 4);
  for (int j = 0; j < 32; ++j) y[j] = d * qs[j];
}
// Q2_K: 16 groups of 16; each scale byte holds a 4-bit scale (low) and 4-bit min (high).
// Element e of the super-block: half h = e/128, within it bit-pair s = (e%128)/32 of byte
// qs[32h + e%32].
void deq_q2_k(const uint8_t* b, float* y) {
  const uint8_t* scales = b;
  const uint8_t* qs = b + 16;
  float d = rd_half(b + 80), dmin = rd_half(b + 82);
  for (int e = 0; e < 256; ++e) {
    int h = e / 128, r = e % 128, s = r / 32, l = r % 32;
    int g = e / 16;
    int q = (qs[32 * h + l] >> (2 * s)) & 3;
    y[e] = d * (scales[g] & 0x0f) * q - dmin * (scales[g] >> 4);
  }
}
// Q3_K: 2 low bits in qs (same placement as Q2_K), the third bit in hmask (bit index = e/32),
// 16 signed 6-bit scales packed in 12 bytes.
void q3k_scales(const uint8_t* s12, int* out) {
  for (int g = 0; g < 16; ++g) {
    int low = (g < 8) ? (s12[g] & 0x0f) : (s12[g - 8] >> 4);
    int high = (s12[8 + (g % 4)] >> (2 * (g / 4))) & 3;
    out[g] = (low | (high << 4)) - 32;
  }
}
void deq_q3_k(const uint8_t* b, float* y) {
  const uint8_t* hmask = b;
  const uint8_t* qs = b + 32;
  int sc[16];
  q3k_scales(b + 96, sc);
  float d = rd_half(b + 108);
  for (int e = 0; e < 256; ++e) {
    int h = e / 128, r = e % 128, s = r / 32, l = r % 32;
    int q = (qs[32 * h + l] >> (2 * s)) & 3;
    int hb = (hmask[l] >> (e / 32)) & 1;
    y[e] = d * sc[e / 16] * (q - (hb ? 0 : 4));
  }
}
void deq_q4_k(const uint8_t* b, float* y) {
  float d = rd_half(b), dmin = rd_half(b + 2);
  const uint8_t* sc12 = b + 4;
  const uint8_t* qs = b + 16;
  for (int p = 0; p < 4; ++p) {  // pairs of 32-element sub-blocks share 32 bytes of qs
    int s0, m0, s1, m1;
    k4_scale_min(sc12, 2 * p, s0, m0);
    k4_scale_min(sc12, 2 * p + 1, s1, m1);
    for (int l = 0; l < 32; ++l) {
      y[64 * p + l] = d * s0 * (qs[32 * p + l] & 0x0f) - dmin * m0;
      y[64 * p + 32 + l] = d * s1 * (qs[32 * p + l] >> 4) - dmin * m1;
    }
  }
}
void deq_q5_k(const uint8_t* b, float* y) {
  float d = rd_half(b), dmin = rd_half(b + 2);
  const uint8_t* sc12 = b + 4;
  const uint8_t* qh = b + 16;
  const uint8_t* qs = b + 48;
  for (int p = 0; p < 4; ++p) {
    int s0, m0, s1, m1;
    k4_scale_min(sc12, 2 * p, s0, m0);
    k4_scale_min(sc12, 2 * p + 1, s1, m1);
    for (int l = 0; l < 32; ++l) {
      int h0 = (qh[l] >> (2 * p)) & 1;
      int h1 = (qh[l] >> (2 * p + 1)) & 1;
      y[64 * p + l] = d * s0 * ((qs[32 * p + l] & 0x0f) | (h0 << 4)) - dmin * m0;
      y[64 * p + 32 + l] = d * s1 * ((qs[32 * p + l] >> 4) | (h1 << 4)) - dmin * m1;
    }
  }
}
// Q6_K: element e, half h = e/128, r = e%128, quarter k = r/32, l = r%32.
//   low nibble: ql[64h + l + 32*(k&1)], nibble (k>>1); high 2 bits: qh[32h + l] >> 2k.
void deq_q6_k(const uint8_t* b, float* y) {
  const uint8_t* ql = b;
  const uint8_t* qh = b + 128;
  const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
  float d = rd_half(b + 208);
  for (int e = 0; e < 256; ++e) {
    int h = e / 128, r = e % 128, k = r / 32, l = r % 32;
    int lo = (ql[64 * h + l + 32 * (k & 1)] >> (4 * (k >> 1))) & 0x0f;
    int hi = (qh[32 * h + l] >> (2 * k)) & 3;
    y[e] = d * sc[e / 16] * ((lo | (hi << 4)) - 32);
  }
}
void deq_q8_k(const uint8_t* b, float* y) {
  float d;
  std::memcpy(&d, b, 4);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 4);
  for (int j = 0; j < 256; ++j) y[j] = d * qs[j];
}
void deq_iq4_nl(const uint8_t* b, float* y) {
  float d = rd_half(b);
  const uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    y[j] = d * kIQ4NLValues[qs[j] & 0x0f];
    y[j + 16] = d * kIQ4NLValues[qs[j] >> 4];
  }
}
void deq_iq4_xs(const uint8_t* b, float* y) {
  float d = rd_half(b);
  uint16_t sh;
  std::memcpy(&sh, b + 2, 2);
  const uint8_t* sl = b + 4;
  const uint8_t* qs = b + 8;
  for (int ib = 0; ib < 8; ++ib) {
    int ls = ((sl[ib / 2] >> (4 * (ib % 2))) & 0x0f) | (((sh >> (2 * ib)) & 3) << 4);
    float dl = d * (ls - 32);
    for (int j = 0; j < 16; ++j) {
      y[32 * ib + j] = dl * kIQ4NLValues[qs[16 * ib + j] & 0x0f];
      y[32 * ib + j + 16] = dl * kIQ4NLValues[qs[16 * ib + j] >> 4];
    }
  }
}

// ---- quantisers ----

int nearest_int(float x) { return static_cast<int>(std::lrintf(x)); }

void q_q8_0(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[j]));
  uint16_t dh = float_to_half(amax / 127.f);
  std::memcpy(b, &dh, 2);
  float d = half_to_float(dh);
  float id = d > 0.f ? 1.f / d : 0.f;
  int8_t* qs = reinterpret_cast<int8_t*>(b + 2);
  for (int j = 0; j < 32; ++j) qs[j] = static_cast<int8_t>(std::clamp(nearest_int(x[j] * id), -127, 127));
}

void q_q4_0(const float* x, uint8_t* b) {
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[j]));
  uint16_t dh = float_to_half(amax / 7.f);
  std::memcpy(b, &dh, 2);
  float d = half_to_float(dh);
  float id = d > 0.f ? 1.f / d : 0.f;
  uint8_t* qs = b + 2;
  for (int j = 0; j < 16; ++j) {
    int q0 = std::clamp(nearest_int(x[j] * id) + 8, 0, 15);
    int q1 = std::clamp(nearest_int(x[j + 16] * id) + 8, 0, 15);
    qs[j] = static_cast<uint8_t>(q0 | (q1 << 4));
  }
}

void q_q4_k(const float* x, uint8_t* b) {
  float scale[8], minv[8];
  float max_scale = 0.f, max_min = 0.f;
  for (int s = 0; s < 8; ++s) {
    float mn = x[32 * s], mx = x[32 * s];
    for (int l = 1; l < 32; ++l) {
      mn = std::min(mn, x[32 * s + l]);
      mx = std::max(mx, x[32 * s + l]);
    }
    if (mn > 0.f) mn = 0.f;
    scale[s] = (mx - mn) / 15.f;
    minv[s] = -mn;
    max_scale = std::max(max_scale, scale[s]);
    max_min = std::max(max_min, minv[s]);
  }
  uint16_t dh = float_to_half(max_scale / 63.f);
  uint16_t mh = float_to_half(max_min / 63.f);
  std::memcpy(b, &dh, 2);
  std::memcpy(b + 2, &mh, 2);
  float d = half_to_float(dh), dmin = half_to_float(mh);
  int sc[8], mq[8];
  for (int s = 0; s < 8; ++s) {
    sc[s] = d > 0.f ? std::clamp(nearest_int(scale[s] / d), 0, 63) : 0;
    mq[s] = dmin > 0.f ? std::clamp(nearest_int(minv[s] / dmin), 0, 63) : 0;
  }
  k4_pack_scale_min(sc, mq, b + 4);
  uint8_t* qs = b + 16;
  uint8_t q[256];
  for (int s = 0; s < 8; ++s) {
    float ds = d * sc[s], dm = dmin * mq[s];
    float ids = ds > 0.f ? 1.f / ds : 0.f;
    for (int l = 0; l < 32; ++l)
      q[32 * s + l] = static_cast<uint8_t>(std::clamp(nearest_int((x[32 * s + l] + dm) * ids), 0, 15));
  }
  for (int p = 0; p < 4; ++p)
    for (int l = 0; l < 32; ++l) qs[32 * p + l] = static_cast<uint8_t>(q[64 * p + l] | (q[64 * p + 32 + l] << 4));
}

void q_q6_k(const float* x, uint8_t* b) {
  float gscale[16];
  float max_abs_scale = 0.f;
  for (int g = 0; g < 16; ++g) {
    float amax = 0.f;
    for (int l = 0; l < 16; ++l) amax = std::max(amax, std::fabs(x[16 * g + l]));
    gscale[g] = amax / 31.f;
    max_abs_scale = std::max(max_abs_scale, gscale[g]);
  }
  uint16_t dh = float_to_half(max_abs_scale / 127.f);
  float d = half_to_float(dh);
  int8_t* sc = reinterpret_cast<int8_t*>(b + 192);
  uint8_t q[256];
  for (int g = 0; g < 16; ++g) {
    int s = d > 0.f ? std::clamp(nearest_int(gscale[g] / d), 0, 127) : 0;
    sc[g] = static_cast<int8_t>(s);
    float eff = d * s;
    float ie = eff > 0.f ? 1.f / eff : 0.f;
    for (int l = 0; l < 16; ++l) q[16 * g + l] = static_cast<uint8_t>(std::clamp(nearest_int(x[16 * g + l] * ie), -32, 31) + 32);
  }
  uint8_t* ql = b;
  uint8_t* qh = b + 128;
  for (int h = 0; h < 2; ++h) {
    for (int l = 0; l < 32; ++l) {
      int q1 = q[128 * h + l], q2 = q[128 * h + 32 + l], q3 = q[128 * h + 64 + l], q4 = q[128 * h + 96 + l];
      ql[64 * h + l] = static_cast<uint8_t>((q1 & 0x0f) | ((q3 & 0x0f) << 4));
      ql[64 * h + 32 + l] = static_cast<uint8_t>((q2 & 0x0f) | ((q4 & 0x0f) << 4));
      qh[32 * h + l] = static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  }
  std::memcpy(b + 208, &dh, 2);
}

template <class F>
void parallel_rows(int64_t rows, int threads, F&& f) {
  if (threads <= 1 || rows < 64) {
    f(0, rows);
    return;
  }
  threads = static_cast<int>(std::min<int64_t>(threads, rows));
  std::vector<std::thread> ts;
  int64_t per = (rows + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    int64_t r0 = t * per, r1 = std::min(rows, r0 + per);
    if (r0 >= r1) break;
    ts.emplace_back([&, r0, r1] { f(r0, r1); });
  }
  for (auto& th : ts) th.join();
}

}  // namespace

void dequantize_row(GType t, const void* src, float* dst, int64_t n) {
  const uint8_t* s = static_cast<const uint8_t*>(src);
  auto tr = gtype_traits(t);
  if (n % tr.block_elems) throw std::runtime_error("dequantize_row: length not block aligned");
  int64_t nb = n / tr.block_elems;
  switch (t) {
    case GType::F32: std::memcpy(dst, src, n * 4); return;
    case GType::F16:
      for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, s + 2 * i, 2); dst[i] = half_to_float(h); }
      return;
    case GType::BF16:
      for (int64_t i = 0; i < n; ++i) { uint16_t h; std::memcpy(&h, s + 2 * i, 2); dst[i] = bf16_to_float(h); }
      return;
    default: break;
  }
  for (int64_t i = 0; i < nb; ++i) {
    const uint8_t* blk = s + i * tr.block_bytes;
    float* y = dst + i * tr.block_elems;
    switch (t) {
      case GType::Q4_0: deq_q4_0(blk, y); break;
      case GType::Q4_1: deq_q4_1(blk, y); break;
      case GType::Q5_0: deq_q5(blk, y, false); break;
      case GType::Q5_1: deq_q5(blk, y, true); break;
      case GType::Q8_0: deq_q8_0(blk, y); break;
      case GType::Q8_1: deq_q8_1(blk, y); break;
      case GType::Q2_K: deq_q2_k(blk, y); break;
      case GType::Q3_K: deq_q3_k(blk, y); break;
      case GType::Q4_K: deq_q4_k(blk, y); break;
      case GType::Q5_K: deq_q5_k(blk, y); break;
      case GType::Q6_K: deq_q6_k(blk, y); break;
      case GType::Q8_K: deq_q8_k(blk, y); break;
      case GType::IQ4_NL: deq_iq4_nl(blk, y); break;
      case GType::IQ4_XS: deq_iq4_xs(blk, y); break;
      default: throw std::runtime_error(std::string("dequantize_row: unsupported type ") + tr.name);
    }
  }
}

bool can_quantize(GType t) {
  switch (t) {
    case GType::F32: case GType::F16: case GType::BF16: case GType::Q8_0: case GType::Q4_0:
    case GType::Q4_K: case GType::Q6_K:
      return true;
    default:
      return false;
  }
}

void quantize_row(GType t, const float* src, void* dst, int64_t n) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  auto tr = gtype_traits(t);
  if (n % tr.block_elems) throw std::runtime_error("quantize_row: length not block aligned");
  switch (t) {
    case GType::F32: std::memcpy(dst, src, n * 4); return;
    case GType::F16:
      for (int64_t i = 0; i < n; ++i) { uint16_t h = float_to_half(src[i]); std::memcpy(d + 2 * i, &h, 2); }
      return;
    case GType::BF16:
      for (int64_t i = 0; i < n; ++i) { uint16_t h = float_to_bf16(src[i]); std::memcpy(d + 2 * i, &h, 2); }
      return;
    default: break;
  }
  int64_t nb = n / tr.block_elems;
  for (int64_t i = 0; i < nb; ++i) {
    const float* x = src + i * tr.block_elems;
    uint8_t* b = d + i * tr.block_bytes;
    switch (t) {
      case GType::Q8_0: q_q8_0(x, b); break;
      case GType::Q4_0: q_q4_0(x, b); break;
      case GType::Q4_K: q_q4_k(x, b); break;
      case GType::Q6_K: q_q6_k(x, b); break;
      default: throw std::runtime_error(std::string("quantize_row: unsupported type ") + tr.name);
    }
  }
}

void dequantize_tensor(GType t, const void* src, float* dst, int64_t rows, int64_t row_elems, int threads) {
  size_t rb = gtype_row_bytes(t, row_elems);
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r)
      dequantize_row(t, static_cast<const uint8_t*>(src) + r * rb, dst + r * row_elems, row_elems);
  });
}

void quantize_tensor(GType t, const float* src, void* dst, int64_t rows, int64_t row_elems, int threads) {
  size_t rb = gtype_row_bytes(t, row_elems);
  parallel_rows(rows, threads, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r)
      quantize_row(t, src + r * row_elems, static_cast<uint8_t*>(dst) + r * rb, row_elems);
  });
}

}  // namespace vmc
