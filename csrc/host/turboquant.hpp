// TurboQuant KV-cache layout and quantiser tables (host side).
//
// Slot layout (kept byte-identical to the reference, include/vm_c/memory/kv_cache_manager.hpp:
// 121-162 and src/cuda/turboquant_kernels.cu:39-45): one slot per (block, offset, kv head), NHD
// order, slot = [K packed | K norm (2 B) | V packed | V scale (2 B) | V min (2 B)] padded to an
// even size. K is the unit-normalised, rotated key quantised to Lloyd-Max centroids for N(0, 1/d)
// (4 or 3 bits; 3-bit values packed 8 per 3 bytes, little-endian), or fp8 e4m3 for k8v4 (no norm,
// no rotation); V is asymmetric min/max quantisation per vector (4 or 3 bits).
#pragma once
#include <string>
#include <vector>

namespace vmc {

struct TqLayout {
  int head_dim = 0;
  int key_bits = 4;
  int value_bits = 4;
  bool norm_correction = true;
  bool key_fp8 = false;
  int n_centroids = 16;
  int mse_bytes = 0;
  int key_packed = 0;
  int val_bytes = 0;
  int value_packed = 0;
  int slot = 0;
  int slot_aligned = 0;

  // method: turboquant_4bit_nc | turboquant_k8v4 | turboquant_k3v4_nc | turboquant_3bit_nc
  static TqLayout from_method(int head_dim, const std::string& method);
};

bool is_turboquant_method(const std::string& method);

// Lloyd-Max (minimum-MSE) scalar quantiser of N(0, sigma^2) with 2^bits levels: the centroids in
// increasing order. Fixed point of c_i = E[x | b_{i-1} < x < b_i], b_i = (c_i + c_{i+1}) / 2, with
// the conditional means in closed form (Gaussian pdf / cdf), iterated to convergence.
std::vector<double> lloyd_max_gaussian(int bits, double sigma);

}  // namespace vmc
