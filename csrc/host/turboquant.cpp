#include "turboquant.hpp"

#include <cmath>
#include <stdexcept>

namespace vmc {

bool is_turboquant_method(const std::string& m) {
  return m == "turboquant_4bit_nc" || m == "turboquant_k8v4" || m == "turboquant_k3v4_nc" ||
         m == "turboquant_3bit_nc";
}

TqLayout TqLayout::from_method(int head_dim, const std::string& method) {
  if (!is_turboquant_method(method)) throw std::invalid_argument("unknown TurboQuant method: " + method);
  if (head_dim % 16 != 0) throw std::invalid_argument("TurboQuant needs head_dim % 16 == 0");
  TqLayout l;
  l.head_dim = head_dim;
  if (method == "turboquant_k8v4") {
    l.key_bits = 8, l.value_bits = 4, l.norm_correction = false, l.key_fp8 = true;
  } else if (method == "turboquant_k3v4_nc") {
    l.key_bits = 3, l.value_bits = 4;
  } else if (method == "turboquant_3bit_nc") {
    l.key_bits = 3, l.value_bits = 3;
  } else {
    l.key_bits = 4, l.value_bits = 4;
  }
  l.n_centroids = 1 << l.key_bits;
  if (l.key_fp8) {
    l.mse_bytes = head_dim;
    l.key_packed = head_dim;
  } else {
    l.mse_bytes = (head_dim * l.key_bits + 7) / 8;
    l.key_packed = l.mse_bytes + 2;
  }
  l.val_bytes = (head_dim * l.value_bits + 7) / 8;
  l.value_packed = l.val_bytes + 4;
  l.slot = l.key_packed + l.value_packed;
  l.slot_aligned = l.slot + (l.slot % 2);
  return l;
}

namespace {
double pdf(double z) { return std::exp(-0.5 * z * z) / std::sqrt(2.0 * M_PI); }
double cdf(double z) { return 0.5 * std::erfc(-z / std::sqrt(2.0)); }
}  // namespace

std::vector<double> lloyd_max_gaussian(int bits, double sigma) {
  if (bits < 1 || bits > 8 || !(sigma > 0)) throw std::invalid_argument("lloyd_max_gaussian: bad arguments");
  const int n = 1 << bits;
  std::vector<double> c(n), b(n - 1);
  for (int i = 0; i < n; ++i) c[i] = sigma * (-3.0 + 6.0 * (i + 0.5) / n);
  for (int it = 0; it < 100000; ++it) {
    for (int i = 0; i + 1 < n; ++i) b[i] = 0.5 * (c[i] + c[i + 1]);
    double change = 0;
    for (int i = 0; i < n; ++i) {
      const double za = i == 0 ? -INFINITY : b[i - 1] / sigma;
      const double zb = i == n - 1 ? INFINITY : b[i] / sigma;
      const double pa = std::isinf(za) ? 0.0 : pdf(za), pb = std::isinf(zb) ? 0.0 : pdf(zb);
      const double mass = cdf(zb) - cdf(za);
      const double nc = mass > 0 ? sigma * (pa - pb) / mass : c[i];
      change = std::fmax(change, std::fabs(nc - c[i]));
      c[i] = nc;
    }
    if (change < 1e-15 * sigma) break;
  }
  return c;
}

}  // namespace vmc
