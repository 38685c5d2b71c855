// TurboQuant cache description passed from the host to the store and attention kernels (plain
// struct: included by host-compiled code too).
#pragma once
#include <stdint.h>

namespace vmc {

struct TqDev {
  uint8_t* cache;          // this layer: [num_blocks][16][Hkv][slot] bytes
  int slot;                // slot bytes (even)
  int mse_bytes;           // packed K bytes
  int key_packed;          // mse_bytes + 2 (norm), or head_dim for fp8 keys
  int val_bytes;           // packed V bytes
  int key_bits, value_bits;
  int norm_correction;     // renormalise the reconstructed unit key before scaling by the norm
  int key_fp8;             // keys stored as fp8 e4m3 (k8v4): no rotation, no norm
  const float* centroids;  // [2^key_bits] Lloyd-Max centroids for N(0, 1/d)
  const float* midpoints;  // [2^key_bits - 1]
  uint32_t rot_seed;       // 0: plain normalised Hadamard; else per (layer, kv head) random signs first
  int layer;
};

}  // namespace vmc
