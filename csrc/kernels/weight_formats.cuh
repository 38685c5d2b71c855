// On-device weight formats used by the tcgen05 GEMM.
//
// At load time every linear weight [N, K] is repacked ("tiled") so that the bytes one CTA needs for
// one (128-row, K-chunk) tile are contiguous and 16-byte aligned: a single cp.async.bulk brings a
// whole tile into shared memory. N is padded to a multiple of 128 (zero rows), K to the chunk.
//
//  kBF16 : chunk = 64 K-elements. Tile = 128 rows x 128 bytes of bf16, already in the UMMA
//          K-major SWIZZLE_128B image (16-byte chunk c of row r stored at chunk c ^ (r & 7)).
//  kQ4K  : chunk = 256. Tile = 128 rows x 160 bytes: the 8 sub-block scales decoded at load time
//          into bf16 pairs (d * scale_j, -dmin * min_j) — 32 bytes, the values the dequant used
//          to compute per chunk, rounded the same way — then the GGUF block's 128 bytes of
//          nibbles with the bytes of each 4-byte group stored in the order (0,2,1,3), so that
//          masking one 32-bit word yields two adjacent elements in the two 16-bit halves.
//  kQ6K  : chunk = 256. Tile = 128 rows x 224 bytes: 128 bytes of low nibbles (8-element groups,
//          byte b0 = e0|e4<<4, b1 = e2|e6<<4, b2 = e1|e5<<4, b3 = e3|e7<<4), 64 bytes of high
//          2-bit fields (16-element groups: bits [2k,2k+2) = hi(e_2k), [16+2k,18+2k) = hi(e_2k+1)),
//          16 bf16 group scales (d * scale_g).
//  kQ8_0 : chunk = 256. Tile = 128 rows x 272 bytes: 8 bf16 block scales, then 256 int8 values
//          with each 4-byte group stored in the order (0,2,1,3).
#pragma once
#include <stdint.h>

namespace vmc {

enum WeightFormat : int { kWfBF16 = 0, kWfQ4K = 1, kWfQ6K = 2, kWfQ8_0 = 3 };

__host__ __device__ constexpr int wf_chunk(int wf) { return wf == kWfBF16 ? 64 : 256; }
__host__ __device__ constexpr int wf_row_bytes(int wf) {
  return wf == kWfBF16 ? 128 : wf == kWfQ4K ? 160 : wf == kWfQ6K ? 224 : 272;
}
__host__ __device__ constexpr int wf_tile_bytes(int wf) { return 128 * wf_row_bytes(wf); }

}  // namespace vmc
