// Host interface of the paged attention kernels (attention.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "turboquant_types.h"

namespace vmc {

struct AttnLaunch {
  const void* q;             // bf16 [T, Hq, D]
  const void* kv;            // bf16 [num_blocks, 2, Hkv, 16, D] (one layer)
  const int32_t* q_start;    // [R + 1] token offsets of the requests (device)
  const int32_t* ctx_len;    // [R] context length after this step (device)
  const int32_t* block_tables;  // [R, max_blocks] (device)
  int max_blocks;
  int num_reqs;              // requests handled by this launch
  int req_offset;            // index of the first of them in q_start / ctx_len / block_tables
  int max_qlen;              // upper bound of q_len over these requests
  int total_tokens;          // rows of the split-KV partial buffers
  int Hq, Hkv, D;
  float scale;
  bool decode;               // true: q_len * (Hq/Hkv) <= 16 decode kernel; false: prefill kernel
  int splits;                // split-KV CTAs per (request, kv head) for decode
  float* part_o;             // [splits, total_tokens, Hq, D] fp32 (splits > 1)
  float* part_lse;           // [splits, total_tokens, Hq] fp32
  void* out;                 // bf16 [T, Hq, D]
  const TqDev* tq = nullptr; // TurboQuant cache of this layer instead of bf16 pages (kv unused)
  const uint64_t* tree_mask = nullptr;  // [T] tree-verification masks (prefill path only), or null
  int tree_span = 0;         // bit 0 of a mask is the key at position ctx - tree_span
  int64_t num_blocks = 0;    // blocks of the bf16 page array (0: unknown; the tcgen05 prefill path needs it)
  uint32_t* err = nullptr;   // device error word for expired bounded waits (tcgen05 prefill path)
};

void paged_attention(const AttnLaunch& a, cudaStream_t st);

// Prefill chunks of bf16 caches with head dim 128 and causal masks run on the tcgen05 kernel
// (attention_tc.cu); everything else on the mma.sync kernels. VMC_ATTN_TC=0 (or
// attn_prefill_tc_enable(0)) keeps prefill on mma.sync.
bool attn_prefill_tc_eligible(const AttnLaunch& a);
void attn_prefill_tc(const AttnLaunch& a, cudaStream_t st);
void attn_prefill_tc_enable(int on);

// Move KV rows inside a bf16 paged cache [L, num_blocks, 2, Hkv, 16, D] (all layers, K and V, all
// KV heads): request r moves cnt[r] rows, src[r * max_moves + i] -> dst[r * max_moves + i] (slot
// indices). All rows of a request are read before any is written, so a destination may be another
// move's source (tree verification compacting the accepted branch).
void kv_move(void* cache, int L, int64_t layer_elems, int Hkv, int D, const int32_t* src, const int32_t* dst,
             const int32_t* cnt, int num_reqs, int max_moves, cudaStream_t st);

// Resident decode CTAs per SM (occupancy of the decode kernel for head dim D).
int attn_decode_ctas_per_sm(int D);

}  // namespace vmc

// The allocation-free C entry point of split-KV decode attention (attention_noalloc.cu).
#include "attention_noalloc.h"
