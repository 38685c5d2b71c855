// Host interface of the MoE routing / combine kernels (moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

struct MoeRouteArgs {
  const float* logits;   // router logits [T, E] (row stride ld_logits)
  int ld_logits;
  int T, E, k;
  int norm_topk;         // renormalise the k selected probabilities to sum 1
  int e0, e_local;       // experts held by this rank: [e0, e0 + e_local)
  int32_t* topk_id;      // [T, k] global expert ids
  float* topk_w;         // [T, k] routing weights
  int32_t* counts;       // [e_local] rows per local expert
  int32_t* offsets;      // [e_local] first sorted row of each local expert
  int32_t* sorted_src;   // [T * k] source token of each sorted row (tail rows: 0)
  int32_t* slot_row;     // [T, k] sorted row of each (token, slot) pair, -1 if not local
  int32_t* total_rows;   // [1] number of sorted rows
};

void moe_route(const MoeRouteArgs& a, cudaStream_t st);

// out[t, :] = sum_j topk_w[t, j] * y[slot_row[t, j], :] over local pairs (fp32).
void moe_combine(const float* y, int ldy, const int32_t* slot_row, const float* topk_w, int T, int k, int H,
                 float* out, int ldo, cudaStream_t st);

}  // namespace vmc
