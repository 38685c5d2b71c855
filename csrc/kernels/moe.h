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


// Expert-parallel dispatch (all-to-all by peer stores). Each rank routes only the token rows it owns
// (rows [rank * rpr, ...) of the step, `rows` of them): softmax over the E router logits, top-k (ties to
// the lower id), weights renormalised when norm_topk; then for each selected expert e it takes a slot
// on e's owner rank (o = e / e_local) with an atomic add on that rank's per-expert row counter, stores
// the bf16 row there (row slot of expert e % e_local in recv_x[o], `cap` rows per expert) together with
// a return word (rank << 24) | (row << 3) | j, and keeps the weight in topk_w[row * k + j]. Every CTA
// then releases its stores and counts one arrival at every rank; CTA 0 returns once all ranks'
// dispatches have arrived here, so the expert GEMMs that follow may read their rows and counts.
struct MoeDispatchArgs {
  const float* logits;   // this rank's rows [rows][ld_logits]
  int ld_logits;
  const void* x;         // this rank's rows, bf16 [rows][H]
  int rows, rpr, H, E, k, norm_topk, e_local, cap, rank, nranks;
  void* recv_x[8];       // every rank's expert input buffer [e_local][cap][H] bf16
  int32_t* recv_ret[8];  // every rank's return words [e_local][cap]
  uint32_t* cnt[8];      // every rank's per-expert row counters [e_local] (this layer's parity)
  float* topk_w;         // this rank: [rpr][k]
  uint32_t* arrive[8];   // every rank's dispatch arrival counter
  uint32_t* state;       // this rank: [0] arrival target, [1] CTAs done
  uint32_t* err;
};
void moe_dispatch(const MoeDispatchArgs& a, cudaStream_t st);
// CTAs moe_dispatch launches for rpr rows per rank (the same on every rank).
inline int moe_dispatch_ctas(int rpr) { return rpr <= 0 ? 1 : (rpr + 7) / 8; }
}  // namespace vmc
