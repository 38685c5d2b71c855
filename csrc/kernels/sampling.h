// Host interface of the sampling kernels (sampling.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "sample_params.hpp"

namespace vmc {

void sample(const float* logits, int S, int V, int64_t ld, const SampleParams* params, int32_t* out_tok, float* out_lp,
            cudaStream_t st);
void apply_penalties(float* logits, int64_t ld, const int32_t* row_of, const int32_t* tok, const int32_t* out_count,
                     const SampleParams* params, int n, cudaStream_t st);

// Vocabulary-parallel sampling state of one rank: the exchange buffers (peer addresses, one per
// rank, each [nranks][max_rows] slots of tp_sample_row_bytes()) and arrival counters in the
// symmetric region, and this rank's private bookkeeping (2 words, zero-initialised).
struct TpSample {
  int nranks = 1, rank = 0;
  void* xbuf[8] = {};
  uint32_t* count[8] = {};
  uint32_t* state = nullptr;
  int max_rows = 0;
  uint32_t* err = nullptr;
};
// Samples S rows whose logits are split by vocabulary over the ranks (this rank holds entries
// [rank * V_local, (rank + 1) * V_local), row stride ld); every rank writes the same tokens. Two
// kernels: local reduction + push, then merge. Rows take the same choices sample() makes.
void tp_sample(const TpSample& t, const float* logits, int S, int V_local, int64_t ld, const SampleParams* params,
               int32_t* out_tok, float* out_lp, cudaStream_t st);
size_t tp_sample_row_bytes();
}  // namespace vmc
