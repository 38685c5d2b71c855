// Host interface of the peer-memory collectives (comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

struct ArArgs {
  const float* data[8];   // fp32 partial [T, H] of every rank (peer pointers; own rank included)
  uint32_t* flags[8];     // flag arrays [256][8] of every rank
  uint32_t* epochs;       // this rank's per-CTA epoch counters [256]
  int nranks, rank;
  int T, H;
  int nsplit;             // per-split partial slices per rank (split-K GEMM output)
  int64_t split_stride;   // elements between the slices
  float* resid;           // fp32 residual stream [T, H] (updated in place)
  const float* w;         // RMSNorm weight [H]
  float eps;
  void* out;              // bf16 [T, H]
  uint32_t* err;          // device error word
};

// One-shot all-reduce of the partials + residual add + RMSNorm (see comm.cu).
void ar_add_rmsnorm(const ArArgs& a, int max_ctas, cudaStream_t st);

// Symmetric allocations through CUDA IPC (handle_out: 64-byte cudaIpcMemHandle_t).
uint64_t sym_alloc(size_t bytes, void* handle_out);
uint64_t sym_open(const void* handle);
void sym_close(uint64_t peer_ptr);
void sym_free(uint64_t ptr);

}  // namespace vmc
