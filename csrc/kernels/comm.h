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

// Tensor-parallel communication state of one rank for the reduce-scatter / all-gather design
// (rs_norm_ag below and the scatter epilogue of the row-parallel GEMM, gemm_tcgen05.h).
//
// Rows of a step's token batch are owned round the ranks in contiguous shards of rpr = ceil(T / N)
// rows (rank o owns rows [o * rpr, (o + 1) * rpr)). Each rank's symmetric region (CUDA IPC, mapped
// on every peer) holds:
//   recv[site]  bf16 [N * splits][rpr][H]: the partial sums of this rank's rows, one slot per
//               (source rank, K split), written by the sources' GEMM epilogues;
//   h           bf16 [max_tokens][H]: the normalised activations of every row, written by the
//               owners (the all-gather) and read by the next column-parallel GEMM;
//   counters    uint32 rs[site], ag[site]: monotonic arrival counters (peers add to them).
// `state` is this rank's private bookkeeping (the counter targets of the next call per site).
struct TpComm {
  int nranks = 1, rank = 0;
  void* recv[2][8] = {};          // [site][rank]: each rank's receive buffer of this site
  int64_t recv_rows = 0;          // rows of one receive buffer
  void* h[8] = {};                // each rank's h buffer
  uint32_t* rs_count[2][8] = {};  // [site][rank]
  uint32_t* ag_count[3][8] = {};  // [site][rank]; site 2: the expert-parallel combine
  uint32_t* state = nullptr;      // [3 sites][4] (rs target, ag target, CTAs done, the source-side CTA
                                  // counter of the site's scatter GEMM); site 2 is the expert-parallel
                                  // combine
  uint32_t* err = nullptr;
  int max_ctas = 148;
};

// Rows per rank of a T-token step.
inline int tp_rows_per_rank(int T, int nranks) { return (T + nranks - 1) / nranks; }
// CTAs of rs_norm_ag for rpr rows per rank (the same on every rank).
inline int tp_norm_ctas(int rpr, int max_ctas) { return rpr < 1 ? 1 : (rpr < max_ctas ? rpr : max_ctas); }

// Two-level arrival counting (VMC_TP_TWO_LEVEL=1; off by default): the CTAs of a signalling kernel
// count themselves in their own GPU's memory and the last one signals each rank once, instead of
// every CTA signalling every rank. Measured on 8 B200s it is slower (fused decode site 37.9 vs
// 33.8 us, decode step 4.17 vs 3.92 ms): the remote atomics do not contend, and the last CTA's extra
// system-scope release is on the critical path.
bool tp_two_level();
// The scatter GEMM's CTA counter of a site (gemm_tcgen05_scatter local_count), or null when every CTA
// signals; tp_scatter_arrivals: the arrivals per call an owner then receives from all sources.
inline uint32_t* tp_scatter_local(const TpComm& c, int site) { return tp_two_level() ? c.state + 4 * site + 3 : nullptr; }
inline int tp_scatter_arrivals(const TpComm& c, int grid) { return tp_two_level() ? c.nranks : grid * c.nranks; }

// Owner side of one row-parallel site: waits until every source rank's GEMM has delivered its
// partial rows (rs_inc arrivals: one per source rank when the GEMMs count through
// tp_scatter_local, else sources x their GEMM's CTAs), sums the N * splits partials of each
// owned row in a fixed order, adds the residual (fp32, updated in place for the owned rows only),
// applies RMSNorm with weight w, and writes the bf16 row into every rank's h (all-gather by push).
// CTA 0 returns only after every rank's rows have arrived here, so the next kernel may read all of h.
// gather = 0 writes the normalised rows into this rank's h only (the consumer needs only its own
// rows, e.g. the router of an expert-parallel MoE layer); no all-gather, no wait.
void rs_norm_ag(const TpComm& c, int site, int T, int H, int splits, int rs_inc, float* resid, const float* w,
                float eps, cudaStream_t st, int gather = 1);

// Owner side of an expert-parallel MoE layer's combine: waits for comb_inc arrivals (every expert
// rank's down GEMM CTAs), forms for each owned row the router-weighted sum of its k expert outputs
// (comb: this rank's [rpr][k][H] bf16 rows, topk_w [rpr][k]), adds the residual, applies RMSNorm and
// all-gathers like rs_norm_ag; then zeroes `reset` (this rank's expert row counters of the layer).
void moe_combine_norm_ag(const TpComm& c, const void* comb, uint32_t* comb_count, int comb_inc, const float* topk_w,
                         int k, uint32_t* reset, int reset_n, int T, int H, float* resid, const float* w, float eps,
                         cudaStream_t st);

// Symmetric allocations through CUDA IPC (handle_out: 64-byte cudaIpcMemHandle_t).
uint64_t sym_alloc(size_t bytes, void* handle_out);
uint64_t sym_open(const void* handle);
void sym_close(uint64_t peer_ptr);
void sym_free(uint64_t ptr);

}  // namespace vmc
