// Host interface of the tcgen05 fused-dequant GEMM (gemm_tcgen05.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vmc {

enum GemmOut : int {
  kGemmOutBF16 = 0,    // out[m, n] = acc (bf16)
  kGemmOutF32 = 1,     // out[m, n] = acc (fp32)
  kGemmOutF32Add = 2,  // out[m, n] += acc (fp32 red.add; required for split-K; output pre-zeroed)
  kGemmOutSwiGLU = 3,  // rows interleave gate/up: out[m, f] = silu(acc[2f]) * acc[2f+1] (bf16)
  kGemmOutF32Split = 4,  // out[split][m, n] = partial over this split's K range (fp32, no atomics)
  kGemmOutScatterBF16 = 5,  // tensor-parallel reduce-scatter: rows stored into their owner rank's buffer
  kGemmOutRowScatterBF16 = 6,  // expert-parallel combine: each row returned to its token's rank and slot
};

// out = x[M, K] (bf16, row stride ldx) @ W[N, K]^T with W in a tiled format (weight_formats.cuh).
// splits > 1 partitions K across CTAs (out_mode must be kGemmOutF32Add). bn = 0 picks the token
// tile from M. `err` receives a DeviceError code if a bounded wait expires.
// Returns the number of CTAs launched.
int gemm_tcgen05(int wf, const void* w_tiled, int N, int K, const void* x, int M, int ldx, void* out, int ldo,
                 int out_mode, int splits, int bn, uint32_t* err, cudaStream_t st, int64_t split_stride = 0);
// Row-parallel GEMM of a tensor-parallel layer with the reduce-scatter in its epilogue: row m of the
// bf16 product goes to rank o = m / ceil(M / nranks) (row m - o * rpr of slot rank * splits + split of
// recv[o], row stride N). After its last unit a CTA releases its stores at system scope; with
// local_count (a zeroed uint32 in this GPU's memory, reset by each call) the grid's last CTA then
// adds 1 to counters[q] of every rank q (one arrival per call), otherwise every CTA does. recv /
// counters are the peers' IPC-mapped addresses. Returns the CTA count; *splits_used receives the
// effective K splits.
int gemm_tcgen05_scatter(int wf, const void* w_tiled, int N, int K, const void* x, int M, int ldx, int splits,
                         void* const* recv, uint32_t* const* counters, int nranks, int rank, int64_t recv_rows,
                         uint32_t* err, cudaStream_t st, int* splits_used, uint32_t* local_count = nullptr);
// Grouped GEMM (MoE experts): for every group g with rows [offsets[g], offsets[g] + counts[g]) of
// x (device arrays, at most max_rows rows per group), out[rows] = x[rows] @ W_g^T where W_g starts
// w_group_stride bytes after W_{g-1}. One launch for all groups; no host synchronisation on the
// counts. out_mode: kGemmOutBF16, kGemmOutF32 or kGemmOutSwiGLU.
void gemm_tcgen05_grouped(int wf, const void* w_tiled, int64_t w_group_stride, int N, int K, const void* x,
                          int rows_total, int ldx, void* out, int ldo, int out_mode, int groups,
                          const int32_t* counts, const int32_t* offsets, int max_rows, int bn, uint32_t* err,
                          cudaStream_t st);
// Grouped GEMM (local experts) whose output rows go back over NVLink to the rank / row / top-k slot
// packed in row_ret[m] ((rank << 24) | (row << 3) | j; negative = skip): row (row * row_k + j) of
// dst[rank] (bf16, stride N). The CTAs then release their stores and count arrivals at every rank as
// in gemm_tcgen05_scatter (one per call with local_count, one per CTA without). Returns the CTA count.
int gemm_tcgen05_grouped_rowscatter(int wf, const void* w_tiled, int64_t w_group_stride, int N, int K, const void* x,
                                    int rows_total, int ldx, int groups, const int32_t* counts, const int32_t* offsets,
                                    int max_rows, int bn, const int32_t* row_ret, int row_k, void* const* dst,
                                    uint32_t* const* counters, int nranks, uint32_t* err, cudaStream_t st,
                                    uint32_t* local_count = nullptr);
int gemm_pick_bn(int M);
// Allocates this device's stream-K workspace (call once per device before any stream capture).
void gemm_prepare();
// Whether decode-width quantized GEMMs use the stream-K schedule (VMC_STREAMK=0 turns it off).
bool gemm_streamk();
// Diagnostics: when set, CTA 0 of every GEMM writes per-role clock64 stamps into buf[512].
void gemm_set_trace(unsigned long long* buf);
int gemm_smem_bytes(int wf, int bn);
void make_act_tensor_map(CUtensorMap* map, const void* x, int M, int K, int ldx, int box_rows);

}  // namespace vmc
