// Native step forward of the Llama / Mixtral-dense graph: the whole per-step kernel sequence issued
// from C++ (no Python between launches), on device buffers owned by the caller.
//
// The graph is the one the reference builds with libllama (src/official/llama/models/llama.cpp:98-253):
// embed -> [per layer] RMSNorm -> QKV -> RoPE + paged KV store -> attention -> O -> (TP reduce) ->
// residual + RMSNorm -> gate/up + SwiGLU -> down -> (TP reduce) -> residual + RMSNorm -> ... ->
// final norm on the sampled rows -> lm_head -> sampler. Tensor-parallel steps use the fused
// peer-memory reduce-scatter / all-gather kernels (comm.h); NCCL is never called from here.
//
// Host-only code: it depends on the kernel launchers and the CUDA runtime, not on PyTorch, so a
// plain C++ runtime can drive it as well as the Python engine.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "comm.h"
#include "sampling.h"
#include "turboquant_types.h"

namespace vmc {

struct LinearDesc {
  int wf = 0;                // tiled weight format (weight_formats.cuh)
  const void* w = nullptr;   // tiled weight bytes
  int N = 0, K = 0;
};

// Mixture-of-experts FFN of a layer (Mixtral): the router and this rank's experts, stacked.
struct MoeDesc {
  LinearDesc router;         // [E, H]
  LinearDesc gate_up;        // one expert [2 F_local, H], gate / up rows interleaved
  int64_t gate_up_stride = 0;  // bytes between experts
  LinearDesc down;           // one expert [H, F_local]
  int64_t down_stride = 0;
  int e0 = 0, e_local = 0, f_local = 0;
};

struct LayerDesc {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  int n_qkv = 0;             // 1..3 QKV weights (fused, or split where the GGUF types differ)
  LinearDesc qkv[3];
  int qkv_col[3] = {0, 0, 0};  // first output column of each part
  LinearDesc wo, gate_up, down;  // gate_up rows interleave gate / up (fused SwiGLU)
  bool moe = false;
  MoeDesc m;
};

// MoE model settings and buffers. Expert-sliced layout (the reference's, single rank): router,
// routing, gather, grouped GEMMs and combine on this rank. Expert-parallel (ep = tp > 1): each rank
// routes its own token rows and the rows travel to the experts' ranks and back through peer memory
// (moe_dispatch, the grouped GEMMs, the row-scatter down GEMM and moe_combine_norm_ag).
struct MoeBuffers {
  int E = 0, k = 0, norm_topk = 1;
  bool ep = false;
  // expert-sliced path
  float* logits = nullptr;     // [max_tokens, E]
  int32_t* topk_id = nullptr;
  float* topk_w = nullptr;
  int32_t* counts = nullptr;
  int32_t* offsets = nullptr;
  int32_t* sorted_src = nullptr;
  int32_t* slot_row = nullptr;
  int32_t* total = nullptr;
  void* xs = nullptr;          // bf16 [max_tokens * k, H]
  void* act = nullptr;         // bf16 [max_tokens * k, F_local]
  float* y = nullptr;          // fp32 [max_tokens * k, H]
  float* out = nullptr;        // fp32 [max_tokens, H]
  // expert-parallel path
  int cap = 0;                 // rows per expert in the receive buffers
  void* recv_x[8] = {};        // every rank's [e_local][cap][H] bf16
  int32_t* recv_ret[8] = {};   // every rank's [e_local][cap]
  uint32_t* cnt[2][8] = {};    // [layer parity][rank]: per-expert row counters [e_local]
  void* comb[8] = {};          // every rank's [rpr_max][k][H] bf16
  uint32_t* disp_arrive[8] = {};
  uint32_t* comb_arrive[8] = {};
  uint32_t* disp_state = nullptr;  // this rank: 2 words
  float* ep_logits = nullptr;  // this rank: [rpr_max, E]
  float* ep_topk_w = nullptr;  // this rank: [rpr_max, k]
  void* ep_act = nullptr;      // this rank: [e_local * cap, F_local] bf16
  int32_t* ep_offsets = nullptr;  // this rank: [e_local] = e * cap
};

struct ForwardConfig {
  int L = 0, H = 0, Hq = 0, Hkv = 0, D = 0;  // Hq / Hkv: heads held by this rank
  int F = 0;                 // FFN width held by this rank
  int V_local = 0;           // lm_head rows held by this rank
  int max_tokens = 0, max_samples = 0, max_blocks = 0;
  float eps = 1e-5f, scale = 1.f;
  bool neox = false;
  const void* embd = nullptr;
  int embd_type = 0;
  int64_t embd_row_bytes = 0;
  const float* out_norm = nullptr;
  LinearDesc lm_head;
  const float* cos_sin = nullptr;
  int num_sms = 148;
};

// Device buffers (all caller-owned; sizes follow the Python Workspace of models/llama.py).
struct ForwardBuffers {
  float* resid = nullptr;    // fp32 [max_tokens, H]
  void* h = nullptr;         // bf16 [max_tokens, H]
  void* qkv_bf16 = nullptr;  // bf16 [max_tokens, qkv_n]
  float* split_ws = nullptr; // fp32 split-K partials
  int64_t split_ws_elems = 0;
  void* q = nullptr;         // bf16 [max_tokens, Hq * D]
  void* attn = nullptr;      // bf16 [max_tokens, Hq * D]
  void* o16 = nullptr;       // bf16 [max_tokens, H]
  void* act = nullptr;       // bf16 [max_tokens, F]
  void* hs = nullptr;        // bf16 [max_samples, H]
  float* logits = nullptr;   // fp32 [max_samples, V_local]
  float* part_o = nullptr;   // split-KV partials [max_splits, max_samples, Hq, D]
  float* part_lse = nullptr;
  int attn_max_splits = 1;
  // step metadata written by the scheduler (device copies)
  const int32_t* ids = nullptr;
  const int32_t* pos = nullptr;
  const int32_t* slots = nullptr;
  const int32_t* q_start = nullptr;
  const int32_t* ctx_len = nullptr;
  const int32_t* block_tables = nullptr;
  const int32_t* logits_idx = nullptr;
  const void* params = nullptr;  // SampleParams [max_samples]
  int32_t* out_tok = nullptr;
  float* out_lp = nullptr;
  // KV cache: layer l starts kv_layer_bytes * l bytes after kv (bf16 pages or TurboQuant slots)
  void* kv = nullptr;
  int64_t kv_layer_bytes = 0;
  bool tq = false;
  TqDev tq_tab{};            // cache / layer are set per layer
  uint32_t* err = nullptr;
};

struct StepDims {
  int T = 0;          // tokens (padding rows included)
  int R = 0;          // requests
  int S = 0;          // sampled rows
  int nd = 0;         // leading decode requests
  int max_qlen = 0;   // max prefill q_len
  int decode_qlen = 1;
  int attn_splits = 1;
  bool sample = true;  // false: stop after the lm_head logits (the caller applies penalties / samples)
};

class Forward {
 public:
  Forward(const ForwardConfig& cfg, std::vector<LayerDesc> layers, const ForwardBuffers& bufs);
  // Tensor-parallel communication (peer-memory reduce-scatter + all-gather); absent for one rank.
  void set_comm(const TpComm& comm);
  // Vocabulary-parallel sampling over the ranks' lm_head shards (sampling.h); absent for one rank.
  void set_sampler(const TpSample& s);
  // Buffers of the MoE layers (required when any layer is MoE).
  void set_moe(const MoeBuffers& m);
  // Issues one step on `st`; returns the number of kernels launched.
  int run(const StepDims& d, cudaStream_t st);
  // K-split count the step uses for weight w at M tokens (the consumer kernels sum exactly this many).
  int splits_for(const LinearDesc& w, int M) const;

 private:
  int gemm(const void* x, int ldx, const LinearDesc& w, void* out, int ldo, int M, int mode, int splits,
           int64_t split_stride, cudaStream_t st);
  int qkv(const LayerDesc& lw, int l, const StepDims& d, cudaStream_t st);
  int attention(int l, const StepDims& d, cudaStream_t st);
  int row_parallel(int site, const void* x, int ldx, const LinearDesc& w, const float* norm_w, int M,
                   cudaStream_t st, int gather = 1);
  int gate_up(const LayerDesc& lw, int M, cudaStream_t st);
  int moe_layer(const LayerDesc& lw, int l, const float* next_norm, int T, cudaStream_t st);
  TqDev tq_for(int l) const;

  ForwardConfig c_;
  std::vector<LayerDesc> layers_;
  ForwardBuffers b_;
  int qkv_n_ = 0;
  bool has_comm_ = false;
  TpComm comm_{};
  bool has_tps_ = false;
  TpSample tps_{};
  bool has_moe_ = false;
  MoeBuffers moe_{};
};

// Split-K policy shared with the Python wrappers (ops.pick_splits / ops.effective_splits): the
// number of K splits of a persistent GEMM that minimises (weight bytes + partial-sum traffic)
// divided by the SM-balance efficiency of the resulting work units.
int gemm_pick_splits(int wf, int N, int K, int M, int num_sms, int max_splits = 8);
int gemm_effective_splits(int wf, int K, int s);

}  // namespace vmc
