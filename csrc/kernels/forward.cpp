// Native step forward (forward.h): the per-step kernel program of the Llama graph issued from C++.
//
// One call launches every kernel of a step on one stream, in the order of the Python reference
// implementation in vm_c_b200/models/llama.py (LlamaModel.forward), with the same split-K policy,
// so that both produce identical results; the Python path remains for tracing, CPU offload, MoE
// layers and token-tree masks. Reference graph: src/official/llama/models/llama.cpp:98-253; the
// two tensor-parallel reduction sites after Wo and after the FFN down projection (:171, :196) take
// the fused reduce-scatter / all-gather here instead of the reference's NCCL all-reduce
// (src/distributed/nccl_comm.cu:259-327).
#include "forward.h"

#include <algorithm>
#include <cmath>
#include <stdexcept>
#include <string>

#include "attention.h"
#include "gemm_tcgen05.h"
#include "layers.h"
#include "moe.h"
#include "sampling.h"
#include "turboquant_ops.h"

namespace vmc {

namespace {

int wf_chunk_host(int wf) { return wf == 0 ? 64 : 256; }
int wf_row_bytes_host(int wf) {
  switch (wf) {
    case 0: return 128;
    case 1: return 160;
    case 2: return 224;
    default: return 272;
  }
}
int chunks_of(int wf, int K) { return (K + wf_chunk_host(wf) - 1) / wf_chunk_host(wf); }
int64_t tiled_bytes_host(int wf, int N, int K) {
  return static_cast<int64_t>((N + 127) / 128) * chunks_of(wf, K) * 128 * wf_row_bytes_host(wf);
}
int pick_bn_host(int M) {
  for (int b : {16, 32, 64, 128})
    if (M <= b) return b;
  return 256;
}

void check(bool ok, const char* msg) {
  if (!ok) throw std::runtime_error(std::string("native forward: ") + msg);
}

}  // namespace

int gemm_effective_splits(int wf, int K, int s) {
  const int chunks = chunks_of(wf, K);
  s = std::max(1, std::min(s, chunks));
  const int per = (chunks + s - 1) / s;
  return (chunks + per - 1) / per;
}

int gemm_pick_splits(int wf, int N, int K, int M, int num_sms, int max_splits) {
  const int bn = pick_bn_host(M);
  const int m_tiles = (M + bn - 1) / bn;
  const int chunks = chunks_of(wf, K);
  if (m_tiles > 1 || chunks < 2) return 1;
  const int base = (N + 127) / 128;
  const double wbytes = static_cast<double>(tiled_bytes_host(wf, N, K));
  auto cost = [&](int s) {
    const int units = base * s;
    const double eff = static_cast<double>(units) / (std::ceil(static_cast<double>(units) / num_sms) * num_sms);
    const double partial = s > 1 ? static_cast<double>(s) * M * N * 8 : static_cast<double>(M) * N * 2;
    return (wbytes + partial) / eff;
  };
  int best = 1;
  double best_c = cost(1);
  for (int s = 2; s <= std::min(max_splits, chunks); ++s) {
    const double c = cost(s);
    if (c < best_c) {
      best_c = c;
      best = s;
    }
  }
  return gemm_effective_splits(wf, K, best);
}

Forward::Forward(const ForwardConfig& cfg, std::vector<LayerDesc> layers, const ForwardBuffers& bufs)
    : c_(cfg), layers_(std::move(layers)), b_(bufs) {
  check(c_.L == static_cast<int>(layers_.size()) && c_.L > 0, "layer count");
  check(c_.H > 0 && c_.Hq > 0 && c_.Hkv > 0 && c_.D > 0 && c_.max_tokens > 0, "dimensions");
  qkv_n_ = (c_.Hq + 2 * c_.Hkv) * c_.D;
  for (const LayerDesc& l : layers_) {
    check(l.n_qkv >= 1 && l.n_qkv <= 3, "qkv parts");
    check(l.wo.w && (l.moe ? (l.m.router.w && l.m.gate_up.w && l.m.down.w) : (l.gate_up.w && l.down.w)),
          "layer weights");
  }
}

void Forward::set_comm(const TpComm& comm) {
  comm_ = comm;
  has_comm_ = comm.nranks > 1;
}

void Forward::set_moe(const MoeBuffers& m) {
  moe_ = m;
  has_moe_ = true;
}

// One MoE FFN (after the attention site): writes the next layer's normalised input into h.
int Forward::moe_layer(const LayerDesc& lw, int l, const float* next_norm, int T, cudaStream_t st) {
  check(has_moe_, "MoE layer without MoE buffers");
  const MoeDesc& md = lw.m;
  const MoeBuffers& mb = moe_;
  int n = 0;
  if (!mb.ep) {
    check(!has_comm_, "expert-sliced MoE layers under tensor parallelism take the Python path");
    const int R = T * mb.k;
    gemm(b_.h, c_.H, md.router, mb.logits, mb.E, T, kGemmOutF32, 1, 0, st);
    MoeRouteArgs ra;
    ra.logits = mb.logits;
    ra.ld_logits = mb.E;
    ra.T = T;
    ra.E = mb.E;
    ra.k = mb.k;
    ra.norm_topk = mb.norm_topk;
    ra.e0 = md.e0;
    ra.e_local = md.e_local;
    ra.topk_id = mb.topk_id;
    ra.topk_w = mb.topk_w;
    ra.counts = mb.counts;
    ra.offsets = mb.offsets;
    ra.sorted_src = mb.sorted_src;
    ra.slot_row = mb.slot_row;
    ra.total_rows = mb.total;
    moe_route(ra, st);
    gather_rows(b_.h, mb.sorted_src, R, c_.H, mb.xs, st);
    const int bn = gemm_pick_bn(std::max(1, (R + md.e_local - 1) / md.e_local));
    gemm_tcgen05_grouped(md.gate_up.wf, md.gate_up.w, md.gate_up_stride, md.gate_up.N, md.gate_up.K, mb.xs, R, c_.H,
                         mb.act, md.f_local, kGemmOutSwiGLU, md.e_local, mb.counts, mb.offsets, T, bn, b_.err, st);
    gemm_tcgen05_grouped(md.down.wf, md.down.w, md.down_stride, md.down.N, md.down.K, mb.act, R, md.f_local, mb.y,
                         c_.H, kGemmOutF32, md.e_local, mb.counts, mb.offsets, T, bn, b_.err, st);
    moe_combine(mb.y, c_.H, mb.slot_row, mb.topk_w, T, mb.k, c_.H, mb.out, c_.H, st);
    add_rmsnorm(b_.resid, mb.out, true, 1, 0, next_norm, T, c_.H, c_.eps, b_.h, st);
    return n + 8;
  }
  // expert-parallel: route own rows, dispatch, experts, return, combine + norm + all-gather
  const TpComm& c = comm_;
  const int rpr = tp_rows_per_rank(T, c.nranks);
  const int row0 = c.rank * rpr;
  const int rows = std::max(0, std::min(rpr, T - row0));
  if (rows > 0) {
    gemm(static_cast<const uint16_t*>(b_.h) + static_cast<int64_t>(row0) * c_.H, c_.H, md.router, mb.ep_logits, mb.E,
         rows, kGemmOutF32, 1, 0, st);
    ++n;
  }
  const int par = l & 1;
  MoeDispatchArgs da{};
  da.logits = mb.ep_logits;
  da.ld_logits = mb.E;
  da.x = static_cast<const uint16_t*>(b_.h) + static_cast<int64_t>(row0) * c_.H;
  da.rows = rows;
  da.rpr = rpr;
  da.H = c_.H;
  da.E = mb.E;
  da.k = mb.k;
  da.norm_topk = mb.norm_topk;
  da.e_local = md.e_local;
  da.cap = mb.cap;
  da.rank = c.rank;
  da.nranks = c.nranks;
  for (int q = 0; q < c.nranks; ++q) {
    da.recv_x[q] = mb.recv_x[q];
    da.recv_ret[q] = mb.recv_ret[q];
    da.cnt[q] = mb.cnt[par][q];
    da.arrive[q] = mb.disp_arrive[q];
  }
  da.topk_w = mb.ep_topk_w;
  da.state = mb.disp_state;
  da.err = c.err;
  moe_dispatch(da, st);
  const int rows_cap = md.e_local * mb.cap;
  const int max_rows = std::min(mb.cap, T);
  const int bn = gemm_pick_bn(std::max(1, (T * mb.k + mb.E - 1) / mb.E));
  const int32_t* counts = reinterpret_cast<const int32_t*>(mb.cnt[par][c.rank]);
  gemm_tcgen05_grouped(md.gate_up.wf, md.gate_up.w, md.gate_up_stride, md.gate_up.N, md.gate_up.K,
                       mb.recv_x[c.rank], rows_cap, c_.H, mb.ep_act, md.f_local, kGemmOutSwiGLU, md.e_local, counts,
                       mb.ep_offsets, max_rows, bn, b_.err, st);
  const int grid = gemm_tcgen05_grouped_rowscatter(md.down.wf, md.down.w, md.down_stride, md.down.N, md.down.K,
                                                   mb.ep_act, rows_cap, md.f_local, md.e_local, counts,
                                                   mb.ep_offsets, max_rows, bn, mb.recv_ret[c.rank], mb.k, mb.comb,
                                                   mb.comb_arrive, c.nranks, b_.err, st, tp_scatter_local(c, 2));
  moe_combine_norm_ag(c, mb.comb[c.rank], mb.comb_arrive[c.rank], tp_scatter_arrivals(c, grid), mb.ep_topk_w, mb.k,
                      mb.cnt[par][c.rank], md.e_local, T, c_.H, b_.resid, next_norm, c_.eps, st);
  return n + 4;
}

void Forward::set_sampler(const TpSample& s) {
  tps_ = s;
  has_tps_ = s.nranks > 1;
}

int Forward::splits_for(const LinearDesc& w, int M) const {
  int s = gemm_pick_splits(w.wf, w.N, w.K, M, c_.num_sms);
  while (s > 1 && static_cast<int64_t>(s) * M > c_.max_tokens) --s;
  return gemm_effective_splits(w.wf, w.K, s);
}

int Forward::gemm(const void* x, int ldx, const LinearDesc& w, void* out, int ldo, int M, int mode, int splits,
                  int64_t split_stride, cudaStream_t st) {
  gemm_tcgen05(w.wf, w.w, w.N, w.K, x, M, ldx, out, ldo, mode, splits, 0, b_.err, st, split_stride);
  return 1;
}

TqDev Forward::tq_for(int l) const {
  TqDev t = b_.tq_tab;
  t.cache = static_cast<uint8_t*>(b_.kv) + b_.kv_layer_bytes * l;
  t.layer = l;
  return t;
}

int Forward::qkv(const LayerDesc& lw, int l, const StepDims& d, cudaStream_t st) {
  const int M = d.T;
  const int s = splits_for(lw.qkv[0], M);
  int n = 0;
  const void* src;
  bool f32 = false;
  int64_t sstride = 0;
  if (s > 1) {
    sstride = static_cast<int64_t>(M) * qkv_n_;
    check(sstride * s <= b_.split_ws_elems, "split workspace too small (qkv)");
    for (int i = 0; i < lw.n_qkv; ++i)
      n += gemm(b_.h, c_.H, lw.qkv[i], b_.split_ws + lw.qkv_col[i], qkv_n_, M, kGemmOutF32Split, s, sstride, st);
    src = b_.split_ws;
    f32 = true;
  } else {
    for (int i = 0; i < lw.n_qkv; ++i)
      n += gemm(b_.h, c_.H, lw.qkv[i], static_cast<uint16_t*>(b_.qkv_bf16) + lw.qkv_col[i], qkv_n_, M,
                kGemmOutBF16, 1, 0, st);
    src = b_.qkv_bf16;
  }
  void* kv_l = static_cast<uint8_t*>(b_.kv) + b_.kv_layer_bytes * l;
  if (b_.tq) {
    const TqDev t = tq_for(l);
    rope_store_tq(src, f32, s, sstride, M, c_.Hq, c_.Hkv, c_.D, b_.pos, b_.slots, c_.cos_sin, c_.neox, b_.q, t, st);
  } else {
    rope_store(src, f32, s, sstride, M, c_.Hq, c_.Hkv, c_.D, b_.pos, b_.slots, c_.cos_sin, c_.neox, b_.q, kv_l, st);
  }
  return n + 1;
}

int Forward::attention(int l, const StepDims& d, cudaStream_t st) {
  int n = 0;
  TqDev t;
  if (b_.tq) t = tq_for(l);
  AttnLaunch a;
  a.q = b_.q;
  a.kv = static_cast<uint8_t*>(b_.kv) + b_.kv_layer_bytes * l;
  a.q_start = b_.q_start;
  a.ctx_len = b_.ctx_len;
  a.block_tables = b_.block_tables;
  a.max_blocks = c_.max_blocks;
  a.Hq = c_.Hq;
  a.Hkv = c_.Hkv;
  a.D = c_.D;
  a.scale = c_.scale;
  a.out = b_.attn;
  a.tq = b_.tq ? &t : nullptr;
  a.err = b_.err;
  if (!b_.tq) a.num_blocks = b_.kv_layer_bytes / (static_cast<int64_t>(2) * c_.Hkv * 16 * c_.D * 2);
  const int G = c_.Hq / c_.Hkv;
  if (d.nd > 0) {
    const bool dec_ok = d.decode_qlen * G <= 16;
    int splits = (d.attn_splits > 1 && dec_ok && d.nd <= c_.max_samples) ? d.attn_splits : 1;
    splits = std::min(splits, b_.attn_max_splits);
    a.num_reqs = d.nd;
    a.req_offset = 0;
    a.max_qlen = d.decode_qlen;
    a.total_tokens = d.nd * d.decode_qlen;
    a.decode = dec_ok;
    a.splits = splits;
    a.part_o = splits > 1 ? b_.part_o : nullptr;
    a.part_lse = splits > 1 ? b_.part_lse : nullptr;
    paged_attention(a, st);
    n += (dec_ok && splits > 1) ? 2 : 1;
  }
  if (d.R > d.nd) {
    a.num_reqs = d.R - d.nd;
    a.req_offset = d.nd;
    a.max_qlen = d.max_qlen;
    a.total_tokens = d.T;
    a.decode = false;
    a.splits = 1;
    a.part_o = nullptr;
    a.part_lse = nullptr;
    paged_attention(a, st);
    n += 1;
  }
  return n;
}

// Row-parallel GEMM (x @ w^T), then residual add + RMSNorm(norm_w) into h (all rows; with
// gather = 0 under tensor parallelism, this rank's rows only).
int Forward::row_parallel(int site, const void* x, int ldx, const LinearDesc& w, const float* norm_w, int M,
                          cudaStream_t st, int gather) {
  const int s = splits_for(w, M);
  if (has_comm_) {
    const TpComm& c = comm_;
    int used = s;
    const int grid = gemm_tcgen05_scatter(w.wf, w.w, w.N, w.K, x, M, ldx, s, c.recv[site], c.rs_count[site],
                                          c.nranks, c.rank, c.recv_rows, b_.err, st, &used, tp_scatter_local(c, site));
    rs_norm_ag(c, site, M, c_.H, used, tp_scatter_arrivals(c, grid), b_.resid, norm_w, c_.eps, st, gather);
    return 2;
  }
  if (s > 1) {
    const int64_t stride = static_cast<int64_t>(M) * c_.H;
    check(stride * s <= b_.split_ws_elems, "split workspace too small (row-parallel)");
    gemm(x, ldx, w, b_.split_ws, c_.H, M, kGemmOutF32Split, s, stride, st);
    add_rmsnorm(b_.resid, b_.split_ws, true, s, stride, norm_w, M, c_.H, c_.eps, b_.h, st);
  } else {
    gemm(x, ldx, w, b_.o16, c_.H, M, kGemmOutBF16, 1, 0, st);
    add_rmsnorm(b_.resid, b_.o16, false, 1, 0, norm_w, M, c_.H, c_.eps, b_.h, st);
  }
  return 2;
}

int Forward::gate_up(const LayerDesc& lw, int M, cudaStream_t st) {
  const LinearDesc& w = lw.gate_up;
  const int s = splits_for(w, M);
  if (s > 1) {
    const int64_t stride = static_cast<int64_t>(M) * w.N;
    check(stride * s <= b_.split_ws_elems, "split workspace too small (gate/up)");
    gemm(b_.h, c_.H, w, b_.split_ws, w.N, M, kGemmOutF32Split, s, stride, st);
    swiglu(b_.split_ws, true, s, stride, M, w.N / 2, true, b_.act, st);
    return 2;
  }
  gemm(b_.h, c_.H, w, b_.act, c_.F, M, kGemmOutSwiGLU, 1, 0, st);
  return 1;
}

int Forward::run(const StepDims& d, cudaStream_t st) {
  check(d.T > 0 && d.T <= c_.max_tokens && d.S >= 0 && d.S <= c_.max_samples, "step dimensions");
  int n = 0;
  embed(b_.ids, d.T, c_.embd, c_.embd_type, c_.embd_row_bytes, c_.H, b_.resid, nullptr, st);
  add_rmsnorm(b_.resid, nullptr, false, 1, 0, layers_[0].attn_norm, d.T, c_.H, c_.eps, b_.h, st);
  n += 2;
  for (int l = 0; l < c_.L; ++l) {
    const LayerDesc& lw = layers_[l];
    n += qkv(lw, l, d, st);
    n += attention(l, d, st);
    const float* nxt = l + 1 < c_.L ? layers_[l + 1].attn_norm : c_.out_norm;
    if (lw.moe) {
      // an expert-parallel layer routes only this rank's rows: no all-gather after the attention
      n += row_parallel(0, b_.attn, c_.Hq * c_.D, lw.wo, lw.ffn_norm, d.T, st, moe_.ep ? 0 : 1);
      n += moe_layer(lw, l, nxt, d.T, st);
      continue;
    }
    n += row_parallel(0, b_.attn, c_.Hq * c_.D, lw.wo, lw.ffn_norm, d.T, st);
    n += gate_up(lw, d.T, st);
    n += row_parallel(1, b_.act, c_.F, lw.down, nxt, d.T, st);
  }
  if (d.S > 0) {
    gather_rows(b_.h, b_.logits_idx, d.S, c_.H, b_.hs, st);
    gemm(b_.hs, c_.H, c_.lm_head, b_.logits, c_.V_local, d.S, kGemmOutF32, 1, 0, st);
    n += 2;
    if (d.sample) {
      const SampleParams* sp = static_cast<const SampleParams*>(b_.params);
      if (has_tps_) {
        tp_sample(tps_, b_.logits, d.S, c_.V_local, c_.V_local, sp, b_.out_tok, b_.out_lp, st);
        n += 2;
      } else {
        sample(b_.logits, d.S, c_.V_local, c_.V_local, sp, b_.out_tok, b_.out_lp, st);
        n += 1;
      }
    }
  }
  return n;
}

}  // namespace vmc
