// Python bindings of the sm_100a kernels. Every op takes preallocated torch tensors and launches on
// the current CUDA stream (so the calls can be captured into CUDA graphs); none allocates.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention.h"
#include "comm.h"
#include "forward.h"
#include "gdn.h"
#include "gemm_tcgen05.h"
#include "layers.h"
#include "moe.h"
#include "sampling.h"
#include "turboquant_ops.h"
#include "weights.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
template <typename T>
T* ptr(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void gemm(int wf, torch::Tensor w, int64_t N, int64_t K, torch::Tensor x, int64_t M, torch::Tensor out,
          int64_t out_mode, int64_t splits, int64_t bn, torch::Tensor err, int64_t split_stride) {
  check_cuda(w, "w");
  check_cuda(x, "x");
  check_cuda(out, "out");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16, "gemm: x must be bf16");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "gemm: x must be 2-D with unit inner stride");
  TORCH_CHECK(x.size(0) >= M && x.size(1) >= K, "gemm: x too small");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) >= M, "gemm: bad output");
  const bool f32_out =
      out_mode == vmc::kGemmOutF32 || out_mode == vmc::kGemmOutF32Add || out_mode == vmc::kGemmOutF32Split;
  if (out_mode == vmc::kGemmOutF32Split)
    TORCH_CHECK(split_stride >= M * out.stride(0) &&
                    out.storage().nbytes() >= static_cast<size_t>((splits * split_stride) * 4),
                "gemm: per-split output buffer too small");
  TORCH_CHECK(out.scalar_type() == (f32_out ? torch::kFloat32 : torch::kBFloat16), "gemm: output dtype mismatch");
  TORCH_CHECK(w.numel() >= vmc::tiled_weight_bytes(wf, N, K), "gemm: weight buffer too small");
  vmc::gemm_tcgen05(wf, w.data_ptr(), static_cast<int>(N), static_cast<int>(K), x.data_ptr(), static_cast<int>(M),
                    static_cast<int>(x.stride(0)), out.data_ptr(), static_cast<int>(out.stride(0)),
                    static_cast<int>(out_mode), static_cast<int>(splits), static_cast<int>(bn),
                    ptr<uint32_t>(err), cur_stream(), split_stride);
}

void gemm_grouped(int wf, torch::Tensor w, int64_t w_group_stride, int64_t N, int64_t K, torch::Tensor x,
                  int64_t rows_total, torch::Tensor out, int64_t out_mode, int64_t groups, torch::Tensor counts,
                  torch::Tensor offsets, int64_t max_rows, int64_t bn, torch::Tensor err) {
  check_cuda(w, "w");
  check_cuda(x, "x");
  check_cuda(out, "out");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1, "gemm_grouped: bad x");
  TORCH_CHECK(x.size(0) >= rows_total && x.size(1) >= K, "gemm_grouped: x too small");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) >= rows_total, "gemm_grouped: bad output");
  TORCH_CHECK(counts.scalar_type() == torch::kInt32 && offsets.scalar_type() == torch::kInt32 &&
                  counts.numel() >= groups && offsets.numel() >= groups,
              "gemm_grouped: counts / offsets must be int32 [groups]");
  TORCH_CHECK(w.numel() >= static_cast<int64_t>(groups - 1) * w_group_stride + vmc::tiled_weight_bytes(wf, N, K),
              "gemm_grouped: weight buffer too small");
  const bool f32_out = out_mode == vmc::kGemmOutF32;
  TORCH_CHECK(out.scalar_type() == (f32_out ? torch::kFloat32 : torch::kBFloat16), "gemm_grouped: output dtype");
  vmc::gemm_tcgen05_grouped(wf, w.data_ptr(), w_group_stride, static_cast<int>(N), static_cast<int>(K), x.data_ptr(),
                            static_cast<int>(rows_total), static_cast<int>(x.stride(0)), out.data_ptr(),
                            static_cast<int>(out.stride(0)), static_cast<int>(out_mode), static_cast<int>(groups),
                            ptr<int32_t>(counts), ptr<int32_t>(offsets), static_cast<int>(max_rows),
                            static_cast<int>(bn), ptr<uint32_t>(err), cur_stream());
}

void moe_route(torch::Tensor logits, int64_t T, int64_t E, int64_t k, bool norm_topk, int64_t e0, int64_t e_local,
               torch::Tensor topk_id, torch::Tensor topk_w, torch::Tensor counts, torch::Tensor offsets,
               torch::Tensor sorted_src, torch::Tensor slot_row, torch::Tensor total_rows) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1, "moe_route: fp32 logits");
  TORCH_CHECK(topk_id.numel() >= T * k && topk_w.numel() >= T * k && slot_row.numel() >= T * k &&
                  sorted_src.numel() >= T * k && counts.numel() >= e_local && offsets.numel() >= e_local,
              "moe_route: output buffers too small");
  vmc::MoeRouteArgs a;
  a.logits = ptr<float>(logits);
  a.ld_logits = static_cast<int>(logits.stride(0));
  a.T = static_cast<int>(T);
  a.E = static_cast<int>(E);
  a.k = static_cast<int>(k);
  a.norm_topk = norm_topk ? 1 : 0;
  a.e0 = static_cast<int>(e0);
  a.e_local = static_cast<int>(e_local);
  a.topk_id = ptr<int32_t>(topk_id);
  a.topk_w = ptr<float>(topk_w);
  a.counts = ptr<int32_t>(counts);
  a.offsets = ptr<int32_t>(offsets);
  a.sorted_src = ptr<int32_t>(sorted_src);
  a.slot_row = ptr<int32_t>(slot_row);
  a.total_rows = ptr<int32_t>(total_rows);
  vmc::moe_route(a, cur_stream());
}

void moe_combine(torch::Tensor y, torch::Tensor slot_row, torch::Tensor topk_w, int64_t T, int64_t k, int64_t H,
                 torch::Tensor out) {
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && out.scalar_type() == torch::kFloat32, "moe_combine: fp32");
  vmc::moe_combine(ptr<float>(y), static_cast<int>(y.stride(0)), ptr<int32_t>(slot_row), ptr<float>(topk_w),
                   static_cast<int>(T), static_cast<int>(k), static_cast<int>(H), ptr<float>(out),
                   static_cast<int>(out.stride(0)), cur_stream());
}

void repack_weight(int wf, int src_type, torch::Tensor src, int64_t N, int64_t K, torch::Tensor dst) {
  check_cuda(src, "src");
  check_cuda(dst, "dst");
  TORCH_CHECK(dst.numel() * dst.element_size() >= vmc::tiled_weight_bytes(wf, N, K), "repack: dst too small");
  vmc::repack_weight(wf, src_type, src.data_ptr(), static_cast<int>(N), static_cast<int>(K), dst.data_ptr(),
                     cur_stream());
}

void untile_bf16(torch::Tensor tiles, int64_t N, int64_t K, torch::Tensor out) {
  vmc::untile_bf16(tiles.data_ptr(), static_cast<int>(N), static_cast<int>(K), out.data_ptr(), cur_stream());
}

void quantize_blocks(int gtype, torch::Tensor x, torch::Tensor out) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "quantize: x must be contiguous fp32");
  vmc::quantize_blocks(gtype, ptr<float>(x), x.numel(), out.data_ptr(), cur_stream());
}

// TurboQuant layer description from Python: meta = [slot, mse_bytes, key_packed, val_bytes, key_bits,
// value_bits, norm_correction, key_fp8, rot_seed, layer].
vmc::TqDev make_tq(torch::Tensor cache, const std::vector<int64_t>& meta, torch::Tensor centroids,
                   torch::Tensor midpoints) {
  TORCH_CHECK(meta.size() == 10, "turboquant: meta must have 10 entries");
  TORCH_CHECK(cache.scalar_type() == torch::kUInt8 && cache.is_cuda(), "turboquant: cache must be uint8 CUDA");
  TORCH_CHECK(centroids.scalar_type() == torch::kFloat32 && midpoints.scalar_type() == torch::kFloat32,
              "turboquant: fp32 centroid tables");
  vmc::TqDev t;
  t.cache = cache.data_ptr<uint8_t>();
  t.slot = static_cast<int>(meta[0]);
  t.mse_bytes = static_cast<int>(meta[1]);
  t.key_packed = static_cast<int>(meta[2]);
  t.val_bytes = static_cast<int>(meta[3]);
  t.key_bits = static_cast<int>(meta[4]);
  t.value_bits = static_cast<int>(meta[5]);
  t.norm_correction = static_cast<int>(meta[6]);
  t.key_fp8 = static_cast<int>(meta[7]);
  t.rot_seed = static_cast<uint32_t>(meta[8]);
  t.layer = static_cast<int>(meta[9]);
  t.centroids = centroids.data_ptr<float>();
  t.midpoints = midpoints.data_ptr<float>();
  return t;
}

void rope_store_tq(torch::Tensor qkv, int64_t nsplit, int64_t split_stride, int64_t T, int64_t Hq, int64_t Hkv,
                   int64_t D, torch::Tensor pos, torch::Tensor slots, torch::Tensor cos_sin, bool neox,
                   torch::Tensor q_out, torch::Tensor cache, std::vector<int64_t> meta, torch::Tensor centroids,
                   torch::Tensor midpoints) {
  const vmc::TqDev t = make_tq(cache, meta, centroids, midpoints);
  vmc::rope_store_tq(qkv.data_ptr(), qkv.scalar_type() == torch::kFloat32, static_cast<int>(nsplit), split_stride,
                     static_cast<int>(T), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(D),
                     ptr<int32_t>(pos), ptr<int32_t>(slots), ptr<float>(cos_sin), neox, q_out.data_ptr(), t,
                     cur_stream());
}

void paged_attention(torch::Tensor q, torch::Tensor kv, torch::Tensor q_start, torch::Tensor ctx_len,
                     torch::Tensor block_tables, int64_t num_reqs, int64_t req_offset, int64_t max_qlen,
                     int64_t total_tokens, int64_t Hq, int64_t Hkv, int64_t D, double scale, bool decode,
                     int64_t splits, c10::optional<torch::Tensor> part_o, c10::optional<torch::Tensor> part_lse,
                     torch::Tensor out, c10::optional<torch::Tensor> tq_cache, std::vector<int64_t> tq_meta,
                     c10::optional<torch::Tensor> tq_centroids, c10::optional<torch::Tensor> tq_midpoints,
                     c10::optional<torch::Tensor> tree_mask, int64_t tree_span, c10::optional<torch::Tensor> err) {
  vmc::TqDev tq;
  const bool use_tq = tq_cache.has_value() && tq_cache->defined();
  if (use_tq) tq = make_tq(*tq_cache, tq_meta, *tq_centroids, *tq_midpoints);
  vmc::AttnLaunch a;
  a.q = q.data_ptr();
  a.kv = kv.data_ptr();
  a.q_start = ptr<int32_t>(q_start);
  a.ctx_len = ptr<int32_t>(ctx_len);
  a.block_tables = ptr<int32_t>(block_tables);
  a.max_blocks = static_cast<int>(block_tables.size(-1));
  a.num_reqs = static_cast<int>(num_reqs);
  a.req_offset = static_cast<int>(req_offset);
  a.max_qlen = static_cast<int>(max_qlen);
  a.total_tokens = static_cast<int>(total_tokens);
  a.Hq = static_cast<int>(Hq);
  a.Hkv = static_cast<int>(Hkv);
  a.D = static_cast<int>(D);
  a.scale = static_cast<float>(scale);
  a.decode = decode;
  a.splits = static_cast<int>(splits);
  a.part_o = opt_ptr<float>(part_o);
  a.part_lse = opt_ptr<float>(part_lse);
  a.out = out.data_ptr();
  a.tq = use_tq ? &tq : nullptr;
  if (!use_tq && kv.dim() == 5 && kv.scalar_type() == torch::kBFloat16) a.num_blocks = kv.size(0);
  if (err.has_value() && err->defined()) a.err = ptr<uint32_t>(*err);
  if (tree_mask.has_value() && tree_mask->defined()) {
    TORCH_CHECK(tree_mask->scalar_type() == torch::kInt64 && tree_mask->numel() >= total_tokens,
                "paged_attention: tree_mask must be int64 [T]");
    a.tree_mask = reinterpret_cast<const uint64_t*>(tree_mask->data_ptr());
    a.tree_span = static_cast<int>(tree_span);
  }
  vmc::paged_attention(a, cur_stream());
}

void kv_move(torch::Tensor cache, int64_t Hkv, int64_t D, torch::Tensor src, torch::Tensor dst, torch::Tensor cnt,
             int64_t num_reqs, int64_t max_moves) {
  check_cuda(cache, "cache");
  TORCH_CHECK(cache.scalar_type() == torch::kBFloat16 && cache.dim() == 6, "kv_move: bf16 [L, blocks, 2, Hkv, 16, D]");
  vmc::kv_move(cache.data_ptr(), static_cast<int>(cache.size(0)), cache.stride(0), static_cast<int>(Hkv),
               static_cast<int>(D), ptr<int32_t>(src), ptr<int32_t>(dst), ptr<int32_t>(cnt), static_cast<int>(num_reqs),
               static_cast<int>(max_moves), cur_stream());
}

void gdn_conv(torch::Tensor x, torch::Tensor w, torch::Tensor q_start, torch::Tensor slot, torch::Tensor has_state,
              int64_t nseq, torch::Tensor conv_state, torch::Tensor y) {
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && y.scalar_type() == torch::kFloat32 && x.stride(1) == 1 &&
                  y.stride(1) == 1, "gdn_conv: fp32 row-major x and y");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.size(0) == x.size(1), "gdn_conv: w [C, K] contiguous");
  const int64_t C = w.size(0), K = w.size(1);
  TORCH_CHECK(conv_state.is_contiguous() && conv_state.dim() == 3 && conv_state.size(1) == K - 1 &&
                  conv_state.size(2) == C, "gdn_conv: conv_state [slots, K-1, C]");
  vmc::gdn_conv(ptr<float>(x), x.stride(0), ptr<float>(w), static_cast<int>(C), static_cast<int>(K),
                ptr<int32_t>(q_start), ptr<int32_t>(slot), ptr<int32_t>(has_state), static_cast<int>(nseq),
                ptr<float>(conv_state), ptr<float>(y), y.stride(0), cur_stream());
}

void gdn_recurrent(torch::Tensor qkv, torch::Tensor alpha, torch::Tensor beta, torch::Tensor z, torch::Tensor a_neg,
                   torch::Tensor dt_bias, torch::Tensor norm_w, torch::Tensor state, torch::Tensor slot,
                   torch::Tensor has_state, torch::Tensor q_start, int64_t nseq, int64_t Hk, double eps,
                   torch::Tensor out) {
  check_cuda(qkv, "qkv");
  TORCH_CHECK(state.is_contiguous() && state.dim() == 4 && state.size(2) == state.size(3) &&
                  state.scalar_type() == torch::kFloat32, "gdn_recurrent: state [slots, Hv, D, D] fp32");
  const int64_t Hv = state.size(1), D = state.size(2);
  TORCH_CHECK(qkv.scalar_type() == torch::kFloat32 && qkv.stride(1) == 1 && qkv.size(1) >= (2 * Hk + Hv) * D,
              "gdn_recurrent: qkv [T, (2Hk+Hv)D] fp32");
  TORCH_CHECK(alpha.stride(1) == 1 && beta.stride(1) == 1 && alpha.stride(0) == beta.stride(0) &&
                  alpha.scalar_type() == torch::kFloat32 && beta.scalar_type() == torch::kFloat32,
              "gdn_recurrent: alpha/beta fp32 [T, Hv] with one row stride");
  TORCH_CHECK(z.scalar_type() == torch::kFloat32 && z.stride(1) == 1 && out.scalar_type() == torch::kBFloat16 &&
                  out.stride(1) == 1, "gdn_recurrent: z fp32, out bf16");
  vmc::GdnArgs a{};
  a.qkv = ptr<float>(qkv);
  a.qkv_stride = qkv.stride(0);
  a.alpha = ptr<float>(alpha);
  a.beta = ptr<float>(beta);
  a.ab_stride = alpha.stride(0);
  a.z = ptr<float>(z);
  a.z_stride = z.stride(0);
  a.a_neg = ptr<float>(a_neg);
  a.dt_bias = ptr<float>(dt_bias);
  a.norm_w = ptr<float>(norm_w);
  a.state = ptr<float>(state);
  a.slot = ptr<int32_t>(slot);
  a.has_state = ptr<int32_t>(has_state);
  a.q_start = ptr<int32_t>(q_start);
  a.out = static_cast<__nv_bfloat16*>(out.data_ptr());
  a.out_stride = out.stride(0);
  a.Hk = static_cast<int>(Hk);
  a.Hv = static_cast<int>(Hv);
  a.D = static_cast<int>(D);
  a.eps = static_cast<float>(eps);
  vmc::gdn_recurrent(a, static_cast<int>(nseq), cur_stream());
}

void embed(torch::Tensor ids, int64_t T, torch::Tensor table, int gtype, int64_t row_bytes, int64_t H,
           c10::optional<torch::Tensor> resid, c10::optional<torch::Tensor> out_bf16) {
  vmc::embed(ptr<int32_t>(ids), static_cast<int>(T), table.data_ptr(), gtype, row_bytes, static_cast<int>(H),
             opt_ptr<float>(resid), opt_ptr<void>(out_bf16), cur_stream());
}

void add_rmsnorm(torch::Tensor resid, c10::optional<torch::Tensor> delta, int64_t ndelta, int64_t delta_stride,
                 torch::Tensor w, int64_t T, int64_t H, double eps, c10::optional<torch::Tensor> out) {
  TORCH_CHECK(resid.scalar_type() == torch::kFloat32, "add_rmsnorm: residual must be fp32");
  const bool f32 = delta.has_value() && delta->defined() && delta->scalar_type() == torch::kFloat32;
  vmc::add_rmsnorm(ptr<float>(resid), opt_ptr<void>(delta), f32, static_cast<int>(ndelta), delta_stride, ptr<float>(w),
                   static_cast<int>(T), static_cast<int>(H), static_cast<float>(eps), opt_ptr<void>(out), cur_stream());
}

void rope_store(torch::Tensor qkv, int64_t nsplit, int64_t split_stride, int64_t T, int64_t Hq, int64_t Hkv,
                int64_t D, torch::Tensor pos, torch::Tensor slots, torch::Tensor cos_sin, bool neox,
                torch::Tensor q_out, torch::Tensor kv) {
  vmc::rope_store(qkv.data_ptr(), qkv.scalar_type() == torch::kFloat32, static_cast<int>(nsplit), split_stride,
                  static_cast<int>(T), static_cast<int>(Hq),
                  static_cast<int>(Hkv), static_cast<int>(D), ptr<int32_t>(pos), ptr<int32_t>(slots),
                  ptr<float>(cos_sin), neox, q_out.data_ptr(), kv.data_ptr(), cur_stream());
}

void swiglu(torch::Tensor gu, int64_t nsplit, int64_t split_stride, int64_t T, int64_t F, bool interleaved,
            torch::Tensor out) {
  vmc::swiglu(gu.data_ptr(), gu.scalar_type() == torch::kFloat32, static_cast<int>(nsplit), split_stride, T,
              static_cast<int>(F), interleaved, out.data_ptr(), cur_stream());
}

void gather_rows(torch::Tensor src, torch::Tensor idx, int64_t n, int64_t H, torch::Tensor dst) {
  vmc::gather_rows(src.data_ptr(), ptr<int32_t>(idx), static_cast<int>(n), static_cast<int>(H), dst.data_ptr(),
                   cur_stream());
}

void f32_to_bf16(torch::Tensor x, int64_t n, torch::Tensor y) {
  vmc::f32_to_bf16(ptr<float>(x), n, y.data_ptr(), cur_stream());
}

void sample(torch::Tensor logits, int64_t S, int64_t V, torch::Tensor params, torch::Tensor out_tok,
            c10::optional<torch::Tensor> out_lp) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32, "sample: logits must be fp32");
  vmc::sample(ptr<float>(logits), static_cast<int>(S), static_cast<int>(V), logits.stride(0),
              reinterpret_cast<const vmc::SampleParams*>(params.data_ptr()), ptr<int32_t>(out_tok),
              opt_ptr<float>(out_lp), cur_stream());
}

void apply_penalties(torch::Tensor logits, torch::Tensor row_of, torch::Tensor tok, torch::Tensor out_count,
                     torch::Tensor params, int64_t n) {
  vmc::apply_penalties(ptr<float>(logits), logits.stride(0), ptr<int32_t>(row_of), ptr<int32_t>(tok),
                       ptr<int32_t>(out_count), reinterpret_cast<const vmc::SampleParams*>(params.data_ptr()),
                       static_cast<int>(n), cur_stream());
}

void ar_add_rmsnorm(std::vector<int64_t> data, std::vector<int64_t> flags, torch::Tensor epochs, int64_t rank,
                    int64_t T, int64_t H, int64_t nsplit, int64_t split_stride, torch::Tensor resid, torch::Tensor w,
                    double eps, torch::Tensor out, torch::Tensor err, int64_t max_ctas) {
  vmc::ArArgs a;
  TORCH_CHECK(data.size() == flags.size() && !data.empty() && data.size() <= 8, "ar_add_rmsnorm: bad peer lists");
  for (size_t i = 0; i < 8; ++i) {
    a.data[i] = i < data.size() ? reinterpret_cast<const float*>(data[i]) : nullptr;
    a.flags[i] = i < flags.size() ? reinterpret_cast<uint32_t*>(flags[i]) : nullptr;
  }
  a.epochs = ptr<uint32_t>(epochs);
  a.nranks = static_cast<int>(data.size());
  a.rank = static_cast<int>(rank);
  a.T = static_cast<int>(T);
  a.H = static_cast<int>(H);
  a.nsplit = static_cast<int>(nsplit);
  a.split_stride = split_stride;
  a.resid = ptr<float>(resid);
  a.w = ptr<float>(w);
  a.eps = static_cast<float>(eps);
  a.out = out.data_ptr();
  a.err = ptr<uint32_t>(err);
  vmc::ar_add_rmsnorm(a, static_cast<int>(max_ctas), cur_stream());
}

py::tuple sym_alloc(int64_t bytes) {
  char h[64];
  uint64_t p = vmc::sym_alloc(static_cast<size_t>(bytes), h);
  return py::make_tuple(static_cast<int64_t>(p), py::bytes(h, 64));
}
int64_t sym_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == 64, "sym_open: handle must be 64 bytes");
  return static_cast<int64_t>(vmc::sym_open(s.data()));
}
// A torch view over raw device memory owned elsewhere (symmetric buffers).
torch::Tensor wrap_ptr(int64_t p, std::vector<int64_t> sizes, int dtype, int device) {
  auto opts = torch::TensorOptions().dtype(static_cast<c10::ScalarType>(dtype)).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(p), sizes, opts);
}

// ---- native step forward (forward.h) ----------------------------------------------------------
// Layers arrive as flat int lists: [attn_norm, ffn_norm, n_qkv, (wf, ptr, N, K) x 3, col x 3,
// wo (4), gate_up (4), down (4)]; pointers are device addresses of tensors the Python model owns.
vmc::LinearDesc lin_at(const std::vector<int64_t>& v, size_t o) {
  vmc::LinearDesc d;
  d.wf = static_cast<int>(v[o]);
  d.w = reinterpret_cast<const void*>(v[o + 1]);
  d.N = static_cast<int>(v[o + 2]);
  d.K = static_cast<int>(v[o + 3]);
  return d;
}
template <typename T>
T* dptr(const py::dict& d, const char* k) {
  return d.contains(k) ? reinterpret_cast<T*>(d[k].cast<int64_t>()) : nullptr;
}

std::shared_ptr<vmc::Forward> make_forward(py::dict cfg, std::vector<std::vector<int64_t>> layers, py::dict bufs) {
  vmc::ForwardConfig c;
  c.L = cfg["L"].cast<int>();
  c.H = cfg["H"].cast<int>();
  c.Hq = cfg["Hq"].cast<int>();
  c.Hkv = cfg["Hkv"].cast<int>();
  c.D = cfg["D"].cast<int>();
  c.F = cfg["F"].cast<int>();
  c.V_local = cfg["V_local"].cast<int>();
  c.max_tokens = cfg["max_tokens"].cast<int>();
  c.max_samples = cfg["max_samples"].cast<int>();
  c.max_blocks = cfg["max_blocks"].cast<int>();
  c.eps = cfg["eps"].cast<float>();
  c.scale = cfg["scale"].cast<float>();
  c.neox = cfg["neox"].cast<bool>();
  c.embd = dptr<const void>(cfg, "embd");
  c.embd_type = cfg["embd_type"].cast<int>();
  c.embd_row_bytes = cfg["embd_row_bytes"].cast<int64_t>();
  c.out_norm = dptr<const float>(cfg, "out_norm");
  c.lm_head = lin_at(cfg["lm_head"].cast<std::vector<int64_t>>(), 0);
  c.cos_sin = dptr<const float>(cfg, "cos_sin");
  c.num_sms = cfg["num_sms"].cast<int>();
  std::vector<vmc::LayerDesc> ls;
  for (const auto& v : layers) {
    TORCH_CHECK(v.size() == 30 || v.size() == 48, "make_forward: layer descriptors have 30 (dense) or 48 (MoE) entries");
    vmc::LayerDesc d;
    d.attn_norm = reinterpret_cast<const float*>(v[0]);
    d.ffn_norm = reinterpret_cast<const float*>(v[1]);
    d.n_qkv = static_cast<int>(v[2]);
    for (int i = 0; i < 3; ++i) {
      d.qkv[i] = lin_at(v, 3 + 4 * i);
      d.qkv_col[i] = static_cast<int>(v[15 + i]);
    }
    d.wo = lin_at(v, 18);
    d.gate_up = lin_at(v, 22);
    d.down = lin_at(v, 26);
    if (v.size() == 48) {  // [30] = 1, router (4), gate_up (4), stride, down (4), stride, e0, e_local, f_local
      d.moe = v[30] != 0;
      d.m.router = lin_at(v, 31);
      d.m.gate_up = lin_at(v, 35);
      d.m.gate_up_stride = v[39];
      d.m.down = lin_at(v, 40);
      d.m.down_stride = v[44];
      d.m.e0 = static_cast<int>(v[45]);
      d.m.e_local = static_cast<int>(v[46]);
      d.m.f_local = static_cast<int>(v[47]);
    }
    ls.push_back(d);
  }
  vmc::ForwardBuffers b;
  b.resid = dptr<float>(bufs, "resid");
  b.h = dptr<void>(bufs, "h");
  b.qkv_bf16 = dptr<void>(bufs, "qkv_bf16");
  b.split_ws = dptr<float>(bufs, "split_ws");
  b.split_ws_elems = bufs["split_ws_elems"].cast<int64_t>();
  b.q = dptr<void>(bufs, "q");
  b.attn = dptr<void>(bufs, "attn");
  b.o16 = dptr<void>(bufs, "o16");
  b.act = dptr<void>(bufs, "act");
  b.hs = dptr<void>(bufs, "hs");
  b.logits = dptr<float>(bufs, "logits");
  b.part_o = dptr<float>(bufs, "part_o");
  b.part_lse = dptr<float>(bufs, "part_lse");
  b.attn_max_splits = bufs["attn_max_splits"].cast<int>();
  b.ids = dptr<const int32_t>(bufs, "ids");
  b.pos = dptr<const int32_t>(bufs, "pos");
  b.slots = dptr<const int32_t>(bufs, "slots");
  b.q_start = dptr<const int32_t>(bufs, "q_start");
  b.ctx_len = dptr<const int32_t>(bufs, "ctx_len");
  b.block_tables = dptr<const int32_t>(bufs, "block_tables");
  b.logits_idx = dptr<const int32_t>(bufs, "logits_idx");
  b.params = dptr<const void>(bufs, "params");
  b.out_tok = dptr<int32_t>(bufs, "out_tok");
  b.out_lp = dptr<float>(bufs, "out_lp");
  b.kv = dptr<void>(bufs, "kv");
  b.kv_layer_bytes = bufs["kv_layer_bytes"].cast<int64_t>();
  b.err = dptr<uint32_t>(bufs, "err");
  if (bufs.contains("tq_meta")) {
    const auto meta = bufs["tq_meta"].cast<std::vector<int64_t>>();
    TORCH_CHECK(meta.size() == 10, "make_forward: tq_meta must have 10 entries");
    b.tq = true;
    b.tq_tab.slot = static_cast<int>(meta[0]);
    b.tq_tab.mse_bytes = static_cast<int>(meta[1]);
    b.tq_tab.key_packed = static_cast<int>(meta[2]);
    b.tq_tab.val_bytes = static_cast<int>(meta[3]);
    b.tq_tab.key_bits = static_cast<int>(meta[4]);
    b.tq_tab.value_bits = static_cast<int>(meta[5]);
    b.tq_tab.norm_correction = static_cast<int>(meta[6]);
    b.tq_tab.key_fp8 = static_cast<int>(meta[7]);
    b.tq_tab.rot_seed = static_cast<uint32_t>(meta[8]);
    b.tq_tab.centroids = dptr<const float>(bufs, "tq_centroids");
    b.tq_tab.midpoints = dptr<const float>(bufs, "tq_midpoints");
  }
  return std::make_shared<vmc::Forward>(c, std::move(ls), b);
}

// TpComm from Python: peer address lists of the symmetric region.
vmc::TpComm make_tp_comm(py::dict d) {
  vmc::TpComm c;
  c.nranks = d["nranks"].cast<int>();
  c.rank = d["rank"].cast<int>();
  TORCH_CHECK(c.nranks >= 1 && c.nranks <= 8, "tp comm: 1..8 ranks");
  c.recv_rows = d["recv_rows"].cast<int64_t>();
  c.max_ctas = d["max_ctas"].cast<int>();
  const auto recv0 = d["recv0"].cast<std::vector<int64_t>>(), recv1 = d["recv1"].cast<std::vector<int64_t>>();
  const auto h = d["h"].cast<std::vector<int64_t>>();
  const auto rs0 = d["rs0"].cast<std::vector<int64_t>>(), rs1 = d["rs1"].cast<std::vector<int64_t>>();
  const auto ag0 = d["ag0"].cast<std::vector<int64_t>>(), ag1 = d["ag1"].cast<std::vector<int64_t>>();
  const auto ag2 = d.contains("ag2") ? d["ag2"].cast<std::vector<int64_t>>() : ag1;
  for (int q = 0; q < c.nranks; ++q) {
    c.recv[0][q] = reinterpret_cast<void*>(recv0.at(q));
    c.recv[1][q] = reinterpret_cast<void*>(recv1.at(q));
    c.h[q] = reinterpret_cast<void*>(h.at(q));
    c.rs_count[0][q] = reinterpret_cast<uint32_t*>(rs0.at(q));
    c.rs_count[1][q] = reinterpret_cast<uint32_t*>(rs1.at(q));
    c.ag_count[0][q] = reinterpret_cast<uint32_t*>(ag0.at(q));
    c.ag_count[1][q] = reinterpret_cast<uint32_t*>(ag1.at(q));
    c.ag_count[2][q] = reinterpret_cast<uint32_t*>(ag2.at(q));
  }
  c.state = reinterpret_cast<uint32_t*>(d["state"].cast<int64_t>());
  c.err = reinterpret_cast<uint32_t*>(d["err"].cast<int64_t>());
  return c;
}

vmc::MoeBuffers make_moe(py::dict d) {
  vmc::MoeBuffers m;
  m.E = d["E"].cast<int>();
  m.k = d["k"].cast<int>();
  m.norm_topk = d["norm_topk"].cast<int>();
  m.ep = d["ep"].cast<bool>();
  m.logits = dptr<float>(d, "logits");
  m.topk_id = dptr<int32_t>(d, "topk_id");
  m.topk_w = dptr<float>(d, "topk_w");
  m.counts = dptr<int32_t>(d, "counts");
  m.offsets = dptr<int32_t>(d, "offsets");
  m.sorted_src = dptr<int32_t>(d, "sorted_src");
  m.slot_row = dptr<int32_t>(d, "slot_row");
  m.total = dptr<int32_t>(d, "total");
  m.xs = dptr<void>(d, "xs");
  m.act = dptr<void>(d, "act");
  m.y = dptr<float>(d, "y");
  m.out = dptr<float>(d, "out");
  if (m.ep) {
    m.cap = d["cap"].cast<int>();
    const auto rx = d["recv_x"].cast<std::vector<int64_t>>(), rr = d["recv_ret"].cast<std::vector<int64_t>>();
    const auto c0 = d["cnt0"].cast<std::vector<int64_t>>(), c1 = d["cnt1"].cast<std::vector<int64_t>>();
    const auto cb = d["comb"].cast<std::vector<int64_t>>(), da = d["disp_arrive"].cast<std::vector<int64_t>>();
    const auto ca = d["comb_arrive"].cast<std::vector<int64_t>>();
    for (size_t q = 0; q < rx.size() && q < 8; ++q) {
      m.recv_x[q] = reinterpret_cast<void*>(rx[q]);
      m.recv_ret[q] = reinterpret_cast<int32_t*>(rr[q]);
      m.cnt[0][q] = reinterpret_cast<uint32_t*>(c0[q]);
      m.cnt[1][q] = reinterpret_cast<uint32_t*>(c1[q]);
      m.comb[q] = reinterpret_cast<void*>(cb[q]);
      m.disp_arrive[q] = reinterpret_cast<uint32_t*>(da[q]);
      m.comb_arrive[q] = reinterpret_cast<uint32_t*>(ca[q]);
    }
    m.disp_state = dptr<uint32_t>(d, "disp_state");
    m.ep_logits = dptr<float>(d, "ep_logits");
    m.ep_topk_w = dptr<float>(d, "ep_topk_w");
    m.ep_act = dptr<void>(d, "ep_act");
    m.ep_offsets = dptr<int32_t>(d, "ep_offsets");
  }
  return m;
}

vmc::TpSample make_tp_sample(py::dict d) {
  vmc::TpSample t;
  t.nranks = d["nranks"].cast<int>();
  t.rank = d["rank"].cast<int>();
  t.max_rows = d["max_rows"].cast<int>();
  const auto xs = d["xbuf"].cast<std::vector<int64_t>>(), cs = d["xcount"].cast<std::vector<int64_t>>();
  for (int q = 0; q < t.nranks; ++q) {
    t.xbuf[q] = reinterpret_cast<void*>(xs.at(q));
    t.count[q] = reinterpret_cast<uint32_t*>(cs.at(q));
  }
  t.state = reinterpret_cast<uint32_t*>(d["xstate"].cast<int64_t>());
  t.err = reinterpret_cast<uint32_t*>(d["err"].cast<int64_t>());
  return t;
}

void tp_sample(py::dict d, torch::Tensor logits, int64_t S, int64_t V_local, torch::Tensor params, torch::Tensor out_tok,
               c10::optional<torch::Tensor> out_lp) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1, "tp_sample: fp32 logits");
  vmc::tp_sample(make_tp_sample(d), ptr<float>(logits), static_cast<int>(S), static_cast<int>(V_local),
                 logits.stride(0), reinterpret_cast<const vmc::SampleParams*>(params.data_ptr()), ptr<int32_t>(out_tok),
                 opt_ptr<float>(out_lp), cur_stream());
}

// One reduce-scatter + norm + all-gather site driven from Python (tests and the comm benchmark):
// x [M, K] bf16 times the tiled weight, partial rows scattered, then rs_norm_ag.
int64_t tp_row_parallel(py::dict comm, int site, int wf, torch::Tensor w, int64_t N, int64_t K, torch::Tensor x,
                        int64_t M, int64_t splits, torch::Tensor resid, torch::Tensor norm_w, double eps,
                        torch::Tensor err) {
  const vmc::TpComm c = make_tp_comm(comm);
  int used = static_cast<int>(splits);
  const int grid = vmc::gemm_tcgen05_scatter(
      wf, w.data_ptr(), static_cast<int>(N), static_cast<int>(K), x.data_ptr(), static_cast<int>(M),
      static_cast<int>(x.stride(0)), static_cast<int>(splits), c.recv[site], c.rs_count[site], c.nranks, c.rank,
      c.recv_rows, ptr<uint32_t>(err), cur_stream(), &used, vmc::tp_scatter_local(c, site));
  vmc::rs_norm_ag(c, site, static_cast<int>(M), static_cast<int>(N), used, vmc::tp_scatter_arrivals(c, grid),
                  ptr<float>(resid),
                  ptr<float>(norm_w), static_cast<float>(eps), cur_stream());
  return used;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "vm_c_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("moe_route", &moe_route);
  m.def("moe_combine", &moe_combine);
  m.def("gemm_smem_bytes", &vmc::gemm_smem_bytes);
  m.def("gemm_set_trace", [](c10::optional<torch::Tensor> t) {
    vmc::gemm_set_trace(t.has_value() && t->defined() ? reinterpret_cast<unsigned long long*>(t->data_ptr()) : nullptr);
  });
  m.def("gemm_pick_bn", &vmc::gemm_pick_bn);
  m.def("gemm_prepare", &vmc::gemm_prepare);
  m.def("tiled_weight_bytes", &vmc::tiled_weight_bytes);
  m.def("repack_weight", &repack_weight);
  m.def("untile_bf16", &untile_bf16);
  m.def("quantize_blocks", &quantize_blocks);
  m.def("paged_attention", &paged_attention, py::arg("q"), py::arg("kv"), py::arg("q_start"), py::arg("ctx_len"),
        py::arg("block_tables"), py::arg("num_reqs"), py::arg("req_offset"), py::arg("max_qlen"),
        py::arg("total_tokens"), py::arg("Hq"), py::arg("Hkv"), py::arg("D"), py::arg("scale"), py::arg("decode"),
        py::arg("splits"), py::arg("part_o"), py::arg("part_lse"), py::arg("out"), py::arg("tq_cache") = py::none(),
        py::arg("tq_meta") = std::vector<int64_t>{}, py::arg("tq_centroids") = py::none(),
        py::arg("tq_midpoints") = py::none(), py::arg("tree_mask") = py::none(), py::arg("tree_span") = 0,
        py::arg("err") = py::none());
  m.def("attention_tc", [](bool on) { vmc::attn_prefill_tc_enable(on ? 1 : 0); },
        "route bf16 head-dim-128 prefill attention to the tcgen05 kernel (true) or the mma.sync kernel");
  m.def("kv_move", &kv_move);
  m.def("rope_store_tq", &rope_store_tq);
  m.def("embed", &embed);
  m.def("add_rmsnorm", &add_rmsnorm);
  m.def("rope_store", &rope_store);
  m.def("gdn_conv", &gdn_conv);
  m.def("gdn_recurrent", &gdn_recurrent);
  m.def("swiglu", &swiglu);
  m.def("gather_rows", &gather_rows);
  m.def("f32_to_bf16", &f32_to_bf16);
  m.def("attn_decode_ctas_per_sm", &vmc::attn_decode_ctas_per_sm);
  m.def("sample", &sample);
  m.def("apply_penalties", &apply_penalties);
  m.def("ar_add_rmsnorm", &ar_add_rmsnorm);
  m.def("sym_alloc", &sym_alloc);
  m.def("sym_open", &sym_open);
  m.def("sym_close", [](int64_t p) { vmc::sym_close(static_cast<uint64_t>(p)); });
  m.def("sym_free", [](int64_t p) { vmc::sym_free(static_cast<uint64_t>(p)); });
  m.def("wrap_ptr", &wrap_ptr);
  py::class_<vmc::Forward, std::shared_ptr<vmc::Forward>>(m, "Forward")
      .def("run",
           [](vmc::Forward& f, int T, int R, int S, int nd, int max_qlen, int decode_qlen, int attn_splits,
              bool do_sample) {
             vmc::StepDims d;
             d.T = T;
             d.R = R;
             d.S = S;
             d.nd = nd;
             d.max_qlen = max_qlen;
             d.decode_qlen = decode_qlen;
             d.attn_splits = attn_splits;
             d.sample = do_sample;
             return f.run(d, cur_stream());
           })
      .def("set_comm", [](vmc::Forward& f, py::dict d) {
        f.set_comm(make_tp_comm(d));
        f.set_sampler(make_tp_sample(d));
      })
      .def("set_moe", [](vmc::Forward& f, py::dict d) { f.set_moe(make_moe(d)); })
      .def("splits_for", [](vmc::Forward& f, int wf, int N, int K, int M) {
        vmc::LinearDesc w;
        w.wf = wf;
        w.N = N;
        w.K = K;
        return f.splits_for(w, M);
      });
  m.def("make_forward", &make_forward);
  m.def("tp_row_parallel", &tp_row_parallel);
  m.def("tp_sample", &tp_sample);
  m.def("tp_sample_row_bytes", &vmc::tp_sample_row_bytes);
  m.def("gemm_pick_splits", [](int wf, int N, int K, int M, int sms) { return vmc::gemm_pick_splits(wf, N, K, M, sms); });
  m.attr("OUT_BF16") = static_cast<int>(vmc::kGemmOutBF16);
  m.attr("OUT_F32") = static_cast<int>(vmc::kGemmOutF32);
  m.attr("OUT_F32_ADD") = static_cast<int>(vmc::kGemmOutF32Add);
  m.attr("OUT_SWIGLU") = static_cast<int>(vmc::kGemmOutSwiGLU);
  m.attr("OUT_F32_SPLIT") = static_cast<int>(vmc::kGemmOutF32Split);
}
