// vmc_run: the serving loop without Python or PyTorch.
//
// Loads a llama-architecture GGUF onto one GPU, tiles its weights for the tcgen05 GEMMs, and serves a
// closed batch of prompts with the native continuous-batching scheduler (csrc/host/scheduler.cpp),
// the native step forward (csrc/kernels/forward.cpp) and decode steps replayed from CUDA graphs
// captured per batch bucket. Device buffers are owned with cudaMalloc; kernels are called through their
// C++ launchers. Counterpart of the reference's main step loop and engine
// (src/main.cpp:331, :813-840; src/core/engine.cpp:493-556), which drive libllama.
//
//   vmc_run MODEL.gguf --prompts FILE [--gen N] [--max-num-seqs S] [--max-num-batched-tokens T]
//           [--max-model-len L] [--num-blocks B] [--no-graphs] [--dump-tokens FILE.json] [--runs K]
//           [--warmup W]
//   vmc_run MODEL.gguf --serve [--host H] [--port P] [--model-name NAME] [--port-file PATH]
//           [--max-num-seqs S] [--max-num-batched-tokens T] [--max-model-len L] [--num-blocks B] [--no-graphs]
//
// --prompts: little-endian int32 count, int32 length, then count * length token ids. Greedy decoding
// with ignore_eos (every request produces N tokens). One JSON line on stdout: device time of the timed
// runs, output tokens/s, p50 time to first token and inter-token latency.
//
// --serve: the OpenAI-compatible HTTP server (csrc/server/) over the same engine. The serving loop runs
// on the main thread (it owns the stream, the graphs and the scheduler); HTTP connections are served on
// their own threads. Sampling parameters and penalties come from each request (the sampler kernels of
// sampling.cu); SIGINT / SIGTERM stop it. Counterpart of the reference's server mode
// (src/main.cpp:521-794 with src/server/http_server.cpp).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "attention.h"
#include "block_manager.hpp"
#include "forward.h"
#include "gemm_tcgen05.h"
#include "gguf.hpp"
#include "http.hpp"
#include "openai.hpp"
#include "quants.hpp"
#include "sampling.h"
#include "scheduler.hpp"
#include "serve_loop.hpp"
#include "stop_signals.hpp"
#include "text_tokenizer.hpp"
#include "weights.h"

namespace {

using vmc::GType;

#define CK(x)                                                                                        \
  do {                                                                                               \
    cudaError_t e_ = (x);                                                                            \
    if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

struct Args {
  std::string model, prompts, dump;
  int gen = 16, max_seqs = 64, max_batched = 2048, max_model_len = 0, runs = 1, warmup = 0, num_blocks = 0;
  bool graphs = true;
  // --serve
  bool serve = false;
  std::string host = "127.0.0.1", model_name, port_file;
  int port = 8000;
};

Args parse(int argc, char** argv) {
  Args a;
  if (argc < 2) throw std::runtime_error("usage: vmc_run MODEL.gguf --prompts FILE [options]");
  a.model = argv[1];
  for (int i = 2; i < argc; ++i) {
    const std::string k = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + k);
      return argv[++i];
    };
    if (k == "--prompts") a.prompts = val();
    else if (k == "--dump-tokens") a.dump = val();
    else if (k == "--gen") a.gen = std::stoi(val());
    else if (k == "--max-num-seqs") a.max_seqs = std::stoi(val());
    else if (k == "--max-num-batched-tokens") a.max_batched = std::stoi(val());
    else if (k == "--max-model-len") a.max_model_len = std::stoi(val());
    else if (k == "--runs") a.runs = std::stoi(val());
    else if (k == "--warmup") a.warmup = std::stoi(val());
    else if (k == "--num-blocks") a.num_blocks = std::stoi(val());
    else if (k == "--no-graphs") a.graphs = false;
    else if (k == "--serve") a.serve = true;
    else if (k == "--host") a.host = val();
    else if (k == "--port") a.port = std::stoi(val());
    else if (k == "--model-name") a.model_name = val();
    else if (k == "--port-file") a.port_file = val();
    else throw std::runtime_error("unknown option " + k);
  }
  return a;
}

// ---- device memory -------------------------------------------------------------------------------

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  DevBuf() = default;
  explicit DevBuf(size_t bytes, bool zero = true) : n(bytes) {
    CK(cudaMalloc(&p, bytes ? bytes : 1));
    if (zero) CK(cudaMemset(p, 0, bytes ? bytes : 1));
  }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n) { o.p = nullptr; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) {
      if (p) cudaFree(p);
      p = o.p;
      n = o.n;
      o.p = nullptr;
    }
    return *this;
  }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

// ---- model ---------------------------------------------------------------------------------------

struct Hyper {
  int L, H, Hq, Hkv, D, F, V;
  int E = 0, K = 0;  // experts per layer and experts used per token (0: dense FFN)
  float eps, theta;
  bool neox = false;
  int ctx;
  std::map<std::string, double> rope_scaling;
  std::string rope_type;
  std::vector<int32_t> eos;
};

std::string arch_of(const vmc::GgufFile& f) { return f.get_str("general.architecture", "llama"); }

Hyper read_hyper(const vmc::GgufFile& f) {
  const std::string a = arch_of(f);
  if (a != "llama" && a != "mixtral") throw std::runtime_error("vmc_run serves llama-architecture GGUFs, not " + a);
  Hyper h{};
  h.L = static_cast<int>(f.get_int("llama.block_count", 0));
  h.H = static_cast<int>(f.get_int("llama.embedding_length", 0));
  h.F = static_cast<int>(f.get_int("llama.feed_forward_length", 0));
  h.Hq = static_cast<int>(f.get_int("llama.attention.head_count", 0));
  h.Hkv = static_cast<int>(f.get_int("llama.attention.head_count_kv", h.Hq));
  h.D = static_cast<int>(f.get_int("llama.attention.key_length", h.H / h.Hq));
  h.eps = static_cast<float>(f.get_float("llama.attention.layer_norm_rms_epsilon", 1e-5));
  h.theta = static_cast<float>(f.get_float("llama.rope.freq_base", 10000.0));
  h.ctx = static_cast<int>(f.get_int("llama.context_length", 4096));
  h.E = static_cast<int>(f.get_int("llama.expert_count", 0));
  h.K = static_cast<int>(f.get_int("llama.expert_used_count", h.E > 0 ? 2 : 0));
  if (h.E > 32) throw std::runtime_error("vmc_run: at most 32 experts per layer");
  const vmc::GTensorInfo* emb = f.find_tensor("token_embd.weight");
  if (!emb) throw std::runtime_error("token_embd.weight missing");
  h.V = static_cast<int>(f.get_int("llama.vocab_size", emb->ne[1]));
  const std::string st = f.get_str("llama.rope.scaling.type", "none");
  if (st != "none") {
    h.rope_type = st;
    h.rope_scaling["factor"] = f.get_float("llama.rope.scaling.factor", 1.0);
    h.rope_scaling["original_context_length"] = static_cast<double>(f.get_int("llama.rope.scaling.original_context_length", h.ctx));
  }
  h.eos.push_back(static_cast<int32_t>(f.get_int("tokenizer.ggml.eos_token_id", 2)));
  return h;
}

// Per-pair inverse RoPE frequencies (linear and Llama-3 scaling), as vm_c_b200.config.rope_inv_freq.
std::vector<double> rope_inv_freq(const Hyper& h) {
  std::vector<double> inv(h.D / 2);
  for (int i = 0; i < h.D / 2; ++i) inv[i] = 1.0 / std::pow(static_cast<double>(h.theta), 2.0 * i / h.D);
  if (h.rope_type == "linear") {
    for (auto& f : inv) f /= h.rope_scaling.at("factor");
  } else if (h.rope_type == "llama3") {
    const double factor = h.rope_scaling.count("factor") ? h.rope_scaling.at("factor") : 8.0;
    const double lf = 1.0, hf = 4.0;
    const double old = h.rope_scaling.count("original_context_length") ? h.rope_scaling.at("original_context_length") : 8192;
    const double lw = old / lf, hw = old / hf;
    for (auto& f : inv) {
      const double wl = 2 * M_PI / f;
      if (wl < hw) continue;
      if (wl > lw) f = f / factor;
      else {
        const double s = (old / wl - lf) / (hf - lf);
        f = (1 - s) * f / factor + s * f;
      }
    }
  }
  return inv;
}

int wf_of(GType t) {
  switch (t) {
    case GType::Q4_K: return 1;
    case GType::Q6_K: return 2;
    case GType::Q8_0: return 3;
    case GType::F32:
    case GType::F16:
    case GType::BF16: return 0;
    default: return -1;
  }
}

struct Tiled {
  DevBuf buf;
  vmc::LinearDesc d;
};

class Loader {
 public:
  Loader(std::shared_ptr<vmc::GgufFile> f, cudaStream_t st) : f_(std::move(f)), st_(st) {}

  const vmc::GTensorInfo& info(const std::string& n) const {
    const vmc::GTensorInfo* t = f_->find_tensor(n);
    if (!t) throw std::runtime_error("tensor missing: " + n);
    return *t;
  }
  // Rows [r0, r1) of a tensor (GGUF bytes; one row = ne[0] elements).
  std::vector<uint8_t> rows(const std::string& n, int64_t r0, int64_t r1) const {
    const auto& t = info(n);
    const size_t rb = vmc::gtype_row_bytes(t.type, t.ne[0]);
    const uint8_t* p = f_->tensor_data(t) + r0 * rb;
    return std::vector<uint8_t>(p, p + (r1 - r0) * rb);
  }
  std::vector<float> as_f32(GType t, const std::vector<uint8_t>& raw, int64_t n) const {
    std::vector<float> out(n);
    vmc::dequantize_row(t, raw.data(), out.data(), n);
    return out;
  }
  // Tile [N, K] rows of GGUF type t (host bytes) for the GEMMs.
  Tiled tile(GType t, const std::vector<uint8_t>& raw, int N, int K) {
    int wf = wf_of(t);
    std::vector<uint8_t> src = raw;
    GType st = t;
    if (wf < 0) {  // no tiled GPU format: dequantise on the host, tile as bf16
      const auto f = as_f32(t, raw, static_cast<int64_t>(N) * K);
      src.assign(reinterpret_cast<const uint8_t*>(f.data()), reinterpret_cast<const uint8_t*>(f.data() + f.size()));
      st = GType::F32;
      wf = 0;
    }
    DevBuf s(src.size(), false);
    CK(cudaMemcpy(s.p, src.data(), src.size(), cudaMemcpyHostToDevice));
    Tiled out;
    out.buf = DevBuf(static_cast<size_t>(vmc::tiled_weight_bytes(wf, N, K)), false);
    vmc::repack_weight(wf, static_cast<int>(st), s.p, N, K, out.buf.p, st_);
    CK(cudaStreamSynchronize(st_));
    out.d.wf = wf;
    out.d.w = out.buf.p;
    out.d.N = N;
    out.d.K = K;
    return out;
  }
  // Gate / up rows [F, K] interleaved (row 2f = gate f, row 2f + 1 = up f) for the fused SwiGLU
  // epilogue; raw blocks when both share a type, else dequantised rows tiled as bf16.
  Tiled tile_gate_up(GType tg, const std::vector<uint8_t>& g, GType tu, const std::vector<uint8_t>& u, int F, int K) {
    if (tg == tu) {
      const size_t rb = vmc::gtype_row_bytes(tg, K);
      std::vector<uint8_t> inter(2 * rb * F);
      for (int r = 0; r < F; ++r) {
        memcpy(inter.data() + (2 * r) * rb, g.data() + r * rb, rb);
        memcpy(inter.data() + (2 * r + 1) * rb, u.data() + r * rb, rb);
      }
      return tile(tg, inter, 2 * F, K);
    }
    const auto gf = as_f32(tg, g, static_cast<int64_t>(F) * K), uf = as_f32(tu, u, static_cast<int64_t>(F) * K);
    std::vector<float> inter(2 * static_cast<size_t>(F) * K);
    for (int r = 0; r < F; ++r) {
      memcpy(&inter[(2 * static_cast<size_t>(r)) * K], &gf[static_cast<size_t>(r) * K], K * 4);
      memcpy(&inter[(2 * static_cast<size_t>(r) + 1) * K], &uf[static_cast<size_t>(r) * K], K * 4);
    }
    std::vector<uint8_t> raw(reinterpret_cast<uint8_t*>(inter.data()), reinterpret_cast<uint8_t*>(inter.data() + inter.size()));
    return tile(GType::F32, raw, 2 * F, K);
  }
  Tiled tile_tensor(const std::string& n) {
    const auto& t = info(n);
    return tile(t.type, rows(n, 0, t.ne[1]), static_cast<int>(t.ne[1]), static_cast<int>(t.ne[0]));
  }
  DevBuf norm(const std::string& n) {
    const auto& t = info(n);
    const auto f = as_f32(t.type, rows(n, 0, t.ne.size() > 1 ? t.ne[1] : 1), t.n_elements());
    DevBuf b(f.size() * 4, false);
    CK(cudaMemcpy(b.p, f.data(), f.size() * 4, cudaMemcpyHostToDevice));
    return b;
  }
  const vmc::GgufFile& file() const { return *f_; }

 private:
  std::shared_ptr<vmc::GgufFile> f_;
  cudaStream_t st_;
};

std::string blk(int i, const char* what) { return "blk." + std::to_string(i) + "." + what + ".weight"; }

std::vector<uint8_t> cat(std::initializer_list<const std::vector<uint8_t>*> parts) {
  std::vector<uint8_t> o;
  for (auto* p : parts) o.insert(o.end(), p->begin(), p->end());
  return o;
}

struct Model {
  Hyper h;
  std::vector<Tiled> tiles;  // owns every tiled weight
  std::vector<DevBuf> norms;
  std::vector<vmc::LayerDesc> layers;
  DevBuf embd;
  GType embd_type;
  int64_t embd_row_bytes;
  DevBuf out_norm;
  vmc::LinearDesc lm_head;
  DevBuf cos_sin;
};

// One Mixtral layer's experts (all of them on this GPU, the expert-sliced layout of one rank): the
// router [E, H] as bf16 tiles, then every expert's interleaved gate/up and its down projection tiled
// and packed back to back (one grouped GEMM per projection reads expert e at e * stride).
void load_moe(Loader& ld, Model& m, int i, vmc::LayerDesc& d) {
  const Hyper& h = m.h;
  const int E = h.E, F = h.F, H = h.H;
  d.moe = true;
  vmc::MoeDesc& md = d.m;
  const auto& tr = ld.info(blk(i, "ffn_gate_inp"));
  const auto rf = ld.as_f32(tr.type, ld.rows(blk(i, "ffn_gate_inp"), 0, E), static_cast<int64_t>(E) * H);
  const std::vector<uint8_t> rraw(reinterpret_cast<const uint8_t*>(rf.data()),
                                  reinterpret_cast<const uint8_t*>(rf.data() + rf.size()));
  m.tiles.push_back(ld.tile(GType::F32, rraw, E, H));
  md.router = m.tiles.back().d;
  const auto& tg = ld.info(blk(i, "ffn_gate_exps"));
  const auto& tu = ld.info(blk(i, "ffn_up_exps"));
  const auto& td = ld.info(blk(i, "ffn_down_exps"));
  Tiled gu_all, dn_all;
  for (int e = 0; e < E; ++e) {
    const int64_t f0 = static_cast<int64_t>(e) * F, h0 = static_cast<int64_t>(e) * H;
    Tiled gu = ld.tile_gate_up(tg.type, ld.rows(blk(i, "ffn_gate_exps"), f0, f0 + F), tu.type,
                               ld.rows(blk(i, "ffn_up_exps"), f0, f0 + F), F, H);
    Tiled dn = ld.tile(td.type, ld.rows(blk(i, "ffn_down_exps"), h0, h0 + H), H, F);
    if (e == 0) {
      gu_all.buf = DevBuf(gu.buf.n * E, false);
      gu_all.d = gu.d;
      gu_all.d.w = gu_all.buf.p;
      dn_all.buf = DevBuf(dn.buf.n * E, false);
      dn_all.d = dn.d;
      dn_all.d.w = dn_all.buf.p;
    }
    if (gu.d.wf != gu_all.d.wf || gu.buf.n * E != gu_all.buf.n || dn.d.wf != dn_all.d.wf || dn.buf.n * E != dn_all.buf.n)
      throw std::runtime_error("vmc_run: the experts of layer " + std::to_string(i) + " differ in weight type");
    CK(cudaMemcpy(gu_all.buf.as<uint8_t>() + gu.buf.n * e, gu.buf.p, gu.buf.n, cudaMemcpyDeviceToDevice));
    CK(cudaMemcpy(dn_all.buf.as<uint8_t>() + dn.buf.n * e, dn.buf.p, dn.buf.n, cudaMemcpyDeviceToDevice));
  }
  md.gate_up = gu_all.d;
  md.gate_up_stride = static_cast<int64_t>(gu_all.buf.n / E);
  md.down = dn_all.d;
  md.down_stride = static_cast<int64_t>(dn_all.buf.n / E);
  md.e0 = 0;
  md.e_local = E;
  md.f_local = F;
  m.tiles.push_back(std::move(gu_all));
  m.tiles.push_back(std::move(dn_all));
}

Model load(const std::string& path, int max_pos, cudaStream_t st) {
  auto f = vmc::GgufFile::open(path);
  Loader ld(f, st);
  Model m;
  m.h = read_hyper(*f);
  const Hyper& h = m.h;
  const int D = h.D, H = h.H;
  m.tiles.reserve(8 * h.L + 4);
  m.norms.reserve(2 * h.L + 2);
  for (int i = 0; i < h.L; ++i) {
    vmc::LayerDesc d;
    const auto& tq = ld.info(blk(i, "attn_q"));
    const auto& tk = ld.info(blk(i, "attn_k"));
    const auto& tv = ld.info(blk(i, "attn_v"));
    const auto q = ld.rows(blk(i, "attn_q"), 0, h.Hq * D), k = ld.rows(blk(i, "attn_k"), 0, h.Hkv * D),
               v = ld.rows(blk(i, "attn_v"), 0, h.Hkv * D);
    if (tq.type == tk.type && tk.type == tv.type) {
      m.tiles.push_back(ld.tile(tq.type, cat({&q, &k, &v}), (h.Hq + 2 * h.Hkv) * D, H));
      d.n_qkv = 1;
      d.qkv[0] = m.tiles.back().d;
    } else if (tq.type == tk.type) {
      m.tiles.push_back(ld.tile(tq.type, cat({&q, &k}), (h.Hq + h.Hkv) * D, H));
      d.qkv[0] = m.tiles.back().d;
      m.tiles.push_back(ld.tile(tv.type, v, h.Hkv * D, H));
      d.qkv[1] = m.tiles.back().d;
      d.qkv_col[1] = (h.Hq + h.Hkv) * D;
      d.n_qkv = 2;
    } else {
      m.tiles.push_back(ld.tile(tq.type, q, h.Hq * D, H));
      d.qkv[0] = m.tiles.back().d;
      m.tiles.push_back(ld.tile(tk.type, k, h.Hkv * D, H));
      d.qkv[1] = m.tiles.back().d;
      m.tiles.push_back(ld.tile(tv.type, v, h.Hkv * D, H));
      d.qkv[2] = m.tiles.back().d;
      d.qkv_col[1] = h.Hq * D;
      d.qkv_col[2] = (h.Hq + h.Hkv) * D;
      d.n_qkv = 3;
    }
    m.tiles.push_back(ld.tile_tensor(blk(i, "attn_output")));
    d.wo = m.tiles.back().d;
    if (h.E > 0) {
      load_moe(ld, m, i, d);
    } else {
      const auto& tg = ld.info(blk(i, "ffn_gate"));
      const auto& tu = ld.info(blk(i, "ffn_up"));
      m.tiles.push_back(ld.tile_gate_up(tg.type, ld.rows(blk(i, "ffn_gate"), 0, h.F), tu.type,
                                        ld.rows(blk(i, "ffn_up"), 0, h.F), h.F, H));
      d.gate_up = m.tiles.back().d;
      m.tiles.push_back(ld.tile_tensor(blk(i, "ffn_down")));
      d.down = m.tiles.back().d;
    }
    m.norms.push_back(ld.norm(blk(i, "attn_norm")));
    d.attn_norm = m.norms.back().as<float>();
    m.norms.push_back(ld.norm(blk(i, "ffn_norm")));
    d.ffn_norm = m.norms.back().as<float>();
    m.layers.push_back(d);
  }
  const auto& te = ld.info("token_embd.weight");
  m.embd_type = te.type;
  m.embd_row_bytes = static_cast<int64_t>(vmc::gtype_row_bytes(te.type, H));
  {
    const auto raw = ld.rows("token_embd.weight", 0, te.ne[1]);
    m.embd = DevBuf(raw.size(), false);
    CK(cudaMemcpy(m.embd.p, raw.data(), raw.size(), cudaMemcpyHostToDevice));
  }
  m.out_norm = ld.norm("output_norm.weight");
  m.tiles.push_back(f->find_tensor("output.weight") ? ld.tile_tensor("output.weight") : ld.tile_tensor("token_embd.weight"));
  m.lm_head = m.tiles.back().d;
  // RoPE table [max_pos][D/2][cos, sin], angles in double precision
  const auto inv = rope_inv_freq(h);
  std::vector<float> cs(static_cast<size_t>(max_pos) * (D / 2) * 2);
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < D / 2; ++i) {
      const double ang = static_cast<double>(p) * inv[i];
      cs[(static_cast<size_t>(p) * (D / 2) + i) * 2] = static_cast<float>(std::cos(ang));
      cs[(static_cast<size_t>(p) * (D / 2) + i) * 2 + 1] = static_cast<float>(std::sin(ang));
    }
  m.cos_sin = DevBuf(cs.size() * 4, false);
  CK(cudaMemcpy(m.cos_sin.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  return m;
}

// Split-KV factor of decode attention (vm_c_b200.ops.decode_splits).
int decode_splits(int ctas, int slots, int max_splits = 16) {
  const int sms = slots >= 148 ? slots / std::max(1, slots / 148) : slots;
  ctas = std::max(1, ctas);
  if (ctas >= sms) return 1;
  return std::max(1, std::min(max_splits, sms / ctas));
}

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

double p50(std::vector<double> v) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  return v[v.size() / 2];
}

struct Engine {
  Model& m;
  Args a;
  cudaStream_t st;
  int max_samples, max_tokens, max_model_len, num_blocks;
  vmc::BatchLayout layout;
  std::unique_ptr<vmc::Forward> fwd;
  std::vector<int> buckets;
  std::map<int, cudaGraphExec_t> graphs;
  // buffers
  DevBuf resid, h, qkv_bf16, split_ws, q, attn, o16, act, hs, logits, part_o, part_lse, kv, meta_dev, params_dev,
      tok_dev, lp_dev, err;
  // MoE (expert-sliced, all experts on this GPU): router logits, routing tables, gathered rows, expert
  // activations and outputs, combined output
  DevBuf moe_logits, moe_topk_id, moe_topk_w, moe_counts, moe_offsets, moe_sorted, moe_slot_row, moe_total, moe_xs,
      moe_act, moe_y, moe_out;
  int32_t* meta_host = nullptr;
  vmc::SampleParams* params_host = nullptr;
  int32_t* tok_host = nullptr;
  int decode_slots = 148;

  Engine(Model& model, const Args& args, cudaStream_t s) : m(model), a(args), st(s) {
    const Hyper& hp = m.h;
    max_samples = a.max_seqs;
    max_tokens = std::max(a.max_batched, max_samples);
    max_model_len = a.max_model_len > 0 ? a.max_model_len : hp.ctx;
    for (int b : {1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256})
      if (b <= a.max_seqs) buckets.push_back(b);
    if (a.graphs && !buckets.empty() && buckets.back() < a.max_seqs) buckets.push_back(a.max_seqs);
    const int max_graph = a.graphs && !buckets.empty() ? buckets.back() : 0;
    const int max_blocks = (max_model_len + 15) / 16 + 1;
    layout = vmc::BatchLayout{std::max({a.max_batched, a.max_seqs, max_graph}), std::max(a.max_seqs, max_graph), max_blocks};
    num_blocks = a.num_blocks > 0 ? a.num_blocks : 2 * a.max_seqs * max_blocks + 1;
    const int H = hp.H, D = hp.D, qkv_n = (hp.Hq + 2 * hp.Hkv) * D;
    const int T = max_tokens, S = max_samples;
    resid = DevBuf(static_cast<size_t>(T) * H * 4);
    h = DevBuf(static_cast<size_t>(T) * H * 2);
    qkv_bf16 = DevBuf(static_cast<size_t>(T) * qkv_n * 2);
    const int64_t ws_elems = static_cast<int64_t>(T) * std::max({qkv_n, 2 * hp.F, H});
    split_ws = DevBuf(static_cast<size_t>(ws_elems) * 4);
    q = DevBuf(static_cast<size_t>(T) * hp.Hq * D * 2);
    attn = DevBuf(static_cast<size_t>(T) * hp.Hq * D * 2);
    o16 = DevBuf(static_cast<size_t>(T) * H * 2);
    act = DevBuf(static_cast<size_t>(T) * hp.F * 2);
    hs = DevBuf(static_cast<size_t>(S) * H * 2);
    logits = DevBuf(static_cast<size_t>(S) * hp.V * 4);
    part_o = DevBuf(static_cast<size_t>(16) * S * hp.Hq * D * 4);
    part_lse = DevBuf(static_cast<size_t>(16) * S * hp.Hq * 4);
    const int64_t kv_layer = static_cast<int64_t>(num_blocks) * 2 * hp.Hkv * 16 * D * 2;
    kv = DevBuf(static_cast<size_t>(kv_layer) * hp.L);
    meta_dev = DevBuf(static_cast<size_t>(layout.total()) * 4);
    params_dev = DevBuf(static_cast<size_t>(max_tokens) * sizeof(vmc::SampleParams));
    tok_dev = DevBuf(static_cast<size_t>(max_tokens) * 4);
    lp_dev = DevBuf(static_cast<size_t>(max_tokens) * 4);
    err = DevBuf(16);
    CK(cudaMallocHost(&meta_host, static_cast<size_t>(layout.total()) * 4));
    CK(cudaMallocHost(&params_host, static_cast<size_t>(max_tokens) * sizeof(vmc::SampleParams)));
    CK(cudaMallocHost(&tok_host, static_cast<size_t>(max_tokens) * 4));
    memset(params_host, 0, static_cast<size_t>(max_tokens) * sizeof(vmc::SampleParams));
    vmc::gemm_prepare();
    int dev = 0, sms = 148;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    decode_slots = sms * std::max(1, vmc::attn_decode_ctas_per_sm(D));

    vmc::ForwardConfig c;
    c.L = hp.L;
    c.H = H;
    c.Hq = hp.Hq;
    c.Hkv = hp.Hkv;
    c.D = D;
    c.F = hp.F;
    c.V_local = hp.V;
    c.max_tokens = T;
    c.max_samples = S;
    c.max_blocks = max_blocks;
    c.eps = hp.eps;
    c.scale = 1.f / std::sqrt(static_cast<float>(D));
    c.neox = hp.neox;
    c.embd = m.embd.p;
    c.embd_type = static_cast<int>(m.embd_type);
    c.embd_row_bytes = m.embd_row_bytes;
    c.out_norm = m.out_norm.as<float>();
    c.lm_head = m.lm_head;
    c.cos_sin = m.cos_sin.as<float>();
    c.num_sms = 148;  // the split policy of the Python path (ops.NUM_SMS)
    vmc::ForwardBuffers b;
    b.resid = resid.as<float>();
    b.h = h.p;
    b.qkv_bf16 = qkv_bf16.p;
    b.split_ws = split_ws.as<float>();
    b.split_ws_elems = ws_elems;
    b.q = q.p;
    b.attn = attn.p;
    b.o16 = o16.p;
    b.act = act.p;
    b.hs = hs.p;
    b.logits = logits.as<float>();
    b.part_o = part_o.as<float>();
    b.part_lse = part_lse.as<float>();
    b.attn_max_splits = 16;
    int32_t* md = meta_dev.as<int32_t>();
    b.ids = md + layout.off_input_ids();
    b.pos = md + layout.off_positions();
    b.slots = md + layout.off_slot_mapping();
    b.q_start = md + layout.off_q_start();
    b.ctx_len = md + layout.off_ctx_len();
    b.block_tables = md + layout.off_block_tables();
    b.logits_idx = md + layout.off_logits_idx();
    b.params = params_dev.p;
    b.out_tok = tok_dev.as<int32_t>();
    b.out_lp = lp_dev.as<float>();
    b.kv = kv.p;
    b.kv_layer_bytes = kv_layer;
    b.err = err.as<uint32_t>();
    fwd = std::make_unique<vmc::Forward>(c, m.layers, b);
    if (hp.E > 0) {
      const size_t R = static_cast<size_t>(T) * hp.K;
      moe_logits = DevBuf(static_cast<size_t>(T) * hp.E * 4);
      moe_topk_id = DevBuf(R * 4);
      moe_topk_w = DevBuf(R * 4);
      moe_counts = DevBuf(static_cast<size_t>(hp.E) * 4);
      moe_offsets = DevBuf(static_cast<size_t>(hp.E) * 4);
      moe_sorted = DevBuf(R * 4);
      moe_slot_row = DevBuf(R * 4);
      moe_total = DevBuf(4);
      moe_xs = DevBuf(R * H * 2);
      moe_act = DevBuf(R * hp.F * 2);
      moe_y = DevBuf(R * H * 4);
      moe_out = DevBuf(static_cast<size_t>(T) * H * 4);
      vmc::MoeBuffers mb;
      mb.E = hp.E;
      mb.k = hp.K;
      mb.norm_topk = 1;  // Mixtral renormalises the selected weights
      mb.ep = false;
      mb.logits = moe_logits.as<float>();
      mb.topk_id = moe_topk_id.as<int32_t>();
      mb.topk_w = moe_topk_w.as<float>();
      mb.counts = moe_counts.as<int32_t>();
      mb.offsets = moe_offsets.as<int32_t>();
      mb.sorted_src = moe_sorted.as<int32_t>();
      mb.slot_row = moe_slot_row.as<int32_t>();
      mb.total = moe_total.as<int32_t>();
      mb.xs = moe_xs.p;
      mb.act = moe_act.p;
      mb.y = moe_y.as<float>();
      mb.out = moe_out.as<float>();
      fwd->set_moe(mb);
    }
  }

  ~Engine() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.second);
    cudaFreeHost(meta_host);
    cudaFreeHost(params_host);
    cudaFreeHost(tok_host);
  }

  int bucket(int R) const {
    for (int b : buckets)
      if (b >= R) return b;
    return 0;
  }

  vmc::StepDims dims(int T, int R, int S, int nd, int max_qlen) const {
    vmc::StepDims d;
    d.T = T;
    d.R = R;
    d.S = S;
    d.nd = nd;
    d.max_qlen = max_qlen;
    d.decode_qlen = 1;
    d.attn_splits = decode_splits(nd * m.h.Hkv, decode_slots);
    return d;
  }

  // Decode graphs: metadata of B padding rows (no KV writes), two eager runs, then capture.
  void capture_all() {
    if (!a.graphs) return;
    for (int B : buckets) {
      std::vector<int32_t> hm(layout.total(), 0);
      for (int i = 0; i < B; ++i) {
        hm[layout.off_slot_mapping() + i] = -1;
        hm[layout.off_logits_idx() + i] = i;
      }
      for (int i = 0; i <= B; ++i) hm[layout.off_q_start() + i] = i;
      CK(cudaMemcpyAsync(meta_dev.p, hm.data(), hm.size() * 4, cudaMemcpyHostToDevice, st));
      CK(cudaMemsetAsync(params_dev.p, 0, params_dev.n, st));
      const vmc::StepDims d = dims(B, B, B, B, 1);
      for (int w = 0; w < 2; ++w) fwd->run(d, st);
      CK(cudaStreamSynchronize(st));
      cudaGraph_t g;
      CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      fwd->run(d, st);
      CK(cudaStreamEndCapture(st, &g));
      cudaGraphExec_t ge;
      CK(cudaGraphInstantiate(&ge, g, 0));
      CK(cudaGraphDestroy(g));
      graphs[B] = ge;
    }
    CK(cudaStreamSynchronize(st));
  }

  struct Result {
    std::vector<std::vector<int32_t>> tokens;
    std::vector<double> ttft, itl;
  };

  Result serve(const std::vector<std::vector<int32_t>>& prompts, int64_t id0) {
    vmc::SchedulerConfig sc;
    sc.max_num_seqs = a.max_seqs;
    sc.max_num_batched_tokens = a.max_batched;
    sc.max_model_len = max_model_len;
    auto bm = std::make_shared<vmc::BlockManager>(num_blocks, 16, true);
    vmc::Scheduler sched(sc, bm);
    vmc::SeqParams sp;
    sp.max_tokens = a.gen;
    sp.ignore_eos = true;
    sp.eos_token_ids = m.h.eos;
    for (size_t i = 0; i < prompts.size(); ++i) sched.add_request(id0 + static_cast<int64_t>(i), prompts[i], sp);
    Result r;
    r.tokens.resize(prompts.size());
    std::vector<double> last(prompts.size(), -1);
    const double t0 = now_ms();
    while (sched.has_unfinished()) {
      vmc::Plan plan = sched.schedule();
      if (plan.entries.empty()) continue;
      const bool all_decode = plan.num_decode == static_cast<int>(plan.entries.size());
      const int pad = (all_decode && a.graphs) ? bucket(static_cast<int>(plan.entries.size())) : 0;
      sched.build_batch(plan, layout, meta_host, pad);
      const int32_t* cnt = meta_host + layout.off_counts();
      const int T = cnt[0], R = cnt[1], S = cnt[2], nd = cnt[3], mq = cnt[4], R_pad = pad ? cnt[7] : 0;
      // greedy rows: the zeroed records (temperature 0) are the parameters of every row
      CK(cudaMemcpyAsync(meta_dev.p, meta_host, static_cast<size_t>(layout.total()) * 4, cudaMemcpyHostToDevice, st));
      if (R_pad > 0 && graphs.count(R_pad)) {
        CK(cudaGraphLaunch(graphs[R_pad], st));
      } else {
        fwd->run(dims(T, R, S, nd, mq), st);
      }
      CK(cudaMemcpyAsync(tok_host, tok_dev.p, static_cast<size_t>(S) * 4, cudaMemcpyDeviceToHost, st));
      CK(cudaStreamSynchronize(st));
      std::vector<std::vector<int32_t>> toks;
      for (int k = 0; k < S; ++k) toks.push_back({tok_host[k]});
      const double t = now_ms() - t0;
      for (const auto& ev : sched.update(plan, toks)) {
        const size_t i = static_cast<size_t>(ev.id - id0);
        for (int32_t tk : ev.tokens) r.tokens[i].push_back(tk);
        if (last[i] < 0) r.ttft.push_back(t);
        else r.itl.push_back(t - last[i]);
        last[i] = t;
        if (ev.finished) sched.release(ev.id);
      }
    }
    return r;
  }
};

// The engine as the serving loop's step backend: metadata and per-row sampling parameters are
// staged in pinned memory and copied in on the engine's stream; decode-only steps padded to a graph
// bucket replay that bucket's graph; rows with penalties stop the forward after the lm_head logits,
// apply the penalties and sample with the same kernels the Python engine uses.
class GpuBackend : public vmc::StepBackend {
 public:
  explicit GpuBackend(Engine& e) : eng_(e) {
    CK(cudaGetDevice(&dev_));
    CK(cudaMallocHost(&lp_host_, static_cast<size_t>(eng_.max_tokens) * 4));
    CK(cudaMallocHost(&err_host_, 4));
  }
  ~GpuBackend() override {
    cudaFreeHost(lp_host_);
    cudaFreeHost(err_host_);
    if (pen_host_) cudaFreeHost(pen_host_);
  }
  vmc::BatchLayout layout() const override { return eng_.layout; }
  int vocab() const override { return eng_.m.h.V; }
  int graph_bucket(int n) const override { return eng_.a.graphs ? eng_.bucket(n) : 0; }

  void step(const int32_t* meta, const vmc::SampleParams* params, int S, const vmc::Penalties& pen, int32_t* tokens,
            float* logprobs) override {
    CK(cudaSetDevice(dev_));
    cudaStream_t st = eng_.st;
    const size_t nmeta = static_cast<size_t>(eng_.layout.total());
    memcpy(eng_.meta_host, meta, nmeta * 4);
    const int32_t* cnt = eng_.meta_host + eng_.layout.off_counts();
    const int T = cnt[0], R = cnt[1], nd = cnt[3], mq = cnt[4], Rp = cnt[7];
    // the serving loop padded a decode-only, penalty-free step to graph_bucket(R): replay that graph
    // (its padding rows sample too)
    const bool use_graph = pen.empty() && eng_.a.graphs && nd == R && Rp == eng_.bucket(R) && eng_.graphs.count(Rp);
    const int rows = use_graph ? std::max(S, Rp) : S;
    if (rows > eng_.max_tokens) throw std::runtime_error("serve: more sample rows than the parameter buffer holds");
    if (S > 0) memcpy(eng_.params_host, params, static_cast<size_t>(S) * sizeof(vmc::SampleParams));
    if (rows > S) memset(eng_.params_host + S, 0, static_cast<size_t>(rows - S) * sizeof(vmc::SampleParams));
    CK(cudaMemcpyAsync(eng_.meta_dev.p, eng_.meta_host, nmeta * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(eng_.params_dev.p, eng_.params_host, static_cast<size_t>(rows) * sizeof(vmc::SampleParams),
                       cudaMemcpyHostToDevice, st));
    if (use_graph) {
      CK(cudaGraphLaunch(eng_.graphs[Rp], st));
    } else if (pen.empty()) {
      eng_.fwd->run(eng_.dims(T, R, S, nd, mq), st);
    } else {
      vmc::StepDims d = eng_.dims(T, R, S, nd, mq);
      d.sample = false;
      eng_.fwd->run(d, st);
      const size_t n = pen.row.size();
      stage_penalties(pen, st);
      const int32_t* base = pen_dev_.as<int32_t>();
      vmc::apply_penalties(eng_.logits.as<float>(), eng_.m.h.V, base, base + n, base + 2 * n,
                           eng_.params_dev.as<vmc::SampleParams>(), static_cast<int>(n), st);
      vmc::sample(eng_.logits.as<float>(), S, eng_.m.h.V, eng_.m.h.V, eng_.params_dev.as<vmc::SampleParams>(),
                  eng_.tok_dev.as<int32_t>(), eng_.lp_dev.as<float>(), st);
    }
    CK(cudaGetLastError());
    if (S > 0) {
      CK(cudaMemcpyAsync(eng_.tok_host, eng_.tok_dev.p, static_cast<size_t>(S) * 4, cudaMemcpyDeviceToHost, st));
      CK(cudaMemcpyAsync(lp_host_, eng_.lp_dev.p, static_cast<size_t>(S) * 4, cudaMemcpyDeviceToHost, st));
    }
    CK(cudaMemcpyAsync(err_host_, eng_.err.p, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (*err_host_ != 0) throw std::runtime_error("device error word " + std::to_string(*err_host_));
    memcpy(tokens, eng_.tok_host, static_cast<size_t>(S) * 4);
    memcpy(logprobs, lp_host_, static_cast<size_t>(S) * 4);
  }

 private:
  // (row, token, count) arrays back to back in one pinned staging buffer and one device buffer
  void stage_penalties(const vmc::Penalties& pen, cudaStream_t st) {
    const size_t n = pen.row.size(), bytes = 3 * n * 4;
    if (bytes > pen_cap_) {
      CK(cudaStreamSynchronize(st));
      if (pen_host_) cudaFreeHost(pen_host_);
      pen_cap_ = std::max(bytes, 2 * pen_cap_);
      CK(cudaMallocHost(&pen_host_, pen_cap_));
      pen_dev_ = DevBuf(pen_cap_, false);
    }
    memcpy(pen_host_, pen.row.data(), n * 4);
    memcpy(pen_host_ + n, pen.token.data(), n * 4);
    memcpy(pen_host_ + 2 * n, pen.count.data(), n * 4);
    CK(cudaMemcpyAsync(pen_dev_.p, pen_host_, bytes, cudaMemcpyHostToDevice, st));
  }

  Engine& eng_;
  int dev_ = 0;
  float* lp_host_ = nullptr;
  uint32_t* err_host_ = nullptr;
  int32_t* pen_host_ = nullptr;
  size_t pen_cap_ = 0;
  DevBuf pen_dev_;
};


int serve(const Args& a) {
  vmc::StopSignals stop;  // before the CUDA runtime starts its threads, so that they inherit the mask
  cudaStream_t st;
  CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  auto gguf = vmc::GgufFile::open(a.model);
  auto tok = vmc::TextTokenizer::from_gguf(*gguf);
  Args args = a;
  if (args.max_model_len <= 0) args.max_model_len = 4096;
  if (args.num_blocks <= 0) args.num_blocks = args.max_seqs * ((args.max_model_len + 15) / 16) + 64;
  Model model = load(a.model, args.max_model_len + 1, st);
  Engine eng(model, args, st);
  eng.capture_all();
  GpuBackend be(eng);
  vmc::ServeConfig sc;
  sc.sched.max_num_seqs = args.max_seqs;
  sc.sched.max_num_batched_tokens = args.max_batched;
  sc.sched.max_model_len = args.max_model_len;
  sc.num_blocks = args.num_blocks;
  sc.eos_token_ids = tok->eos_ids();  // eos and end-of-turn, as the Python engine
  vmc::ServeLoop loop(sc, be);
  vmc::OpenAIConfig oc;
  oc.model_name = a.model_name.empty() ? gguf->get_str("general.name", "vm_c") : a.model_name;
  vmc::OpenAIServer api(loop, *tok, oc);
  vmc::http::Server srv;
  api.install(srv);
  const int bound = srv.listen(a.host, a.port);
  fprintf(stderr, "vmc_run: serving %s on %s:%d (chat template: %s)\n", oc.model_name.c_str(), a.host.c_str(), bound,
          api.chat_template().has_template() ? "jinja" : ("ChatML " + api.chat_template().parse_error()).c_str());
  if (!a.port_file.empty()) {
    FILE* f = fopen(a.port_file.c_str(), "w");
    if (!f) throw std::runtime_error("cannot write " + a.port_file);
    fprintf(f, "%d\n", bound);
    fclose(f);
  }
  srv.start();
  std::atomic<bool> done{false};
  std::thread watcher([&] {
    while (!done.load())
      if (stop.wait(100)) {
        loop.request_stop();
        return;
      }
  });
  loop.run();  // the engine's thread: every CUDA call of the server happens here
  done.store(true);
  watcher.join();
  srv.stop();
  CK(cudaStreamSynchronize(st));
  return loop.failed() ? 2 : 0;
}

std::vector<std::vector<int32_t>> read_prompts(const std::string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot open " + path);
  int32_t n = 0, len = 0;
  if (fread(&n, 4, 1, f) != 1 || fread(&len, 4, 1, f) != 1) throw std::runtime_error("bad prompt file");
  std::vector<std::vector<int32_t>> p(n, std::vector<int32_t>(len));
  for (auto& r : p)
    if (fread(r.data(), 4, len, f) != static_cast<size_t>(len)) throw std::runtime_error("short prompt file");
  fclose(f);
  return p;
}

int run(const Args& a) {
  cudaStream_t st;
  CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  const auto prompts = read_prompts(a.prompts);
  Args args = a;
  const int need = static_cast<int>(prompts[0].size()) + a.gen + 16;
  if (args.max_model_len <= 0) args.max_model_len = std::max(2048, need);  // as bench.py
  if (args.num_blocks <= 0) args.num_blocks = args.max_seqs * ((need + 15) / 16) + 64;
  Model model = load(a.model, args.max_model_len + 1, st);
  Engine eng(model, args, st);
  eng.capture_all();
  for (int w = 0; w < a.warmup; ++w) eng.serve(prompts, 1000000 * (w + 1));
  CK(cudaStreamSynchronize(st));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, st));
  Engine::Result r;
  std::vector<double> ttft, itl;
  for (int k = 0; k < a.runs; ++k) {
    r = eng.serve(prompts, 100000000LL * (k + 1));
    ttft.insert(ttft.end(), r.ttft.begin(), r.ttft.end());
    itl.insert(itl.end(), r.itl.begin(), r.itl.end());
  }
  CK(cudaEventRecord(e1, st));
  CK(cudaEventSynchronize(e1));
  float ms = 0;
  CK(cudaEventElapsedTime(&ms, e0, e1));
  uint32_t err = 0;
  CK(cudaMemcpy(&err, eng.err.p, 4, cudaMemcpyDeviceToHost));
  const double toks = static_cast<double>(a.runs) * prompts.size() * a.gen;
  printf("{\"ms_total\": %.3f, \"runs\": %d, \"tok_per_s\": %.2f, \"p50_ttft_ms\": %.3f, \"p50_itl_ms\": %.4f, "
         "\"n_req\": %zu, \"gen_len\": %d, \"device_error\": %u}\n",
         ms, a.runs, toks / (ms / 1e3), p50(ttft), p50(itl), prompts.size(), a.gen, err);
  fflush(stdout);
  if (!a.dump.empty()) {
    FILE* f = fopen(a.dump.c_str(), "w");
    fprintf(f, "[");
    for (size_t i = 0; i < r.tokens.size(); ++i) {
      fprintf(f, "%s[", i ? ", " : "");
      for (size_t j = 0; j < r.tokens[i].size(); ++j) fprintf(f, "%s%d", j ? ", " : "", r.tokens[i][j]);
      fprintf(f, "]");
    }
    fprintf(f, "]\n");
    fclose(f);
  }
  CK(cudaStreamDestroy(st));
  return err == 0 ? 0 : 2;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    const Args a = parse(argc, argv);
    return a.serve ? serve(a) : run(a);
  } catch (const std::exception& e) {
    fprintf(stderr, "vmc_run: %s\n", e.what());
    return 1;
  }
}
