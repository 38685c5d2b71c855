// Reference arm driver: serves the benchmark workload through the reference's own forward-pass API
// (its vendored, vm_c-patched libllama: llama_decode on a llama_context configured as vm_c's
// LlamaRuntime configures it, src/official/llama_runtime.cpp:178-538) and its own GPU sampler
// (src/cuda/sampler_kernels.cu gpu_filtered_sampling, called as src/core/engine.cpp:1116-1154 does).
// The scheduling loop restates vm_c's decode-first continuous batching (src/core/scheduler.cpp:98-297)
// for a closed batch of requests: every running decode request gets one token per step, then prefill
// chunks fill the rest of the token budget in arrival order.
//
//   vmc_ref_bench gen   --preset llama3-8b|tiny-llama --mix Q4_K_M|Q8_0 --seed S --out FILE.gguf
//   vmc_ref_bench bench --model FILE.gguf --prompts FILE.bin [--gen 256] [--batch 2048] [--runs K]
//                       [--warmup W] [--cpu] [--dump-tokens FILE.json]
//
// `gen` writes a random-init checkpoint with the reference's own GGUF writer and quantisers (ggml's
// gguf_* and ggml_quantize_chunk): weights ~ normal(0, 0.02), norms 1, the Q4_K_M mix (Q6_K for the
// output projection and for attn_v / ffn_down in llama.cpp's use_more_bits layers). `--prompts` is a
// little-endian file: int32 count, int32 length, then count * length int32 token ids.
// `bench` prints one JSON line: device time of the timed runs (CUDA events bracketed by device
// synchronisation; every step ends in a stream synchronisation, as the reference engine's does),
// output tokens/s, p50 time-to-first-token and inter-token latency.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#ifndef VMC_REF_CPU_ONLY
#include <cuda_runtime.h>
#endif

#include "ggml.h"
#include "gguf.h"
#include "llama.h"
#ifndef VMC_REF_CPU_ONLY
#include "vm_c/cuda/kernels_sampler.h"
#endif

namespace {

struct Args {
  std::string mode, model, prompts, out, preset = "llama3-8b", mix = "Q4_K_M", dump;
  int gen = 256, batch = 2048, runs = 1, warmup = 1, seed = 0;
  bool cpu = false;
};

Args parse(int argc, char** argv) {
  Args a;
  if (argc < 2) throw std::runtime_error("usage: vmc_ref_bench gen|bench [options]");
  a.mode = argv[1];
  for (int i = 2; i < argc; ++i) {
    std::string k = argv[i];
    auto val = [&]() -> std::string {
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + k);
      return argv[++i];
    };
    if (k == "--model") a.model = val();
    else if (k == "--prompts") a.prompts = val();
    else if (k == "--out") a.out = val();
    else if (k == "--preset") a.preset = val();
    else if (k == "--mix") a.mix = val();
    else if (k == "--dump-tokens") a.dump = val();
    else if (k == "--gen") a.gen = std::stoi(val());
    else if (k == "--batch") a.batch = std::stoi(val());
    else if (k == "--runs") a.runs = std::stoi(val());
    else if (k == "--warmup") a.warmup = std::stoi(val());
    else if (k == "--seed") a.seed = std::stoi(val());
    else if (k == "--cpu") a.cpu = true;
    else throw std::runtime_error("unknown option " + k);
  }
  return a;
}

#ifndef VMC_REF_CPU_ONLY
#define CK(x)                                                                                   \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) throw std::runtime_error(std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)
#else
// CPU-only build: no CUDA runtime; the GPU branches below are compiled out.
#define CK(x) (void)0
typedef void* cudaStream_t;
typedef void* cudaEvent_t;
#endif

// ------------------------------------------------------------------------------------------------
// gen

struct Shape {
  int L, H, Hq, Hkv, D, F, V;
  float eps, theta;
  int ctx;
};

Shape preset_shape(const std::string& p) {
  if (p == "llama3-8b") return {32, 4096, 32, 8, 128, 14336, 128256, 1e-5f, 500000.f, 8192};
  if (p == "tiny-llama") return {4, 256, 8, 4, 32, 688, 32000, 1e-5f, 10000.f, 2048};
  throw std::runtime_error("unknown preset " + p);
}

bool more_bits(int i, int n) { return i < n / 8 || i >= 7 * n / 8 || (i - n / 8) % 3 == 2; }

struct TSpec {
  std::string name;
  int64_t ne0, ne1;
  ggml_type type;
  bool ones;
};

int gen(const Args& a) {
  const Shape s = preset_shape(a.preset);
  const bool km = a.mix == "Q4_K_M";
  const ggml_type base = km ? GGML_TYPE_Q4_K : (a.mix == "Q8_0" ? GGML_TYPE_Q8_0 : GGML_TYPE_F16);
  auto fit = [](ggml_type t, int64_t k) { return k % ggml_blck_size(t) == 0 ? t : GGML_TYPE_F16; };
  std::vector<TSpec> specs;
  specs.push_back({"token_embd.weight", s.H, s.V, fit(base, s.H), false});
  for (int i = 0; i < s.L; ++i) {
    const std::string b = "blk." + std::to_string(i) + ".";
    const ggml_type vt = km && more_bits(i, s.L) ? GGML_TYPE_Q6_K : base;
    specs.push_back({b + "attn_norm.weight", s.H, 1, GGML_TYPE_F32, true});
    specs.push_back({b + "attn_q.weight", s.H, (int64_t)s.Hq * s.D, fit(base, s.H), false});
    specs.push_back({b + "attn_k.weight", s.H, (int64_t)s.Hkv * s.D, fit(base, s.H), false});
    specs.push_back({b + "attn_v.weight", s.H, (int64_t)s.Hkv * s.D, fit(vt, s.H), false});
    specs.push_back({b + "attn_output.weight", (int64_t)s.Hq * s.D, s.H, fit(base, (int64_t)s.Hq * s.D), false});
    specs.push_back({b + "ffn_norm.weight", s.H, 1, GGML_TYPE_F32, true});
    specs.push_back({b + "ffn_gate.weight", s.H, s.F, fit(base, s.H), false});
    specs.push_back({b + "ffn_up.weight", s.H, s.F, fit(base, s.H), false});
    specs.push_back({b + "ffn_down.weight", s.F, s.H, fit(vt, s.F), false});
  }
  specs.push_back({"output_norm.weight", s.H, 1, GGML_TYPE_F32, true});
  specs.push_back({"output.weight", s.H, s.V, fit(km ? GGML_TYPE_Q6_K : base, s.H), false});

  gguf_context* g = gguf_init_empty();
  gguf_set_val_str(g, "general.architecture", "llama");
  gguf_set_val_str(g, "general.name", ("random-init " + a.preset).c_str());
  gguf_set_val_u32(g, "llama.block_count", s.L);
  gguf_set_val_u32(g, "llama.embedding_length", s.H);
  gguf_set_val_u32(g, "llama.feed_forward_length", s.F);
  gguf_set_val_u32(g, "llama.attention.head_count", s.Hq);
  gguf_set_val_u32(g, "llama.attention.head_count_kv", s.Hkv);
  gguf_set_val_u32(g, "llama.attention.key_length", s.D);
  gguf_set_val_u32(g, "llama.attention.value_length", s.D);
  gguf_set_val_f32(g, "llama.attention.layer_norm_rms_epsilon", s.eps);
  gguf_set_val_f32(g, "llama.rope.freq_base", s.theta);
  gguf_set_val_u32(g, "llama.rope.dimension_count", s.D);
  gguf_set_val_u32(g, "llama.context_length", s.ctx);
  gguf_set_val_u32(g, "llama.vocab_size", s.V);
  gguf_set_val_u32(g, "llama.full_attention_interval", 1);
  gguf_set_val_str(g, "tokenizer.ggml.model", "none");  // token ids in, token ids out

  ggml_init_params ip = {specs.size() * ggml_tensor_overhead() + 1024, nullptr, true};
  ggml_context* mc = ggml_init(ip);
  for (auto& t : specs) {
    ggml_tensor* x = t.ne1 == 1 ? ggml_new_tensor_1d(mc, t.type, t.ne0) : ggml_new_tensor_2d(mc, t.type, t.ne0, t.ne1);
    ggml_set_name(x, t.name.c_str());
    gguf_add_tensor(g, x);
  }
  FILE* f = fopen(a.out.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot open " + a.out);
  std::vector<uint8_t> meta(gguf_get_meta_size(g));
  gguf_get_meta_data(g, meta.data());
  fwrite(meta.data(), 1, meta.size(), f);
  // The data section starts right after the metadata block (gguf_get_meta_size includes the padding
  // to the alignment); gguf_get_data_offset is only set for a context read from a file.
  const size_t align = gguf_get_alignment(g);
  const size_t data0 = (meta.size() + align - 1) / align * align;
  const int nthr = std::max(1u, std::thread::hardware_concurrency());
  for (size_t ti = 0; ti < specs.size(); ++ti) {
    const TSpec& t = specs[ti];
    const int64_t rows = t.ne1;
    const size_t rb = ggml_row_size(t.type, t.ne0);
    std::vector<uint8_t> out(rb * rows);
    // Rows are split over threads; each thread's normal stream is seeded by (seed, tensor, thread).
    std::vector<std::thread> th;
    const int64_t per = (rows + nthr - 1) / nthr;
    for (int k = 0; k < nthr; ++k) {
      th.emplace_back([&, k]() {
        const int64_t r0 = k * per, r1 = std::min(rows, r0 + per);
        if (r0 >= r1) return;
        std::mt19937_64 rng(static_cast<uint64_t>(a.seed) * 1000003ull + ti * 4099ull + k);
        std::normal_distribution<float> nd(0.f, 0.02f);
        std::vector<float> v(static_cast<size_t>(r1 - r0) * t.ne0);
        for (auto& x : v) x = t.ones ? 1.f : nd(rng);
        if (t.type == GGML_TYPE_F32) {
          memcpy(out.data() + r0 * rb, v.data(), v.size() * 4);
        } else {
          ggml_quantize_chunk(t.type, v.data(), out.data() + r0 * rb, 0, r1 - r0, t.ne0, nullptr);
        }
      });
    }
    for (auto& x : th) x.join();
    const int64_t id = gguf_find_tensor(g, t.name.c_str());
    fseek(f, static_cast<long>(data0 + gguf_get_tensor_offset(g, id)), SEEK_SET);
    fwrite(out.data(), 1, out.size(), f);
  }
  // pad the file to the end of the last tensor's aligned slot
  fclose(f);
  gguf_free(g);
  ggml_free(mc);
  fprintf(stderr, "wrote %s (%zu tensors)\n", a.out.c_str(), specs.size());
  return 0;
}

// ------------------------------------------------------------------------------------------------
// bench

struct Req {
  std::vector<llama_token> prompt, out;
  int slot = -1;
  int computed = 0;  // prompt tokens in the KV cache
  double t_first = -1, t_last = -1;
  std::vector<double> itl;
};

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

double p50(std::vector<double> v) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  return v[v.size() / 2];
}

std::vector<std::vector<llama_token>> read_prompts(const std::string& path) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot open " + path);
  int32_t n = 0, len = 0;
  if (fread(&n, 4, 1, f) != 1 || fread(&len, 4, 1, f) != 1) throw std::runtime_error("bad prompt file");
  std::vector<std::vector<llama_token>> p(n, std::vector<llama_token>(len));
  for (auto& r : p)
    if (fread(r.data(), 4, len, f) != static_cast<size_t>(len)) throw std::runtime_error("short prompt file");
  fclose(f);
  return p;
}

struct Server {
  llama_context* ctx;
  int V, n_seq, budget, gen_len;
  bool cpu;
  cudaStream_t st = nullptr;
  float* d_logits = nullptr;
  int32_t* d_ids = nullptr;
  float *d_lp = nullptr, *d_temp = nullptr, *d_topp = nullptr, *d_minp = nullptr;
  int32_t* d_topk = nullptr;
  std::vector<int32_t> h_ids;
  std::vector<float> h_lp;
  // Host <-> device traffic of the serving loop (per run): the batch's token ids, positions and
  // sequence ids go to the device; libllama returns every output row's logits to host memory, and
  // the engine sends the sampled rows back up to its sampler and reads the sampled ids and logprobs.
  double h2d = 0, d2h = 0;

  void init() {
    h_ids.resize(n_seq);
    h_lp.resize(n_seq);
    if (cpu) return;
#ifdef VMC_REF_CPU_ONLY
    throw std::runtime_error("this build has no CUDA backend: pass --cpu");
#else
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    CK(cudaMalloc(&d_logits, static_cast<size_t>(n_seq) * V * sizeof(float)));
    CK(cudaMalloc(&d_ids, n_seq * 4));
    CK(cudaMalloc(&d_lp, n_seq * 4));
    CK(cudaMalloc(&d_temp, n_seq * 4));
    CK(cudaMalloc(&d_topk, n_seq * 4));
    CK(cudaMalloc(&d_topp, n_seq * 4));
    CK(cudaMalloc(&d_minp, n_seq * 4));
    // greedy requests: temperature 0 with the default top_k 40 / top_p 0.95 (the engine's request
    // defaults) takes the sampler's greedy branch
    std::vector<float> t0(n_seq, 0.f), tp(n_seq, 0.95f), mp(n_seq, 0.f);
    std::vector<int32_t> tk(n_seq, 40);
    CK(cudaMemcpy(d_temp, t0.data(), n_seq * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_topk, tk.data(), n_seq * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_topp, tp.data(), n_seq * 4, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_minp, mp.data(), n_seq * 4, cudaMemcpyHostToDevice));
#endif
  }

  // Greedy token of each logits row (batch indices `rows`).
  void sample(const std::vector<int>& rows) {
    const int ns = static_cast<int>(rows.size());
    if (cpu) {
      for (int i = 0; i < ns; ++i) {
        const float* l = llama_get_logits_ith(ctx, rows[i]);
        h_ids[i] = static_cast<int32_t>(std::max_element(l, l + V) - l);
      }
      return;
    }
#ifndef VMC_REF_CPU_ONLY
    for (int i = 0; i < ns; ++i) {  // engine.cpp copy_llama_logits_rows
      const float* l = llama_get_logits_ith(ctx, rows[i]);
      CK(cudaMemcpyAsync(d_logits + static_cast<size_t>(i) * V, l, static_cast<size_t>(V) * 4, cudaMemcpyDefault, st));
    }
    vm_c::gpu_filtered_sampling(d_logits, nullptr, d_ids, d_lp, d_temp, d_topk, d_topp, d_minp, ns, V,
                                vm_c::ScalarType::FLOAT32, 0, st);
    CK(cudaMemcpyAsync(h_ids.data(), d_ids, ns * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(h_lp.data(), d_lp, ns * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
#endif
  }

  // One complete serving run of `prompts`; returns the finished requests.
  std::vector<Req> run(const std::vector<std::vector<llama_token>>& prompts, double t0) {
    std::vector<Req> reqs(prompts.size());
    std::deque<int> waiting;
    for (size_t i = 0; i < prompts.size(); ++i) {
      reqs[i].prompt = prompts[i];
      waiting.push_back(static_cast<int>(i));
    }
    std::vector<int> running;
    std::vector<int> free_slots;
    for (int s = n_seq - 1; s >= 0; --s) free_slots.push_back(s);
    llama_batch batch = llama_batch_init(budget, 0, 1);
    llama_memory_t mem = llama_get_memory(ctx);
    size_t done = 0;
    while (done < reqs.size()) {
      batch.n_tokens = 0;
      std::vector<int> sample_req, sample_row;
      auto add = [&](llama_token tok, int pos, int seq, bool logits) {
        const int i = batch.n_tokens++;
        batch.token[i] = tok;
        batch.pos[i] = pos;
        batch.n_seq_id[i] = 1;
        batch.seq_id[i][0] = seq;
        batch.logits[i] = logits;
        return i;
      };
      int left = budget;
      // phase 1: one token for every running request past its prompt
      for (int r : running) {
        Req& q = reqs[r];
        if (q.computed < static_cast<int>(q.prompt.size()) || left == 0) continue;
        const int pos = static_cast<int>(q.prompt.size() + q.out.size()) - 1;
        sample_row.push_back(add(q.out.back(), pos, q.slot, true));
        sample_req.push_back(r);
        --left;
      }
      // phase 3 / 4: prefill chunks of running, then newly admitted requests
      auto prefill = [&](int r) {
        Req& q = reqs[r];
        const int n = std::min(left, static_cast<int>(q.prompt.size()) - q.computed);
        for (int j = 0; j < n; ++j) {
          const int p = q.computed + j;
          const bool last = p == static_cast<int>(q.prompt.size()) - 1;
          const int row = add(q.prompt[p], p, q.slot, last);
          if (last) {
            sample_row.push_back(row);
            sample_req.push_back(r);
          }
        }
        q.computed += n;
        left -= n;
      };
      for (int r : running)
        if (left > 0 && reqs[r].computed < static_cast<int>(reqs[r].prompt.size()) &&
            std::find(sample_req.begin(), sample_req.end(), r) == sample_req.end())
          prefill(r);
      while (left > 0 && !waiting.empty() && !free_slots.empty()) {
        const int r = waiting.front();
        waiting.pop_front();
        reqs[r].slot = free_slots.back();
        free_slots.pop_back();
        running.push_back(r);
        prefill(r);
      }
      if (batch.n_tokens == 0) throw std::runtime_error("scheduler produced an empty step");
      const int rc = llama_decode(ctx, batch);
      if (rc != 0) throw std::runtime_error("llama_decode failed: rc=" + std::to_string(rc));
      sample(sample_row);
      h2d += 12.0 * batch.n_tokens + (cpu ? 0.0 : 4.0 * V * sample_row.size());
      d2h += 4.0 * V * sample_row.size() + 8.0 * sample_row.size();
      const double t = now_ms() - t0;
      for (size_t i = 0; i < sample_req.size(); ++i) {
        Req& q = reqs[sample_req[i]];
        q.out.push_back(h_ids[i]);
        if (q.t_first < 0) q.t_first = t;
        else q.itl.push_back(t - q.t_last);
        q.t_last = t;
        if (static_cast<int>(q.out.size()) >= gen_len) {
          llama_memory_seq_rm(mem, q.slot, -1, -1);
          free_slots.push_back(q.slot);
          running.erase(std::find(running.begin(), running.end(), sample_req[i]));
          ++done;
        }
      }
    }
    llama_batch_free(batch);
    return reqs;
  }
};

int bench(const Args& a) {
  const auto prompts = read_prompts(a.prompts);
  const int n_req = static_cast<int>(prompts.size());
  const int plen = static_cast<int>(prompts[0].size());
  llama_backend_init();
  llama_model_params mp = llama_model_default_params();
  mp.n_gpu_layers = a.cpu ? 0 : -1;
  mp.split_mode = LLAMA_SPLIT_MODE_NONE;
  mp.main_gpu = a.cpu ? -1 : 0;
  mp.use_mmap = false;
  llama_model* model = llama_model_load_from_file(a.model.c_str(), mp);
  if (!model) throw std::runtime_error("llama_model_load_from_file failed");
  const int V = llama_vocab_n_tokens(llama_model_get_vocab(model));
  // Context as LlamaRuntime::load sets it (llama_runtime.cpp:383-447): n_batch = max_num_batched_tokens,
  // n_ubatch = min(512, n_batch), n_seq_max = max_num_seqs, bf16 KV, one host thread, K/Q/V offloaded.
  // Per-sequence KV capacity is n_ctx / n_seq_max, so n_ctx covers every sequence's prompt + output.
  const int per_seq = ((plen + a.gen + 16 + 255) / 256) * 256;
  llama_context_params cp = llama_context_default_params();
  cp.n_ctx = static_cast<uint32_t>(per_seq) * n_req;
  cp.n_batch = a.batch;
  cp.n_ubatch = std::min(512, a.batch);
  cp.n_seq_max = n_req;
  cp.n_threads = a.cpu ? static_cast<int>(std::thread::hardware_concurrency()) : 1;
  cp.n_threads_batch = cp.n_threads;
  cp.type_k = a.cpu ? GGML_TYPE_F32 : GGML_TYPE_BF16;
  cp.type_v = a.cpu ? GGML_TYPE_F32 : GGML_TYPE_BF16;
  cp.offload_kqv = !a.cpu;
  cp.no_perf = true;
  llama_context* ctx = llama_init_from_model(model, cp);
  if (!ctx) throw std::runtime_error("llama_init_from_model failed");
  Server s{ctx, V, n_req, a.batch, a.gen, a.cpu};
  s.init();
  llama_memory_t mem = llama_get_memory(ctx);
  for (int w = 0; w < a.warmup; ++w) {
    llama_memory_clear(mem, true);
    s.run(prompts, now_ms());
  }
#ifndef VMC_REF_CPU_ONLY
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (!a.cpu) {
    CK(cudaDeviceSynchronize());
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0, s.st));
  }
#endif
  const double w0 = now_ms();
  std::vector<double> ttft, itl;
  std::vector<Req> last;
  for (int k = 0; k < a.runs; ++k) {
    llama_memory_clear(mem, true);
    const double t0 = now_ms();
    last = s.run(prompts, t0);
    for (auto& q : last) {
      ttft.push_back(q.t_first);
      itl.insert(itl.end(), q.itl.begin(), q.itl.end());
    }
  }
  double ms = now_ms() - w0;
  const double wall_ms = ms;
#ifndef VMC_REF_CPU_ONLY
  if (!a.cpu) {
    CK(cudaDeviceSynchronize());
    CK(cudaEventRecord(e1, s.st));
    CK(cudaEventSynchronize(e1));
    float dev_ms = 0;
    CK(cudaEventElapsedTime(&dev_ms, e0, e1));
    ms = dev_ms;
  }
#endif
  const double toks = static_cast<double>(a.runs) * n_req * a.gen;
  printf("{\"ms_total\": %.3f, \"ms_wall_total\": %.3f, \"runs\": %d, \"ms_per_run\": %.3f, \"tok_per_s\": %.2f, "
         "\"p50_ttft_ms\": %.3f, \"p50_itl_ms\": %.4f, \"n_req\": %d, \"prompt_len\": %d, \"gen_len\": %d, "
         "\"vocab\": %d, \"h2d_bytes_per_run\": %.0f, \"d2h_bytes_per_run\": %.0f}\n",
         ms, wall_ms, a.runs, ms / a.runs, toks / (ms / 1e3), p50(ttft), p50(itl), n_req, plen, a.gen, V,
         s.h2d / std::max(1, a.runs + a.warmup), s.d2h / std::max(1, a.runs + a.warmup));
  fflush(stdout);
  if (!a.dump.empty()) {
    FILE* f = fopen(a.dump.c_str(), "w");
    fprintf(f, "[");
    for (size_t i = 0; i < last.size(); ++i) {
      fprintf(f, "%s[", i ? ", " : "");
      for (size_t j = 0; j < last[i].out.size(); ++j) fprintf(f, "%s%d", j ? ", " : "", last[i].out[j]);
      fprintf(f, "]");
    }
    fprintf(f, "]\n");
    fclose(f);
  }
  llama_free(ctx);
  llama_model_free(model);
  llama_backend_free();
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    const Args a = parse(argc, argv);
    if (a.mode == "gen") return gen(a);
    if (a.mode == "bench") return bench(a);
    throw std::runtime_error("unknown mode " + a.mode);
  } catch (const std::exception& e) {
    fprintf(stderr, "vmc_ref_bench: %s\n", e.what());
    return 1;
  }
}
