// ThreadSanitizer stress driver of the native host library (scheduler, block manager, quant codecs,
// BPE core). Built with -fsanitize=thread by vm_c_b200/_build.py build_tsan() and run by
// tests/test_tsan_host.py; exit status 0 means no check failed, and with TSAN_OPTIONS
// "halt_on_error=1 exitcode=66" any data race ThreadSanitizer sees ends the run with status 66.
//
// The reference runs its scheduler from several threads with known races (HTTP handlers abort
// requests while the engine thread schedules; unlocked reads of its pending queue). This library's
// contract is the opposite: one owner thread per engine touches the Scheduler and its BlockManager,
// and other threads hand it commands through a mutex-protected queue (vm_c_b200/core/engine.py
// add_request / abort_request / _drain). The driver exercises every place where host code of this
// library meets more than one thread:
//   1. the serving contract: producer threads submit add and abort commands while one owner thread
//      drains them and runs schedule / build_batch / update / release with synthetic tokens (chunked
//      prefill, prefix caching, preemption under a small KV pool);
//   2. independent schedulers on several threads at once, each run compared with a single-threaded
//      run of the same workload (hidden shared mutable state would make them differ or race);
//   3. the multi-threaded quantise / dequantise helpers while other threads run the row codecs;
//   4. one BPE tokenizer shared read-only by several encoding threads.
#include <atomic>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "block_manager.hpp"
#include "quants.hpp"
#include "scheduler.hpp"
#include "tokenizer.hpp"

namespace {

int g_failures = 0;
std::mutex g_fail_mu;

void check(bool ok, const char* what) {
  if (ok) return;
  std::lock_guard<std::mutex> g(g_fail_mu);
  ++g_failures;
  std::fprintf(stderr, "CHECK FAILED: %s\n", what);
}

// ---- 1. serving contract -------------------------------------------------------------------------

struct Command {
  bool abort;
  int64_t id;
  std::vector<int32_t> prompt;
  int max_tokens;
};

class CommandQueue {  // what engine.py's _pending / _aborts deques under _lock are
 public:
  void push(Command c) {
    {
      std::lock_guard<std::mutex> g(mu_);
      q_.push_back(std::move(c));
    }
    cv_.notify_one();
  }
  std::deque<Command> drain(bool wait) {
    std::unique_lock<std::mutex> g(mu_);
    if (wait) cv_.wait_for(g, std::chrono::milliseconds(1), [&] { return !q_.empty(); });
    std::deque<Command> out;
    out.swap(q_);
    return out;
  }

 private:
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Command> q_;
};

// Runs the owner loop until every submitted request has finished; returns the tokens emitted.
int64_t serve(vmc::Scheduler& sched, CommandQueue& q, const std::atomic<bool>& producers_done,
              std::vector<int>* finished_len, int64_t* aborted) {
  vmc::BatchLayout layout{256, 32, 64};
  std::vector<int32_t> meta(static_cast<size_t>(layout.total()));
  int64_t emitted = 0;
  std::mt19937 rng(7);
  while (true) {
    const bool done = producers_done.load(std::memory_order_acquire);
    for (Command& c : q.drain(!sched.has_unfinished())) {
      if (c.abort) {
        if (sched.abort_request(c.id)) {
          ++*aborted;
          sched.release(c.id);
        }
        continue;
      }
      vmc::SeqParams sp;
      sp.max_tokens = c.max_tokens;
      sp.ignore_eos = true;
      sched.add_request(c.id, std::move(c.prompt), sp);
    }
    if (!sched.has_unfinished()) {
      if (done) {
        // a command pushed between the drain above and the flag read is still queued
        auto rest = q.drain(false);
        if (rest.empty()) break;
        for (Command& c : rest) q.push(std::move(c));
      }
      continue;
    }
    vmc::Plan plan = sched.schedule();
    if (plan.entries.empty()) continue;
    sched.build_batch(plan, layout, meta.data());
    std::vector<std::vector<int32_t>> toks;
    for (const auto& e : plan.entries)
      if (e.sample) toks.push_back({static_cast<int32_t>(rng() % 32000)});
    for (const auto& ev : sched.update(plan, toks)) {
      emitted += static_cast<int64_t>(ev.tokens.size());
      if (ev.finished) {
        if (finished_len) finished_len->push_back(static_cast<int>(sched.find(ev.id)->output.size()));
        sched.release(ev.id);
      }
    }
  }
  return emitted;
}

void serving_contract() {
  vmc::SchedulerConfig cfg;
  cfg.max_num_seqs = 32;
  cfg.max_num_batched_tokens = 256;
  cfg.max_model_len = 1024;
  auto kv = std::make_shared<vmc::BlockManager>(160, 16, true);  // small pool: preemption happens
  vmc::Scheduler sched(cfg, kv);
  CommandQueue q;
  std::atomic<bool> done{false};
  std::atomic<int64_t> next_id{1};
  constexpr int kProducers = 4, kPerProducer = 60;
  std::vector<int> finished_len;
  int64_t aborted = 0;
  std::thread owner([&] { serve(sched, q, done, &finished_len, &aborted); });
  std::vector<std::thread> prod;
  for (int p = 0; p < kProducers; ++p) {
    prod.emplace_back([&, p] {
      std::mt19937 rng(100 + p);
      std::vector<int32_t> shared_prefix(48);
      for (auto& t : shared_prefix) t = static_cast<int32_t>(rng() % 32000);
      for (int i = 0; i < kPerProducer; ++i) {
        Command c{false, next_id.fetch_add(1), {}, 4 + static_cast<int>(rng() % 24)};
        if (rng() % 2) c.prompt = shared_prefix;  // prefix-cache hits across requests
        const int extra = 1 + static_cast<int>(rng() % 120);
        for (int k = 0; k < extra; ++k) c.prompt.push_back(static_cast<int32_t>(rng() % 32000));
        const int64_t id = c.id;
        q.push(std::move(c));
        if (rng() % 5 == 0) q.push(Command{true, id, {}, 0});  // abort some of them again
        if (rng() % 8 == 0) std::this_thread::sleep_for(std::chrono::microseconds(200));
      }
    });
  }
  for (auto& t : prod) t.join();
  done.store(true, std::memory_order_release);
  owner.join();
  check(!sched.has_unfinished(), "serving: every request finished or was aborted");
  check(static_cast<int64_t>(finished_len.size()) + aborted == kProducers * kPerProducer,
        "serving: finished + aborted == submitted");
  check(kv->usage() == 0.0, "serving: every KV block returned to the pool");
  std::printf("serving contract: %zu finished, %lld aborted, prefix hits %lld of %lld queries\n",
              finished_len.size(), static_cast<long long>(aborted), static_cast<long long>(sched.prefix_hits()),
              static_cast<long long>(sched.prefix_queries()));
}

// ---- 2. independent schedulers on several threads -------------------------------------------------

struct RunResult {
  int64_t emitted = 0;
  std::vector<int> finished_len;
};

RunResult scheduler_run(int seed) {
  vmc::SchedulerConfig cfg;
  cfg.max_num_seqs = 16;
  cfg.max_num_batched_tokens = 192;
  cfg.max_model_len = 1024;
  cfg.preempt_prefill_on_latency = false;  // the latency policy reads the clock: keep runs comparable
  auto kv = std::make_shared<vmc::BlockManager>(96, 16, true);
  vmc::Scheduler sched(cfg, kv);
  CommandQueue q;
  std::mt19937 rng(seed);
  for (int i = 0; i < 48; ++i) {
    Command c{false, i + 1, {}, 3 + static_cast<int>(rng() % 20)};
    const int n = 1 + static_cast<int>(rng() % 150);
    for (int k = 0; k < n; ++k) c.prompt.push_back(static_cast<int32_t>(rng() % 32000));
    q.push(std::move(c));
  }
  std::atomic<bool> done{true};
  RunResult r;
  int64_t aborted = 0;
  r.emitted = serve(sched, q, done, &r.finished_len, &aborted);
  check(kv->usage() == 0.0, "independent schedulers: KV pool empty at the end");
  return r;
}

void independent_schedulers() {
  constexpr int kThreads = 4;
  std::vector<RunResult> expect(kThreads), got(kThreads);
  for (int t = 0; t < kThreads; ++t) expect[t] = scheduler_run(1000 + t);
  std::vector<std::thread> th;
  for (int t = 0; t < kThreads; ++t) th.emplace_back([&, t] { got[t] = scheduler_run(1000 + t); });
  for (auto& x : th) x.join();
  for (int t = 0; t < kThreads; ++t) {
    check(got[t].emitted == expect[t].emitted, "independent schedulers: same tokens as a lone run");
    check(got[t].finished_len == expect[t].finished_len, "independent schedulers: same finish order");
  }
  std::printf("independent schedulers: %d concurrent runs match their single-threaded runs\n", kThreads);
}

// ---- 3. quant codecs --------------------------------------------------------------------------------

void codec_round(vmc::GType t, int seed) {
  const int64_t rows = 96, cols = 512;
  std::mt19937 rng(seed);
  std::normal_distribution<float> nd(0.f, 0.02f);
  std::vector<float> x(static_cast<size_t>(rows * cols));
  for (auto& v : x) v = nd(rng);
  const auto tr = vmc::gtype_traits(t);
  const size_t row_bytes = static_cast<size_t>(cols / tr.block_elems * tr.block_bytes);
  std::vector<uint8_t> q1(rows * row_bytes), q4(rows * row_bytes);
  for (int64_t r = 0; r < rows; ++r) vmc::quantize_row(t, x.data() + r * cols, q1.data() + r * row_bytes, cols);
  vmc::quantize_tensor(t, x.data(), q4.data(), rows, cols, 4);
  check(q1 == q4, "codecs: threaded quantisation equals the row codec");
  std::vector<float> d1(x.size()), d4(x.size());
  for (int64_t r = 0; r < rows; ++r) vmc::dequantize_row(t, q1.data() + r * row_bytes, d1.data() + r * cols, cols);
  vmc::dequantize_tensor(t, q4.data(), d4.data(), rows, cols, 4);
  check(std::memcmp(d1.data(), d4.data(), d1.size() * sizeof(float)) == 0,
        "codecs: threaded dequantisation equals the row codec");
}

void codecs() {
  const vmc::GType types[] = {vmc::GType::Q4_K, vmc::GType::Q6_K, vmc::GType::Q8_0, vmc::GType::Q4_0};
  std::vector<std::thread> th;
  for (int t = 0; t < 4; ++t)
    th.emplace_back([&, t] {
      for (int it = 0; it < 3; ++it) codec_round(types[(t + it) % 4], 10 * t + it);
    });
  for (auto& x : th) x.join();
  std::printf("codecs: Q4_K / Q6_K / Q8_0 / Q4_0 with 4 worker threads each, on 4 threads at once\n");
}

// ---- 4. shared tokenizer -------------------------------------------------------------------------------

void tokenizer() {
  std::vector<std::string> tokens = {"<unk>", "<s>", "</s>"};
  for (int b = 0; b < 256; ++b) {
    char buf[8];
    std::snprintf(buf, sizeof(buf), "<0x%02X>", b);
    tokens.push_back(buf);
  }
  const char* pieces[] = {"\xe2\x96\x81", "a", "b", "c", "d", "e", "h", "i", "n", "g", "o", "r", "s", "t",
                          "th", "he", "in", "ng", "ing", "the", "\xe2\x96\x81t", "\xe2\x96\x81the", "er", "on",
                          "\xe2\x96\x81" "a", "st", "re", "\xe2\x96\x81s", "ti", "tion"};
  std::vector<float> scores(tokens.size(), 0.f);
  float s = -100.f;
  for (const char* p : pieces) {
    tokens.push_back(p);
    scores.push_back(s += 1.f);
  }
  vmc::BpeTokenizer tok(tokens, scores, {}, "llama");
  tok.set_unk(0);
  std::vector<std::string> texts;
  std::mt19937 rng(3);
  const char* words[] = {"\xe2\x96\x81the", "\xe2\x96\x81string", "\xe2\x96\x81station", "\xe2\x96\x81ration",
                         "\xe2\x96\x81hinge", "\xe2\x96\x81\xc3\xa9t\xc3\xa9", "\xe2\x96\x81zebra"};
  for (int i = 0; i < 200; ++i) {
    std::string t;
    const int n = 1 + static_cast<int>(rng() % 12);
    for (int k = 0; k < n; ++k) t += words[rng() % 7];
    texts.push_back(t);
  }
  std::vector<std::vector<int32_t>> expect;
  for (const auto& t : texts) expect.push_back(tok.encode_piece(t));
  std::atomic<int> mismatches{0};
  std::vector<std::thread> th;
  for (int t = 0; t < 4; ++t)
    th.emplace_back([&, t] {
      for (int rep = 0; rep < 5; ++rep)
        for (size_t i = t; i < texts.size(); ++i)
          if (tok.encode_piece(texts[i]) != expect[i]) mismatches.fetch_add(1);
    });
  for (auto& x : th) x.join();
  check(mismatches.load() == 0, "tokenizer: concurrent encodes equal sequential ones");
  std::printf("tokenizer: 4 threads x %zu texts share one BPE core\n", texts.size());
}

}  // namespace

int main() {
  serving_contract();
  independent_schedulers();
  codecs();
  tokenizer();
  if (g_failures) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failures);
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
