// The native serving loop: request intake, the continuous-batching scheduler, one step backend,
// per-request token streams and metrics.
//
// Threading: one loop thread owns the scheduler and the backend (and therefore the GPU stream);
// HTTP handler threads submit requests, aborts and stop-string finishes through a locked intake
// queue and receive tokens through their request's GenStream. This replaces the reference's design
// where HTTP threads push into the scheduler's queues directly (src/main.cpp:617,778 ->
// src/core/scheduler.cpp:451-468) with a single owner, the same structure as the Python server's
// EngineLoop (vm_c_b200/server/http.py).
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "sample_params.hpp"
#include "scheduler.hpp"

namespace vmc {

// Token-count triples (row, token, count) of the rows that use repetition / frequency / presence
// penalties: every prompt token once with count 0, every generated token with its count.
struct Penalties {
  std::vector<int32_t> row, token, count;
  bool empty() const { return row.empty(); }
};

class StepBackend {
 public:
  virtual ~StepBackend() = default;
  virtual BatchLayout layout() const = 0;
  virtual int vocab() const = 0;
  // Row count a decode-only step of `n` requests is padded to for CUDA-graph replay (0: eager).
  virtual int graph_bucket(int /*n*/) const { return 0; }
  // Runs one step. `meta` holds layout().total() int32 written by Scheduler::build_batch; `params`
  // the S sampled rows' parameters. Writes S tokens and their log-probabilities.
  virtual void step(const int32_t* meta, const SampleParams* params, int S, const Penalties& pen,
                    int32_t* tokens, float* logprobs) = 0;
};

struct GenRequest {
  std::vector<int32_t> prompt;
  int max_tokens = 16;
  int min_tokens = 0;
  bool ignore_eos = false;
  std::vector<int32_t> stop_token_ids;
  // defaults of the reference's SamplingParams (include/vm_c/core/request.hpp:28-42)
  float temperature = 0.8f;
  int top_k = 40;
  float top_p = 0.95f;
  float min_p = 0.f;
  float repetition_penalty = 1.f;
  float frequency_penalty = 0.f;
  float presence_penalty = 0.f;
  bool has_seed = false;
  uint64_t seed = 0;
  std::string name;  // caller's request id (the seed is derived from it when none is given)
  bool greedy() const { return temperature <= 0.f || top_k == 1; }
  bool has_penalties() const {
    return repetition_penalty != 1.f || frequency_penalty != 0.f || presence_penalty != 0.f;
  }
};

struct GenEvent {
  std::vector<int32_t> tokens;
  std::vector<float> logprobs;
  bool finished = false;
  FinishReason reason = FinishReason::NONE;
};

// Consumer side of one request's tokens (HTTP handler threads).
class GenStream {
 public:
  explicit GenStream(int64_t id) : id_(id) {}
  int64_t id() const { return id_; }
  // Waits up to timeout_ms for the next batch of events; false if none arrived.
  bool next(GenEvent& ev, int timeout_ms);

 private:
  friend class ServeLoop;
  void push(GenEvent ev);
  int64_t id_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<GenEvent> q_;
};

struct ServeConfig {
  SchedulerConfig sched;
  int64_t num_blocks = 0;
  int block_size = 16;
  bool prefix_caching = true;
  std::vector<int32_t> eos_token_ids;
  int idle_wait_ms = 20;
};

struct ServeStats {
  int64_t steps = 0, tokens_scheduled = 0, tokens_generated = 0, preemptions = 0, finished = 0, requests = 0;
  int64_t aborted = 0, errors = 0, prefix_queries = 0, prefix_hits = 0;
  int running = 0, waiting = 0;
  double kv_usage = 0, step_time_s = 0;
  double p50_ttft_ms = 0, p50_itl_ms = 0, p99_itl_ms = 0;
};

class ServeLoop {
 public:
  ServeLoop(const ServeConfig& cfg, StepBackend& backend);
  ~ServeLoop();

  // Thread-safe. Throws std::invalid_argument for an empty prompt or out-of-range token ids.
  std::shared_ptr<GenStream> submit(const GenRequest& r);
  void abort(int64_t id);   // the client is gone
  void finish(int64_t id);  // a stop string matched on the host

  void start();  // loop on a background thread
  void run();    // loop on the calling thread until request_stop() / stop()
  void request_stop() { stop_.store(true); }  // async-signal-safe; the loop notices within idle_wait_ms
  void stop();
  // Steps on the calling thread until no request is left (tests, offline use); throws if the
  // scheduler cannot place the remaining requests.
  void run_until_idle();

  ServeStats stats() const;
  bool failed() const { return failed_.load(); }
  std::string last_error() const;

 private:
  struct Live {
    GenRequest req;
    std::shared_ptr<GenStream> stream;
    uint64_t seed = 0;
    int generated = 0;
    std::map<int32_t, int32_t> out_counts;  // penalised rows only
    double arrival = 0, last = -1;
  };
  void loop();
  bool step_once();  // false when nothing ran (idle, or no request fits this step)
  void drain();
  void close(int64_t id, FinishReason reason);
  void publish();  // scheduler counters -> st_ (the loop thread owns the scheduler)

  ServeConfig cfg_;
  StepBackend& be_;
  BatchLayout layout_;
  std::shared_ptr<BlockManager> kv_;
  std::unique_ptr<Scheduler> sched_;
  std::vector<int32_t> meta_;
  std::map<int64_t, Live> live_;

  mutable std::mutex mu_;  // intake, stats, error
  std::condition_variable cv_;
  std::deque<std::pair<int64_t, GenRequest>> intake_;
  std::map<int64_t, std::shared_ptr<GenStream>> intake_streams_;
  std::deque<int64_t> aborts_, finishes_;
  int64_t next_id_ = 1;
  std::atomic<bool> stop_{false}, failed_{false};
  std::string error_;
  std::thread th_;
  ServeStats st_;
  std::vector<double> ttft_ms_, itl_ms_;
};

}  // namespace vmc
