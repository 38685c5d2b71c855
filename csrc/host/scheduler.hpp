// Continuous-batching scheduler with chunked prefill, prefix caching and preemption.
//
// Policy semantics follow the reference (src/core/scheduler.cpp): the decode-first schedule
// (schedule_decode_first :98 — every running decode gets one token, a decode that waited longer
// than decode_latency_target_ms stops new prefill, running prefill chunks, then admission from the
// waiting queue with prompt truncation to max_model_len, prefix-cache lookup capped at
// num_tokens-1, and preemption-by-recompute of the newest running request), the legacy "fair"
// policy (schedule :300-444), chained FNV-1a block hashes (:36-55), update_from_output (:508) and
// finish_request (:480). Differences by design: block allocation happens here, at schedule time,
// so a running decode that cannot get a block preempts the newest request instead of failing in
// the forward pass; a preempted request recomputes prompt and generated tokens; and the step's
// device metadata (token ids, positions, slot mapping, block tables, sample rows) is written by
// build_batch directly into a caller-provided pinned buffer.
#pragma once
#include <chrono>
#include <cstdint>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "block_manager.hpp"

namespace vmc {

struct SchedulerConfig {
  int max_num_seqs = 128;
  int max_num_batched_tokens = 2048;
  int max_model_len = 4096;
  bool enable_chunked_prefill = true;
  int long_prefill_token_threshold = 0;
  bool decode_first = true;  // "decode_first" policy; false selects the legacy "fair" policy
  int max_prefill_per_batch = 0;
  int decode_latency_target_ms = 100;
  bool preempt_prefill_on_latency = true;
  int decode_reserved_tokens = 0;
  int num_lookahead_tokens = 0;  // extra KV slots reserved per decode (speculative decoding)
};

enum class SeqStatus : int { WAITING = 0, RUNNING = 1, FINISHED = 2, PREEMPTED = 3 };
enum class FinishReason : int { NONE = -1, STOP = 0, LENGTH = 1, ERROR = 2, ABORTED = 3 };

struct SeqParams {
  int max_tokens = 16;
  int min_tokens = 0;
  bool ignore_eos = false;
  std::vector<int32_t> stop_token_ids;  // request stop ids (honoured after min_tokens)
  std::vector<int32_t> eos_token_ids;   // model EOS ids (ignored when ignore_eos)
};

struct Seq {
  int64_t id = 0;
  std::vector<int32_t> prompt;
  std::vector<int32_t> output;
  int64_t num_computed = 0;
  SeqStatus status = SeqStatus::WAITING;
  FinishReason finish = FinishReason::NONE;
  SeqParams params;
  int slot = -1;
  int64_t num_cached_tokens = 0;  // prefix-cache hit length at admission
  int num_preemptions = 0;
  double arrival_s = 0, first_token_s = 0, last_token_s = 0;
  int64_t known() const { return static_cast<int64_t>(prompt.size() + output.size()); }
  int32_t token_at(int64_t pos) const {
    return pos < static_cast<int64_t>(prompt.size()) ? prompt[pos] : output[pos - prompt.size()];
  }
  bool is_prefill() const { return num_computed < static_cast<int64_t>(prompt.size()) || known() - num_computed > 1; }
};

struct PlanEntry {
  int64_t id;
  int slot;
  int num_tokens;     // tokens computed this step
  int64_t start;      // num_computed before the step (position of the first token)
  bool sample;        // this step reaches the last known token: sample a new one
  bool is_decode;
};

struct Plan {
  std::vector<PlanEntry> entries;  // decodes first, then prefill chunks
  int total_tokens = 0;
  int num_decode = 0;
  int num_sample = 0;
  int64_t num_cached_tokens = 0;
  std::vector<int64_t> preempted;
  bool decode_latency_preempt = false;
};

// One event per entry that produced tokens or finished.
struct StepEvent {
  int64_t id;
  std::vector<int32_t> tokens;
  bool finished;
  FinishReason reason;
};

struct BatchLayout {
  // Capacities used to place the sections of the int32 metadata buffer.
  int max_tokens;
  int max_reqs;
  int max_blocks_per_seq;
  // Offsets (in int32 elements) of each section.
  int64_t off_input_ids() const { return 0; }
  int64_t off_positions() const { return max_tokens; }
  int64_t off_slot_mapping() const { return 2LL * max_tokens; }
  int64_t off_q_start() const { return 3LL * max_tokens; }                 // max_reqs + 1
  int64_t off_ctx_len() const { return off_q_start() + max_reqs + 1; }      // max_reqs
  int64_t off_seq_slot() const { return off_ctx_len() + max_reqs; }         // max_reqs
  int64_t off_logits_idx() const { return off_seq_slot() + max_reqs; }      // max_reqs (sample rows)
  int64_t off_sample_req() const { return off_logits_idx() + max_reqs; }    // max_reqs
  int64_t off_counts() const { return off_sample_req() + max_reqs; }        // 8 ints
  int64_t off_block_tables() const { return off_counts() + 8; }             // max_reqs * max_blocks
  int64_t total() const { return off_block_tables() + static_cast<int64_t>(max_reqs) * max_blocks_per_seq; }
};

class Scheduler {
 public:
  Scheduler(const SchedulerConfig& cfg, std::shared_ptr<BlockManager> kv);

  void add_request(int64_t id, std::vector<int32_t> prompt, const SeqParams& params);
  // Returns true if the request existed and was not finished yet.
  bool abort_request(int64_t id);
  Plan schedule();
  // Write the device metadata for `plan` into `buf` (layout.total() int32 elements). Decode-only
  // plans can be padded to `pad_to_reqs` rows for CUDA-graph replay.
  void build_batch(const Plan& plan, const BatchLayout& layout, int32_t* buf, int pad_to_reqs = 0) const;
  // tokens[k] holds the new tokens for the k-th sampling entry of `plan` (in entry order).
  std::vector<StepEvent> update(const Plan& plan, const std::vector<std::vector<int32_t>>& tokens);
  // Mark a running request finished (e.g. a stop string matched on the host).
  void finish_request(int64_t id, FinishReason reason);

  int num_waiting() const { return static_cast<int>(waiting_.size()); }
  int num_running() const { return static_cast<int>(running_.size()); }
  bool has_unfinished() const { return !waiting_.empty() || !running_.empty(); }
  const Seq* find(int64_t id) const;
  const SchedulerConfig& config() const { return cfg_; }
  BlockManager& kv() { return *kv_; }
  int64_t prefix_queries() const { return prefix_queries_; }
  int64_t prefix_hits() const { return prefix_hits_; }
  int64_t prefix_hit_tokens() const { return prefix_hit_tokens_; }
  // Drop finished sequences' bookkeeping (their events were already returned).
  void release(int64_t id);

 private:
  static double now_s();
  void schedule_decode_first(Plan& plan);
  void schedule_fair(Plan& plan);
  bool check_decode_latency();
  // Admit waiting requests while the token budget and sequence slots allow.
  void admit_waiting(Plan& plan);
  void add_entry(Plan& plan, const Seq& s, int n, bool is_decode);
  // Make sure `s` owns blocks for `upto` tokens, preempting the newest running requests if needed.
  bool reserve(Seq& s, int64_t upto, Plan& plan);
  void preempt(Seq& victim, Plan& plan);
  int take_slot();
  void give_slot(int slot);
  void cache_prompt_blocks(Seq& s);
  void finish(Seq& s, FinishReason reason);

  SchedulerConfig cfg_;
  std::shared_ptr<BlockManager> kv_;
  std::unordered_map<int64_t, std::unique_ptr<Seq>> seqs_;
  std::deque<Seq*> waiting_;
  std::vector<Seq*> running_;
  std::vector<int> free_slots_;
  int budget_ = 0;  // token budget left while a schedule() call is running
  int64_t prefix_queries_ = 0, prefix_hits_ = 0, prefix_hit_tokens_ = 0;
};

}  // namespace vmc
