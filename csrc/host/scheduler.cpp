#include "scheduler.hpp"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace vmc {

Scheduler::Scheduler(const SchedulerConfig& cfg, std::shared_ptr<BlockManager> kv) : cfg_(cfg), kv_(std::move(kv)) {
  if (cfg_.max_num_seqs <= 0) cfg_.max_num_seqs = 1;
  if (cfg_.max_num_batched_tokens < cfg_.max_num_seqs)
    throw std::runtime_error("--max-num-batched-tokens (" + std::to_string(cfg_.max_num_batched_tokens) +
                             ") must be >= --max-num-seqs (" + std::to_string(cfg_.max_num_seqs) + ")");
  for (int s = cfg_.max_num_seqs - 1; s >= 0; --s) free_slots_.push_back(s);
}

double Scheduler::now_s() {
  using namespace std::chrono;
  return duration_cast<duration<double>>(steady_clock::now().time_since_epoch()).count();
}

int Scheduler::take_slot() {
  if (free_slots_.empty()) throw std::runtime_error("scheduler: no free sequence slot");
  int s = free_slots_.back();
  free_slots_.pop_back();
  return s;
}

void Scheduler::give_slot(int slot) {
  if (slot >= 0) free_slots_.push_back(slot);
}

void Scheduler::add_request(int64_t id, std::vector<int32_t> prompt, const SeqParams& params) {
  if (seqs_.count(id)) throw std::runtime_error("scheduler: duplicate request id " + std::to_string(id));
  if (prompt.empty()) throw std::runtime_error("scheduler: empty prompt");
  auto s = std::make_unique<Seq>();
  s->id = id;
  s->prompt = std::move(prompt);
  s->params = params;
  s->arrival_s = now_s();
  waiting_.push_back(s.get());
  seqs_[id] = std::move(s);
}

const Seq* Scheduler::find(int64_t id) const {
  auto it = seqs_.find(id);
  return it == seqs_.end() ? nullptr : it->second.get();
}

void Scheduler::release(int64_t id) {
  auto it = seqs_.find(id);
  if (it != seqs_.end() && it->second->status == SeqStatus::FINISHED) seqs_.erase(it);
}

bool Scheduler::abort_request(int64_t id) {
  auto it = seqs_.find(id);
  if (it == seqs_.end() || it->second->status == SeqStatus::FINISHED) return false;
  finish(*it->second, FinishReason::ABORTED);
  return true;
}

void Scheduler::finish_request(int64_t id, FinishReason reason) {
  auto it = seqs_.find(id);
  if (it == seqs_.end() || it->second->status == SeqStatus::FINISHED) return;
  finish(*it->second, reason);
}

void Scheduler::cache_prompt_blocks(Seq& s) {
  if (!kv_->prefix_caching() || !kv_->has(s.id)) return;
  int64_t done = std::min<int64_t>(static_cast<int64_t>(s.prompt.size()), s.num_computed);
  int nfull = static_cast<int>(done / kv_->block_size());
  if (nfull <= 0) return;
  auto hashes = BlockManager::block_hashes(s.prompt.data(), static_cast<int64_t>(nfull) * kv_->block_size(), kv_->block_size());
  kv_->cache_full_blocks(s.id, hashes, nfull);
}

void Scheduler::finish(Seq& s, FinishReason reason) {
  if (s.status == SeqStatus::RUNNING) {
    cache_prompt_blocks(s);
    running_.erase(std::remove(running_.begin(), running_.end(), &s), running_.end());
  } else {
    waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), &s), waiting_.end());
  }
  kv_->free(s.id);
  give_slot(s.slot);
  s.slot = -1;
  s.status = SeqStatus::FINISHED;
  s.finish = reason;
}

void Scheduler::add_entry(Plan& plan, const Seq& s, int n, bool is_decode) {
  PlanEntry e;
  e.id = s.id;
  e.slot = s.slot;
  e.num_tokens = n;
  e.start = s.num_computed;
  e.sample = s.num_computed + n >= s.known();
  e.is_decode = is_decode;
  plan.entries.push_back(e);
  budget_ -= n;
}

void Scheduler::preempt(Seq& victim, Plan& plan) {
  // Drop the victim's entry if it was already scheduled in this step.
  auto& es = plan.entries;
  for (size_t k = 0; k < es.size(); ++k) {
    if (es[k].id == victim.id) {
      budget_ += es[k].num_tokens;
      es.erase(es.begin() + static_cast<long>(k));
      break;
    }
  }
  kv_->free(victim.id);
  give_slot(victim.slot);
  victim.slot = -1;
  victim.status = SeqStatus::PREEMPTED;
  victim.num_computed = 0;
  victim.num_preemptions += 1;
  running_.erase(std::remove(running_.begin(), running_.end(), &victim), running_.end());
  waiting_.push_front(&victim);
  plan.preempted.push_back(victim.id);
}

bool Scheduler::reserve(Seq& s, int64_t upto, Plan& plan) {
  while (!kv_->can_allocate(s.id, upto)) {
    Seq* victim = nullptr;
    for (auto it = running_.rbegin(); it != running_.rend(); ++it) {
      if (*it != &s) { victim = *it; break; }
    }
    if (!victim) {
      // Alone and still out of blocks: recompute later (the request itself is the victim).
      if (s.status == SeqStatus::RUNNING) preempt(s, plan);
      return false;
    }
    preempt(*victim, plan);
  }
  if (!kv_->allocate(s.id, upto)) return false;
  return true;
}

bool Scheduler::check_decode_latency() {
  if (!cfg_.preempt_prefill_on_latency || cfg_.decode_latency_target_ms <= 0) return false;
  double now = now_s();
  for (Seq* s : running_) {
    if (s->status != SeqStatus::RUNNING || s->is_prefill() || s->output.empty() || s->last_token_s <= 0) continue;
    if ((now - s->last_token_s) * 1000.0 > cfg_.decode_latency_target_ms) return true;
  }
  return false;
}

void Scheduler::admit_waiting(Plan& plan) {
  int remaining_seqs = cfg_.max_num_seqs - static_cast<int>(running_.size());
  size_t idx = 0;
  const int bs = kv_->block_size();
  while (idx < waiting_.size() && budget_ > 0 && remaining_seqs > 0) {
    Seq& s = *waiting_[idx];
    if (s.output.empty() && static_cast<int64_t>(s.prompt.size()) > cfg_.max_model_len) {
      s.prompt.erase(s.prompt.begin(), s.prompt.end() - cfg_.max_model_len);  // keep the tail
    }
    int64_t cached = 0;
    std::vector<int32_t> hits;
    if (kv_->prefix_caching()) {
      int64_t n = static_cast<int64_t>(s.prompt.size());
      int max_blocks = static_cast<int>((n - 1) / bs);
      if (max_blocks > 0) {
        auto hashes = BlockManager::block_hashes(s.prompt.data(), n, bs);
        ++prefix_queries_;
        int h = kv_->find_longest_prefix_hit(hashes, max_blocks, hits);
        if (h > 0) {
          cached = static_cast<int64_t>(h) * bs;
          ++prefix_hits_;
          prefix_hit_tokens_ += cached;
        }
      }
    }
    int64_t to_compute = s.known() - cached;
    int new_budget = budget_;
    if (cfg_.max_prefill_per_batch > 0) {
      int already = 0;
      for (auto& e : plan.entries) if (!e.is_decode) already += e.num_tokens;
      new_budget = std::min(new_budget, cfg_.max_prefill_per_batch - already);
    }
    if (new_budget <= 0) break;
    int64_t chunk = to_compute;
    if (cfg_.enable_chunked_prefill) {
      if (cfg_.long_prefill_token_threshold > 0) chunk = std::min<int64_t>(chunk, cfg_.long_prefill_token_threshold);
      chunk = std::min<int64_t>(chunk, new_budget);
    } else if (chunk > new_budget) {
      ++idx;
      continue;
    }
    if (chunk <= 0) { ++idx; continue; }
    if (!kv_->allocate(s.id, cached + chunk, hits)) {
      // Try to make room from running requests that are not part of this step.
      bool ok = false;
      while (true) {
        Seq* victim = nullptr;
        for (auto it = running_.rbegin(); it != running_.rend(); ++it) {
          bool scheduled = false;
          for (auto& e : plan.entries) scheduled |= e.id == (*it)->id;
          if (!scheduled) { victim = *it; break; }
        }
        if (!victim) break;
        preempt(*victim, plan);
        ++remaining_seqs;
        if (kv_->allocate(s.id, cached + chunk, hits)) { ok = true; break; }
      }
      if (!ok) { ++idx; continue; }
      // The preempted victims were pushed to the front of the waiting queue; find `s` again.
      idx = static_cast<size_t>(std::find(waiting_.begin(), waiting_.end(), &s) - waiting_.begin());
    }
    s.status = SeqStatus::RUNNING;
    s.slot = take_slot();
    s.num_computed = cached;
    s.num_cached_tokens = cached;
    plan.num_cached_tokens += cached;
    add_entry(plan, s, static_cast<int>(chunk), false);
    running_.push_back(&s);
    waiting_.erase(waiting_.begin() + static_cast<long>(idx));
    --remaining_seqs;
  }
}

void Scheduler::schedule_decode_first(Plan& plan) {
  // Phase 1: one token for every running decode.
  std::vector<Seq*> snapshot = running_;
  for (Seq* s : snapshot) {
    if (s->status != SeqStatus::RUNNING || s->is_prefill()) continue;
    if (budget_ < 1) continue;
    if (!reserve(*s, s->num_computed + 1 + cfg_.num_lookahead_tokens, plan)) continue;
    add_entry(plan, *s, 1, true);
  }
  // Phase 2: a decode that waited too long stops new prefill work this step.
  if (check_decode_latency()) {
    plan.decode_latency_preempt = true;
    return;
  }
  // Phase 3: chunks of running prefills.
  int prefill_budget = budget_;
  if (cfg_.decode_reserved_tokens > 0) prefill_budget = std::max(0, prefill_budget - cfg_.decode_reserved_tokens);
  if (cfg_.max_prefill_per_batch > 0) prefill_budget = std::min(prefill_budget, cfg_.max_prefill_per_batch);
  snapshot = running_;
  for (Seq* s : snapshot) {
    if (prefill_budget <= 0) break;
    if (s->status != SeqStatus::RUNNING || !s->is_prefill()) continue;
    bool scheduled = false;
    for (auto& e : plan.entries) scheduled |= e.id == s->id;
    if (scheduled) continue;
    int64_t chunk = s->known() - s->num_computed;
    if (cfg_.long_prefill_token_threshold > 0) chunk = std::min<int64_t>(chunk, cfg_.long_prefill_token_threshold);
    chunk = std::min<int64_t>(chunk, prefill_budget);
    if (chunk <= 0) continue;
    if (!kv_->allocate(s->id, s->num_computed + chunk)) continue;
    add_entry(plan, *s, static_cast<int>(chunk), false);
    prefill_budget -= static_cast<int>(chunk);
  }
  // Phase 4: admit waiting requests.
  admit_waiting(plan);
}

void Scheduler::schedule_fair(Plan& plan) {
  std::vector<Seq*> snapshot = running_;
  for (Seq* s : snapshot) {
    if (budget_ <= 0) break;
    if (s->status != SeqStatus::RUNNING) continue;
    if (s->is_prefill()) {
      int64_t chunk = s->known() - s->num_computed;
      if (cfg_.long_prefill_token_threshold > 0) chunk = std::min<int64_t>(chunk, cfg_.long_prefill_token_threshold);
      chunk = std::min<int64_t>(chunk, budget_);
      if (chunk <= 0) continue;
      if (!kv_->allocate(s->id, s->num_computed + chunk)) continue;
      add_entry(plan, *s, static_cast<int>(chunk), false);
    } else {
      if (!reserve(*s, s->num_computed + 1 + cfg_.num_lookahead_tokens, plan)) continue;
      add_entry(plan, *s, 1, true);
    }
  }
  admit_waiting(plan);
}

Plan Scheduler::schedule() {
  Plan plan;
  budget_ = cfg_.max_num_batched_tokens;
  if (cfg_.decode_first) schedule_decode_first(plan); else schedule_fair(plan);
  std::stable_partition(plan.entries.begin(), plan.entries.end(), [](const PlanEntry& e) { return e.is_decode; });
  for (auto& e : plan.entries) {
    plan.total_tokens += e.num_tokens;
    plan.num_decode += e.is_decode ? 1 : 0;
    plan.num_sample += e.sample ? 1 : 0;
  }
  return plan;
}

void Scheduler::build_batch(const Plan& plan, const BatchLayout& L, int32_t* buf, int pad_to_reqs) const {
  const int R = static_cast<int>(plan.entries.size());
  const int T = plan.total_tokens;
  const int bs = kv_->block_size();
  if (T > L.max_tokens) throw std::runtime_error("build_batch: too many tokens for the metadata buffer");
  int Rp = std::max(R, pad_to_reqs);
  if (Rp > L.max_reqs) throw std::runtime_error("build_batch: too many requests for the metadata buffer");
  if (pad_to_reqs > R && plan.num_decode != R) throw std::runtime_error("build_batch: padding needs a decode-only plan");
  int32_t* ids = buf + L.off_input_ids();
  int32_t* pos = buf + L.off_positions();
  int32_t* slots = buf + L.off_slot_mapping();
  int32_t* qs = buf + L.off_q_start();
  int32_t* ctx = buf + L.off_ctx_len();
  int32_t* sslot = buf + L.off_seq_slot();
  int32_t* lidx = buf + L.off_logits_idx();
  int32_t* sreq = buf + L.off_sample_req();
  int32_t* counts = buf + L.off_counts();
  int32_t* bt = buf + L.off_block_tables();
  int t = 0, k = 0, max_q = 0;
  int64_t max_ctx = 0;
  for (int r = 0; r < R; ++r) {
    const PlanEntry& e = plan.entries[r];
    const Seq& s = *seqs_.at(e.id);
    const auto& blocks = kv_->blocks_of(e.id);
    if (static_cast<int>(blocks.size()) > L.max_blocks_per_seq) throw std::runtime_error("build_batch: block table row overflow");
    qs[r] = t;
    for (int j = 0; j < e.num_tokens; ++j, ++t) {
      int64_t p = e.start + j;
      ids[t] = s.token_at(p);
      pos[t] = static_cast<int32_t>(p);
      slots[t] = blocks.at(static_cast<size_t>(p / bs)) * bs + static_cast<int32_t>(p % bs);
    }
    ctx[r] = static_cast<int32_t>(e.start + e.num_tokens);
    sslot[r] = e.slot;
    int32_t* row = bt + static_cast<int64_t>(r) * L.max_blocks_per_seq;
    std::copy(blocks.begin(), blocks.end(), row);
    std::fill(row + blocks.size(), row + L.max_blocks_per_seq, 0);
    if (e.sample) {
      lidx[k] = t - 1;
      sreq[k] = r;
      ++k;
    }
    max_q = std::max(max_q, e.num_tokens);
    max_ctx = std::max<int64_t>(max_ctx, e.start + e.num_tokens);
  }
  // Padding rows (decode CUDA graphs): one dummy token each, no KV write, empty context.
  int Tp = T;
  for (int r = R; r < Rp; ++r, ++Tp) {
    qs[r] = Tp;
    ids[Tp] = 0;
    pos[Tp] = 0;
    slots[Tp] = -1;
    ctx[r] = 0;
    sslot[r] = -1;
    std::fill(bt + static_cast<int64_t>(r) * L.max_blocks_per_seq, bt + static_cast<int64_t>(r + 1) * L.max_blocks_per_seq, 0);
    lidx[k] = Tp;
    sreq[k] = r;
    ++k;
  }
  qs[Rp] = Tp;
  counts[0] = T;
  counts[1] = R;
  counts[2] = plan.num_sample;
  counts[3] = plan.num_decode;
  counts[4] = max_q;
  counts[5] = static_cast<int32_t>(max_ctx);
  counts[6] = Tp;
  counts[7] = Rp;
}

std::vector<StepEvent> Scheduler::update(const Plan& plan, const std::vector<std::vector<int32_t>>& tokens) {
  std::vector<StepEvent> events;
  size_t k = 0;
  double now = now_s();
  for (const PlanEntry& e : plan.entries) {
    const std::vector<int32_t>* toks = nullptr;
    if (e.sample) {
      if (k >= tokens.size()) throw std::runtime_error("update: fewer token lists than sampled entries");
      toks = &tokens[k++];
    }
    auto it = seqs_.find(e.id);
    if (it == seqs_.end()) continue;
    Seq& s = *it->second;
    if (s.status != SeqStatus::RUNNING) continue;  // aborted or preempted meanwhile
    bool was_prefill = s.num_computed < static_cast<int64_t>(s.prompt.size());
    s.num_computed = e.start + e.num_tokens;
    if (was_prefill && s.num_computed >= static_cast<int64_t>(s.prompt.size())) cache_prompt_blocks(s);
    if (!toks) continue;
    // Speculative decoding: a decode entry that returns m > 1 tokens had m - 1 of them verified in
    // the same step (their KV is written); only the last one still has to be processed.
    if (!was_prefill && toks->size() > 1) s.num_computed += static_cast<int64_t>(toks->size()) - 1;
    StepEvent ev{s.id, {}, false, FinishReason::NONE};
    for (int32_t tok : *toks) {
      s.output.push_back(tok);
      ev.tokens.push_back(tok);
      if (s.first_token_s <= 0) s.first_token_s = now;
      s.last_token_s = now;
      int n_out = static_cast<int>(s.output.size());
      bool is_eos = std::find(s.params.eos_token_ids.begin(), s.params.eos_token_ids.end(), tok) != s.params.eos_token_ids.end();
      bool is_stop = std::find(s.params.stop_token_ids.begin(), s.params.stop_token_ids.end(), tok) != s.params.stop_token_ids.end();
      bool below_min = n_out <= s.params.min_tokens;
      if (s.params.ignore_eos) is_eos = false;
      if (below_min) is_eos = is_stop = false;
      bool hit_max = n_out >= s.params.max_tokens || s.known() >= cfg_.max_model_len;
      if (is_eos || is_stop || hit_max) {
        ev.finished = true;
        ev.reason = (is_eos || is_stop) ? FinishReason::STOP : FinishReason::LENGTH;
        break;
      }
    }
    if (ev.finished) finish(s, ev.reason);
    events.push_back(std::move(ev));
  }
  return events;
}

}  // namespace vmc
