// Native serving loop (see serve_loop.hpp).
#include "serve_loop.hpp"

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <stdexcept>

namespace vmc {

namespace {

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

double percentile(std::vector<double> v, double p) {
  if (v.empty()) return 0;
  std::sort(v.begin(), v.end());
  const double k = (v.size() - 1) * p / 100.0;
  const size_t f = static_cast<size_t>(k);
  const size_t c = std::min(v.size() - 1, f + 1);
  return v[f] + (v[c] - v[f]) * (k - f);
}

// FNV-1a of the request name: the sampling seed of a request that gave none (deterministic, so a
// replayed request samples the same tokens).
uint64_t name_seed(const std::string& s) {
  uint64_t h = 0xcbf29ce484222325ULL;
  for (unsigned char c : s) {
    h ^= c;
    h *= 0x100000001b3ULL;
  }
  return h & 0x7fffffffffffffffULL;
}

}  // namespace

bool GenStream::next(GenEvent& ev, int timeout_ms) {
  std::unique_lock<std::mutex> lk(mu_);
  if (!cv_.wait_for(lk, std::chrono::milliseconds(timeout_ms), [this] { return !q_.empty(); })) return false;
  ev = std::move(q_.front());
  q_.pop_front();
  // merge whatever else is queued (the consumer fell behind the loop)
  while (!q_.empty() && !ev.finished) {
    GenEvent& n = q_.front();
    ev.tokens.insert(ev.tokens.end(), n.tokens.begin(), n.tokens.end());
    ev.logprobs.insert(ev.logprobs.end(), n.logprobs.begin(), n.logprobs.end());
    ev.finished = n.finished;
    ev.reason = n.reason;
    q_.pop_front();
  }
  return true;
}

void GenStream::push(GenEvent ev) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    q_.push_back(std::move(ev));
  }
  cv_.notify_all();
}

ServeLoop::ServeLoop(const ServeConfig& cfg, StepBackend& backend) : cfg_(cfg), be_(backend) {
  layout_ = be_.layout();
  if (cfg_.num_blocks <= 0) throw std::invalid_argument("ServeLoop: num_blocks must be positive");
  kv_ = std::make_shared<BlockManager>(cfg_.num_blocks, cfg_.block_size, cfg_.prefix_caching);
  sched_ = std::make_unique<Scheduler>(cfg_.sched, kv_);
  meta_.assign(static_cast<size_t>(layout_.total()), 0);
}

ServeLoop::~ServeLoop() { stop(); }

std::shared_ptr<GenStream> ServeLoop::submit(const GenRequest& r) {
  if (r.prompt.empty()) throw std::invalid_argument("empty prompt");
  const int V = be_.vocab();
  for (int32_t t : r.prompt)
    if (t < 0 || t >= V) throw std::invalid_argument("prompt contains token ids outside the model vocabulary");
  std::shared_ptr<GenStream> s;
  {
    std::lock_guard<std::mutex> lk(mu_);
    if (failed_.load()) throw std::runtime_error("engine failed: " + error_);
    const int64_t id = next_id_++;
    s = std::make_shared<GenStream>(id);
    intake_.emplace_back(id, r);
    intake_streams_[id] = s;
    ++st_.requests;
  }
  cv_.notify_all();
  return s;
}

void ServeLoop::abort(int64_t id) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    aborts_.push_back(id);
  }
  cv_.notify_all();
}

void ServeLoop::finish(int64_t id) {
  {
    std::lock_guard<std::mutex> lk(mu_);
    finishes_.push_back(id);
  }
  cv_.notify_all();
}

void ServeLoop::close(int64_t id, FinishReason reason) {
  auto it = live_.find(id);
  if (it == live_.end()) return;
  GenEvent ev;
  ev.finished = true;
  ev.reason = reason;
  it->second.stream->push(std::move(ev));
  sched_->release(id);
  live_.erase(it);
  std::lock_guard<std::mutex> lk(mu_);
  ++st_.finished;
  if (reason == FinishReason::ABORTED) ++st_.aborted;
  if (reason == FinishReason::ERROR) ++st_.errors;
}

void ServeLoop::drain() {
  std::deque<std::pair<int64_t, GenRequest>> in;
  std::map<int64_t, std::shared_ptr<GenStream>> streams;
  std::deque<int64_t> ab, fin;
  {
    std::lock_guard<std::mutex> lk(mu_);
    in.swap(intake_);
    streams.swap(intake_streams_);
    ab.swap(aborts_);
    fin.swap(finishes_);
  }
  const double t = now_ms();
  for (auto& [id, r] : in) {
    SeqParams sp;
    sp.max_tokens = std::max(1, r.max_tokens);
    sp.min_tokens = r.min_tokens;
    sp.ignore_eos = r.ignore_eos;
    sp.stop_token_ids = r.stop_token_ids;
    sp.eos_token_ids = cfg_.eos_token_ids;
    sched_->add_request(id, r.prompt, sp);
    Live l;
    l.seed = r.has_seed ? r.seed : name_seed(r.name.empty() ? "req-" + std::to_string(id) : r.name);
    l.req = std::move(r);
    l.stream = streams[id];
    l.arrival = t;
    live_.emplace(id, std::move(l));
  }
  for (int64_t id : ab)
    if (live_.count(id)) {
      sched_->abort_request(id);
      close(id, FinishReason::ABORTED);
    }
  for (int64_t id : fin)
    if (live_.count(id)) {
      sched_->finish_request(id, FinishReason::STOP);
      close(id, FinishReason::STOP);
    }
}

bool ServeLoop::step_once() {
  drain();
  if (!sched_->has_unfinished()) {
    publish();
    return false;
  }
  const double t0 = now_ms();
  Plan plan = sched_->schedule();
  {
    std::lock_guard<std::mutex> lk(mu_);
    st_.preemptions += static_cast<int64_t>(plan.preempted.size());
  }
  if (plan.entries.empty()) {  // nothing fits this step
    publish();
    return false;
  }
  // sampled rows in entry order: their parameters and penalty triples
  std::vector<SampleParams> params;
  Penalties pen;
  std::vector<int64_t> sample_ids;
  for (const PlanEntry& e : plan.entries) {
    if (!e.sample) continue;
    Live& l = live_.at(e.id);
    const GenRequest& r = l.req;
    SampleParams p{};
    p.temperature = r.greedy() ? 0.f : r.temperature;
    p.top_k = r.top_k;
    p.top_p = r.top_p;
    p.min_p = r.min_p;
    p.repetition_penalty = r.repetition_penalty;
    p.frequency_penalty = r.frequency_penalty;
    p.presence_penalty = r.presence_penalty;
    p.step = l.generated;
    p.seed = l.seed;
    if (r.has_penalties()) {
      const int row = static_cast<int>(params.size());
      std::map<int32_t, int32_t> counts;
      for (int32_t tk : r.prompt) counts.emplace(tk, 0);
      for (const auto& [tk, c] : l.out_counts) counts[tk] = c;
      for (const auto& [tk, c] : counts) {
        pen.row.push_back(row);
        pen.token.push_back(tk);
        pen.count.push_back(c);
      }
    }
    params.push_back(p);
    sample_ids.push_back(e.id);
  }
  const bool all_decode = plan.num_decode == static_cast<int>(plan.entries.size());
  const int pad = (all_decode && pen.empty()) ? be_.graph_bucket(static_cast<int>(plan.entries.size())) : 0;
  sched_->build_batch(plan, layout_, meta_.data(), pad);
  const int32_t* cnt = meta_.data() + layout_.off_counts();
  const int S = cnt[2];
  if (S != static_cast<int>(params.size())) throw std::logic_error("ServeLoop: sample row count mismatch");
  std::vector<int32_t> toks(static_cast<size_t>(std::max(S, 1)));
  std::vector<float> lps(static_cast<size_t>(std::max(S, 1)));
  be_.step(meta_.data(), params.data(), S, pen, toks.data(), lps.data());
  std::vector<std::vector<int32_t>> per_row(static_cast<size_t>(S));
  for (int k = 0; k < S; ++k) per_row[k] = {toks[k]};
  std::map<int64_t, float> lp_of;
  for (int k = 0; k < S; ++k) lp_of[sample_ids[k]] = lps[k];
  const double t1 = now_ms();
  for (StepEvent& ev : sched_->update(plan, per_row)) {
    auto it = live_.find(ev.id);
    if (it == live_.end()) continue;
    Live& l = it->second;
    GenEvent ge;
    ge.tokens = ev.tokens;
    for (size_t k = 0; k < ev.tokens.size(); ++k) ge.logprobs.push_back(lp_of.count(ev.id) ? lp_of[ev.id] : 0.f);
    l.generated += static_cast<int>(ev.tokens.size());
    if (l.req.has_penalties())
      for (int32_t tk : ev.tokens) ++l.out_counts[tk];
    {
      std::lock_guard<std::mutex> lk(mu_);
      st_.tokens_generated += static_cast<int64_t>(ev.tokens.size());
      if (!ev.tokens.empty()) {
        if (l.last < 0) ttft_ms_.push_back(t1 - l.arrival);
        else itl_ms_.push_back(t1 - l.last);
      }
    }
    if (!ev.tokens.empty()) l.last = t1;
    ge.finished = ev.finished;
    ge.reason = ev.reason;
    l.stream->push(std::move(ge));
    if (ev.finished) {
      sched_->release(ev.id);
      live_.erase(it);
      std::lock_guard<std::mutex> lk(mu_);
      ++st_.finished;
    }
  }
  {
    std::lock_guard<std::mutex> lk(mu_);
    ++st_.steps;
    st_.tokens_scheduled += cnt[0];
    st_.step_time_s += (now_ms() - t0) / 1e3;
    for (auto* v : {&ttft_ms_, &itl_ms_})
      if (v->size() > 200000) v->erase(v->begin(), v->begin() + 100000);  // keep recent samples
  }
  publish();
  return true;
}

void ServeLoop::publish() {
  std::lock_guard<std::mutex> lk(mu_);
  st_.running = sched_->num_running();
  st_.waiting = sched_->num_waiting() + static_cast<int>(intake_.size());
  st_.kv_usage = kv_->usage();
  st_.prefix_queries = sched_->prefix_queries();
  st_.prefix_hits = sched_->prefix_hits();
}

void ServeLoop::loop() {
  while (!stop_.load()) {
    bool busy = false;
    try {
      busy = step_once();
    } catch (const std::exception& e) {
      // fail every in-flight request; keep the loop alive so that the server can report the error
      {
        std::lock_guard<std::mutex> lk(mu_);
        error_ = e.what();
      }
      fprintf(stderr, "vmc serve: step failed: %s\n", e.what());
      std::vector<int64_t> ids;
      for (const auto& kv : live_) ids.push_back(kv.first);
      for (int64_t id : ids) {
        sched_->abort_request(id);
        close(id, FinishReason::ERROR);
      }
      if (dynamic_cast<const std::logic_error*>(&e) == nullptr) failed_.store(true);
      busy = false;
    }
    if (!busy) {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait_for(lk, std::chrono::milliseconds(cfg_.idle_wait_ms),
                   [this] { return stop_.load() || !intake_.empty() || !aborts_.empty() || !finishes_.empty(); });
    }
  }
  // shutting down: finish whatever is left
  drain();
  std::vector<int64_t> ids;
  for (const auto& kv : live_) ids.push_back(kv.first);
  for (int64_t id : ids) {
    sched_->abort_request(id);
    close(id, FinishReason::ABORTED);
  }
}

void ServeLoop::start() {
  th_ = std::thread([this] { loop(); });
}

void ServeLoop::run() { loop(); }

void ServeLoop::stop() {
  stop_.store(true);
  cv_.notify_all();
  if (th_.joinable()) th_.join();
}

void ServeLoop::run_until_idle() {
  int stalled = 0;
  for (;;) {
    if (step_once()) {
      stalled = 0;
      continue;
    }
    if (!sched_->has_unfinished()) return;
    if (++stalled > 1000) throw std::runtime_error("ServeLoop: the remaining requests cannot be scheduled");
  }
}

ServeStats ServeLoop::stats() const {
  std::lock_guard<std::mutex> lk(mu_);
  ServeStats s = st_;
  s.p50_ttft_ms = percentile(ttft_ms_, 50);
  s.p50_itl_ms = percentile(itl_ms_, 50);
  s.p99_itl_ms = percentile(itl_ms_, 99);
  return s;
}

std::string ServeLoop::last_error() const {
  std::lock_guard<std::mutex> lk(mu_);
  return error_;
}

}  // namespace vmc
