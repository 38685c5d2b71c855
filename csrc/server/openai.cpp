// OpenAI-compatible routes (see openai.hpp).
#include "openai.hpp"

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <ctime>
#include <functional>
#include <mutex>
#include <random>
#include <stdexcept>

#include "json.hpp"

namespace vmc {

namespace {

using json::Value;

struct HttpError : std::runtime_error {
  int status;
  HttpError(int s, const std::string& m) : std::runtime_error(m), status(s) {}
};

std::string hex_id(size_t n) {
  static std::mutex mu;
  static std::mt19937_64 rng(std::random_device{}() ^
                             static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count()));
  std::lock_guard<std::mutex> lk(mu);
  static const char* d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) s += d[rng() & 15];
  return s;
}

int64_t unix_now() { return static_cast<int64_t>(time(nullptr)); }

const char* finish_str(FinishReason r) {
  switch (r) {
    case FinishReason::LENGTH: return "length";
    case FinishReason::ERROR: return "error";
    case FinishReason::ABORTED: return "abort";
    default: return "stop";
  }
}

void send_json(http::Responder& res, int status, const Value& v) { res.send(status, "application/json", json::dump(v)); }

void send_error(http::Responder& res, int status, const std::string& msg, const char* type = "invalid_request_error") {
  Value e = Value::object();
  e.set("message", msg).set("type", type).set("code", status);
  Value v = Value::object();
  v.set("error", e);
  send_json(res, status, v);
}

Value parse_body(const http::Request& rq) {
  try {
    Value v = json::parse(rq.body);
    if (!v.is_object()) throw HttpError(400, "the request body must be a JSON object");
    return v;
  } catch (const json::ParseError&) {
    throw HttpError(400, "invalid JSON body");
  }
}

// Sampling parameters of one request body (the Python server's _sampling_from).
struct BodyParams {
  GenRequest gen;
  std::vector<std::string> stop;
  bool enable_thinking = true, add_generation_prompt = true, echo = false;
  bool stream = false, include_usage = false, running_usage = false;
};

BodyParams body_params(const Value& b, int default_max) {
  BodyParams p;
  GenRequest& g = p.gen;
  // An HTTP request samples with temperature 1, top-p 1 and no top-k unless it says otherwise (the
  // OpenAI defaults, as the reference's request parsers apply them: src/server/http_server.cpp:157-162).
  g.temperature = 1.f;
  g.top_p = 1.f;
  g.top_k = 0;
  try {
    int64_t mt = b.get_int("max_completion_tokens", 0);
    if (mt == 0) mt = b.get_int("max_tokens", 0);
    g.max_tokens = static_cast<int>(mt > 0 ? mt : default_max);
    g.temperature = static_cast<float>(b.get_double("temperature", g.temperature));
    g.top_p = static_cast<float>(b.get_double("top_p", g.top_p));
    g.min_p = static_cast<float>(b.get_double("min_p", g.min_p));
    g.repetition_penalty = static_cast<float>(b.get_double("repetition_penalty", g.repetition_penalty));
    g.frequency_penalty = static_cast<float>(b.get_double("frequency_penalty", g.frequency_penalty));
    g.presence_penalty = static_cast<float>(b.get_double("presence_penalty", g.presence_penalty));
    g.top_k = static_cast<int>(b.get_int("top_k", g.top_k));
    if (const Value* s = b.get("stop")) {
      if (s->is_string()) p.stop.push_back(s->as_string());
      else if (s->is_array())
        for (const Value& x : s->as_array()) p.stop.push_back(x.as_string());
    }
    if (const Value* s = b.get("stop_token_ids"); s && s->is_array())
      for (const Value& x : s->as_array()) g.stop_token_ids.push_back(static_cast<int32_t>(x.as_int()));
    g.ignore_eos = b.get_bool("ignore_eos", false);
    g.min_tokens = static_cast<int>(b.get_int("min_tokens", 0));
    if (const Value* s = b.get("seed"); s && !s->is_null()) {
      g.has_seed = true;
      g.seed = static_cast<uint64_t>(s->as_int());
    }
    const Value* kw = b.get("chat_template_kwargs");
    const Value* et = kw ? kw->get("enable_thinking") : nullptr;
    if (!et || et->is_null()) et = b.get("enable_thinking");
    if (et && !et->is_null()) p.enable_thinking = et->as_bool();
    p.stream = b.get_bool("stream", false);
    p.echo = b.get_bool("echo", false);
    p.add_generation_prompt = b.get_bool("add_generation_prompt", true);
    if (const Value* so = b.get("stream_options"); so && so->is_object()) {
      p.include_usage = so->get_bool("include_usage", false);
      p.running_usage = so->get_bool("continuous_usage_stats", false);
    }
  } catch (const HttpError&) {
    throw;
  } catch (const std::exception& e) {
    throw HttpError(400, std::string("bad request parameter: ") + e.what());
  }
  if (g.max_tokens < 1) throw HttpError(400, "max_tokens must be positive");
  return p;
}

std::string content_text(const Value& c) {
  if (c.is_string()) return c.as_string();
  std::string out;
  if (c.is_array())
    for (const Value& part : c.as_array())
      if (part.is_object()) out += part.get_string("text", "");
  return out;
}

Value usage(size_t prompt, size_t completion) {
  Value u = Value::object();
  u.set("prompt_tokens", static_cast<int64_t>(prompt))
      .set("completion_tokens", static_cast<int64_t>(completion))
      .set("total_tokens", static_cast<int64_t>(prompt + completion));
  return u;
}

bool sse(http::Responder& res, const Value& v) { return res.write("data: " + json::dump(v) + "\n\n"); }

// Request diagnostics (the reference's env switches, src/main.cpp:527-570, 673-700):
// VMC_LOG_PROMPT_VERBOSE=1 logs each prompt with its token ids and whether detokenising them gives it
// back; VMC_LOG_DETOK=1 logs every generated token's id and text when a request ends.
bool env_on(const char* name) {
  const char* v = getenv(name);
  return v && v[0] == '1';
}

void log_prompt(const TextTokenizer& tok, const std::string& prompt, const std::vector<int32_t>& ids) {
  static const bool on = env_on("VMC_LOG_PROMPT_VERBOSE");
  if (!on) return;
  std::string first, last;
  for (size_t i = 0; i < ids.size() && i < 5; ++i) first += std::to_string(ids[i]) + " ";
  for (size_t i = ids.size() > 5 ? ids.size() - 5 : 0; i < ids.size(); ++i) last += std::to_string(ids[i]) + " ";
  auto strip = [](const std::string& x) { return x.substr(std::min(x.find_first_not_of(' '), x.size())); };
  const bool rt = strip(tok.decode(ids, true)) == strip(prompt);  // special tokens (BOS) do not count
  fprintf(stderr, "[PROMPT] %zu tokens first5=[%s] last5=[%s] round-trip=%s text=%s\n", ids.size(), first.c_str(),
          last.c_str(), rt ? "Y" : "N", json::quote(prompt).c_str());
}

// Submits a request (validation errors become 400 responses before any stream starts), then drives
// it to completion: detokenized deltas go through on_delta (which returns false when the client is
// gone). drive() returns false if the request was aborted for a lost client.
struct GenResult {
  std::string text;
  size_t n = 0;
  FinishReason reason = FinishReason::STOP;
};

std::shared_ptr<GenStream> submit(ServeLoop& loop, const GenRequest& g) {
  try {
    return loop.submit(g);
  } catch (const std::invalid_argument& e) {
    throw HttpError(400, e.what());
  } catch (const std::exception& e) {
    throw HttpError(503, e.what());
  }
}

bool drive(ServeLoop& loop, const TextTokenizer& tok, const std::shared_ptr<GenStream>& st, const BodyParams& p,
           int poll_ms, http::Responder& res, GenResult& out,
           const std::function<bool(const std::string&, size_t)>& on_delta) {
  static const bool log_detok = env_on("VMC_LOG_DETOK");
  std::vector<int32_t> ids;
  IncrementalDetokenizer detok(tok, p.stop);
  for (;;) {
    GenEvent ev;
    if (!st->next(ev, poll_ms)) {
      if (res.client_gone()) {
        loop.abort(st->id());
        return false;
      }
      continue;
    }
    out.n += ev.tokens.size();
    if (log_detok) ids.insert(ids.end(), ev.tokens.begin(), ev.tokens.end());
    bool finished = ev.finished;
    FinishReason reason = ev.reason;
    const std::string delta = detok.push(ev.tokens, finished);
    if (detok.stopped()) {  // a stop string ends the request even when its last token also hit a limit
      if (!finished) loop.finish(st->id());
      finished = true;
      reason = FinishReason::STOP;
    }
    if (!delta.empty()) {
      out.text += delta;
      if (on_delta && !on_delta(delta, out.n)) {
        if (!finished) loop.abort(st->id());
        return false;
      }
    }
    if (finished) {
      out.reason = reason == FinishReason::NONE ? FinishReason::STOP : reason;
      if (log_detok) {
        std::string line;
        for (int32_t t : ids) line += "(" + std::to_string(t) + ", " + json::quote(tok.decode({t}, false)) + ") ";
        fprintf(stderr, "[DETOK] request %lld: %s\n", static_cast<long long>(st->id()), line.c_str());
      }
      return true;
    }
  }
}

}  // namespace

OpenAIServer::OpenAIServer(ServeLoop& loop, const TextTokenizer& tok, OpenAIConfig cfg)
    : loop_(loop),
      tok_(tok),
      cfg_(std::move(cfg)),
      bos_text_(tok.bos_id() >= 0 && tok.bos_id() < tok.vocab_size() ? tok.token(tok.bos_id()) : ""),
      eos_text_(!tok.eos_ids().empty() && tok.eos_ids()[0] >= 0 && tok.eos_ids()[0] < tok.vocab_size()
                    ? tok.token(tok.eos_ids()[0])
                    : ""),
      chat_(tok.chat_template(), bos_text_, eos_text_) {
  if (cfg_.system_fingerprint.empty()) cfg_.system_fingerprint = "fp_" + hex_id(10);
}

void OpenAIServer::install(http::Server& srv) {
  using namespace std::placeholders;
  auto wrap = [this](void (OpenAIServer::*fn)(const http::Request&, http::Responder&)) {
    return [this, fn](const http::Request& rq, http::Responder& res) {
      try {
        (this->*fn)(rq, res);
      } catch (const HttpError& e) {
        if (!res.responded()) send_error(res, e.status, e.what(), e.status >= 500 ? "server_error" : "invalid_request_error");
      }
    };
  };
  srv.route("POST", "/v1/chat/completions", wrap(&OpenAIServer::chat));
  srv.route("POST", "/v1/completions", wrap(&OpenAIServer::completions));
  srv.route("GET", "/v1/models", wrap(&OpenAIServer::models));
  srv.route("GET", "/health", wrap(&OpenAIServer::health));
  srv.route("GET", "/version", wrap(&OpenAIServer::version));
  srv.route("POST", "/tokenize", wrap(&OpenAIServer::tokenize));
  srv.route("POST", "/detokenize", wrap(&OpenAIServer::detokenize));
  srv.route("GET", "/metrics", wrap(&OpenAIServer::metrics));
}

void OpenAIServer::chat(const http::Request& rq, http::Responder& res) {
  const Value body = parse_body(rq);
  const Value* msgs = body.get("messages");
  if (!msgs || !msgs->is_array() || msgs->size() == 0) throw HttpError(400, "messages must be a non-empty list");
  BodyParams p = body_params(body, cfg_.default_max_tokens);
  std::vector<ChatMessage> cm;
  for (const Value& m : msgs->as_array()) {
    if (!m.is_object()) throw HttpError(400, "every message must be an object");
    const Value* c = m.get("content");
    cm.push_back({m.get_string("role", "user"), c ? content_text(*c) : ""});
  }
  const std::string prompt = chat_.render(cm, p.add_generation_prompt, p.enable_thinking);
  const bool add_bos = !bos_text_.empty() && prompt.compare(0, bos_text_.size(), bos_text_) != 0;
  p.gen.prompt = tok_.encode(prompt, add_bos ? 1 : 0);
  log_prompt(tok_, prompt, p.gen.prompt);
  const std::string cid = "chatcmpl-" + hex_id(32);
  p.gen.name = cid;
  Value base = Value::object();
  base.set("id", cid).set("created", unix_now()).set("model", cfg_.model_name).set("system_fingerprint",
                                                                                    cfg_.system_fingerprint);
  const size_t n_prompt = p.gen.prompt.size();
  GenResult r;
  const auto st = submit(loop_, p.gen);
  if (!p.stream) {
    if (!drive(loop_, tok_, st, p, cfg_.poll_ms, res, r, nullptr)) return;
    const auto [reasoning, content] = split_reasoning(r.text, p.enable_thinking);
    Value msg = Value::object();
    msg.set("role", "assistant").set("content", p.echo ? prompt + content : content);
    if (!reasoning.empty()) msg.set("reasoning_content", reasoning);
    Value choice = Value::object();
    choice.set("index", 0).set("message", msg).set("finish_reason", finish_str(r.reason));
    Value v = base;
    v.set("object", "chat.completion").set("choices", Value::Array{choice}).set("usage", usage(n_prompt, r.n));
    send_json(res, 200, v);
    return;
  }
  res.begin_stream(200, "text/event-stream");
  Value chunk = base;
  chunk.set("object", "chat.completion.chunk");
  auto send = [&](const Value& delta, const char* finish, size_t n_out = 0) {
    Value choice = Value::object();
    choice.set("index", 0).set("delta", delta).set("finish_reason", finish ? Value(finish) : Value());
    Value v = chunk;
    v.set("choices", Value::Array{choice});
    if (n_out > 0) v.set("usage", usage(n_prompt, n_out));  // stream_options.continuous_usage_stats
    return sse(res, v);
  };
  Value first = Value::object();
  first.set("role", "assistant").set("content", "");
  send(first, nullptr);
  ReasoningStream rs(p.enable_thinking);
  const bool ok = drive(loop_, tok_, st, p, cfg_.poll_ms, res, r, [&](const std::string& d, size_t n_out) {
    const auto [reasoning, content] = rs.feed(d);
    const size_t u = p.running_usage ? n_out : 0;
    bool w = true;
    if (!reasoning.empty()) {
      Value dv = Value::object();
      dv.set("reasoning_content", reasoning);
      w = send(dv, nullptr, u);
    }
    if (w && !content.empty()) {
      Value dv = Value::object();
      dv.set("content", content);
      w = send(dv, nullptr, u);
    }
    return w;
  });
  if (!ok) return;
  send(Value::object(), finish_str(r.reason));
  if (p.include_usage) {
    Value v = chunk;
    v.set("choices", Value::array()).set("usage", usage(n_prompt, r.n));
    sse(res, v);
  }
  res.write("data: [DONE]\n\n");
}

void OpenAIServer::completions(const http::Request& rq, http::Responder& res) {
  const Value body = parse_body(rq);
  BodyParams p = body_params(body, cfg_.default_completion_max_tokens);
  const Value* pr = body.get("prompt");
  std::string prompt_text;
  try {
    if (pr && pr->is_array()) {
      if (pr->size() > 0 && pr->as_array()[0].is_number()) {
        for (const Value& x : pr->as_array()) p.gen.prompt.push_back(static_cast<int32_t>(x.as_int()));
        prompt_text = tok_.decode(p.gen.prompt, false);
      } else {  // several prompt strings form one prompt, one per line (as the reference joins them)
        for (const Value& x : pr->as_array()) prompt_text += (prompt_text.empty() ? "" : "\n") + x.as_string();
        p.gen.prompt = tok_.encode(prompt_text);
      }
    } else {
      prompt_text = pr && !pr->is_null() ? pr->as_string() : "";
      p.gen.prompt = tok_.encode(prompt_text);
    }
  } catch (const std::runtime_error& e) {
    throw HttpError(400, std::string("bad prompt: ") + e.what());
  }
  log_prompt(tok_, prompt_text, p.gen.prompt);
  const std::string id = "cmpl-" + hex_id(32);
  p.gen.name = id;
  Value base = Value::object();
  base.set("id", id).set("created", unix_now()).set("model", cfg_.model_name)
      .set("system_fingerprint", cfg_.system_fingerprint).set("object", "text_completion");
  const size_t n_prompt = p.gen.prompt.size();
  GenResult r;
  auto choice = [](const std::string& text, const char* finish) {
    Value c = Value::object();
    c.set("index", 0).set("text", text).set("logprobs", Value()).set("finish_reason", finish ? Value(finish) : Value());
    return c;
  };
  const auto st = submit(loop_, p.gen);
  if (!p.stream) {
    if (!drive(loop_, tok_, st, p, cfg_.poll_ms, res, r, nullptr)) return;
    Value v = base;
    v.set("choices", Value::Array{choice(p.echo ? prompt_text + r.text : r.text, finish_str(r.reason))})
        .set("usage", usage(n_prompt, r.n));
    send_json(res, 200, v);
    return;
  }
  res.begin_stream(200, "text/event-stream");
  const bool ok = drive(loop_, tok_, st, p, cfg_.poll_ms, res, r, [&](const std::string& d, size_t n_out) {
    Value v = base;
    v.set("choices", Value::Array{choice(d, nullptr)});
    if (p.running_usage) v.set("usage", usage(n_prompt, n_out));
    return sse(res, v);
  });
  if (!ok) return;
  Value v = base;
  v.set("choices", Value::Array{choice("", finish_str(r.reason))});
  sse(res, v);
  if (p.include_usage) {
    Value u = base;
    u.set("choices", Value::array()).set("usage", usage(n_prompt, r.n));
    sse(res, u);
  }
  res.write("data: [DONE]\n\n");
}

void OpenAIServer::models(const http::Request&, http::Responder& res) {
  const int64_t t = unix_now();
  Value perm = Value::object();
  perm.set("id", "modelperm-" + hex_id(24)).set("object", "model_permission").set("created", t)
      .set("allow_create_engine", false).set("allow_sampling", true).set("allow_logprobs", true)
      .set("allow_search_indices", false).set("allow_view", true).set("allow_fine_tuning", false)
      .set("organization", "*").set("group", Value()).set("is_blocking", false);
  Value m = Value::object();
  m.set("id", cfg_.model_name).set("object", "model").set("created", t).set("owned_by", "vm_c")
      .set("root", cfg_.model_name).set("permission", Value::Array{perm});
  Value v = Value::object();
  v.set("object", "list").set("data", Value::Array{m});
  send_json(res, 200, v);
}

void OpenAIServer::health(const http::Request&, http::Responder& res) {
  Value v = Value::object();
  if (loop_.failed()) {
    v.set("status", "error").set("error", loop_.last_error());
    send_json(res, 503, v);
    return;
  }
  v.set("status", "ok");
  send_json(res, 200, v);
}

void OpenAIServer::version(const http::Request&, http::Responder& res) {
  Value v = Value::object();
  v.set("version", cfg_.version);
  send_json(res, 200, v);
}

void OpenAIServer::tokenize(const http::Request& rq, http::Responder& res) {
  const Value body = parse_body(rq);
  // "text" is the reference's field; "content" and "prompt" are accepted as well
  std::string text = body.get_string("text", body.get_string("content", body.get_string("prompt", "")));
  const auto ids = tok_.encode(text, body.get_bool("add_special", false) ? 1 : 0);
  Value arr = Value::array();
  for (int32_t t : ids) arr.push(static_cast<int64_t>(t));
  Value v = Value::object();
  v.set("tokens", arr);
  send_json(res, 200, v);
}

void OpenAIServer::detokenize(const http::Request& rq, http::Responder& res) {
  const Value body = parse_body(rq);
  std::vector<int32_t> ids;
  if (const Value* t = body.get("tokens"); t && t->is_array())
    for (const Value& x : t->as_array()) ids.push_back(static_cast<int32_t>(x.as_int()));
  Value v = Value::object();
  const std::string text = tok_.decode(ids, false);
  v.set("text", text).set("content", text);  // "text" as the reference answers
  send_json(res, 200, v);
}

void OpenAIServer::metrics(const http::Request&, http::Responder& res) {
  const ServeStats s = loop_.stats();
  std::string out;
  auto g = [&](const char* name, double v) {
    char buf[64];
    snprintf(buf, sizeof(buf), "%.6g", v);
    out += std::string("# TYPE vmc_") + name + " gauge\nvmc_" + name + " " + buf + "\n";
  };
  g("steps", static_cast<double>(s.steps));
  g("tokens_scheduled", static_cast<double>(s.tokens_scheduled));
  g("tokens_generated", static_cast<double>(s.tokens_generated));
  g("preemptions", static_cast<double>(s.preemptions));
  g("finished", static_cast<double>(s.finished));
  g("requests", static_cast<double>(s.requests));
  g("aborted", static_cast<double>(s.aborted));
  g("errors", static_cast<double>(s.errors));
  g("p50_ttft_ms", s.p50_ttft_ms);
  g("p50_itl_ms", s.p50_itl_ms);
  g("p99_itl_ms", s.p99_itl_ms);
  g("kv_cache_usage", s.kv_usage);
  g("prefix_cache_queries", static_cast<double>(s.prefix_queries));
  g("prefix_cache_hits", static_cast<double>(s.prefix_hits));
  out += "vmc_num_running " + std::to_string(s.running) + "\nvmc_num_waiting " + std::to_string(s.waiting) + "\n";
  res.send(200, "text/plain; version=0.0.4", out);
}

}  // namespace vmc
