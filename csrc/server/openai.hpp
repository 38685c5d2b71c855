// OpenAI-compatible routes of the native server.
//
// Routes and JSON / SSE shapes follow the reference's HttpServer (src/server/http_server.cpp:316-449):
// POST /v1/chat/completions, POST /v1/completions, GET /v1/models, GET /health, GET /version,
// POST /tokenize, POST /detokenize; streaming chunks end with `data: [DONE]`;
// `stream_options.include_usage` adds a usage chunk; reasoning text before `</think>` is returned as
// `reasoning_content`; a request whose client disconnects is aborted. Added: GET /metrics
// (Prometheus text). The same surface as the Python server (vm_c_b200/server/http.py).
#pragma once
#include <string>

#include "chat.hpp"
#include "http.hpp"
#include "serve_loop.hpp"
#include "text_tokenizer.hpp"

namespace vmc {

struct OpenAIConfig {
  std::string model_name = "vm_c";
  int default_max_tokens = 4096;            // chat completions without max_tokens
  int default_completion_max_tokens = 16;   // completions without max_tokens
  std::string system_fingerprint;           // generated when empty
  std::string version = "vm_c_b200 0.1.0 (native)";
  int poll_ms = 50;                         // handlers check their client between waits of this length
};

class OpenAIServer {
 public:
  OpenAIServer(ServeLoop& loop, const TextTokenizer& tok, OpenAIConfig cfg);
  void install(http::Server& srv);
  const ChatTemplate& chat_template() const { return chat_; }

 private:
  void chat(const http::Request& rq, http::Responder& res);
  void completions(const http::Request& rq, http::Responder& res);
  void models(const http::Request& rq, http::Responder& res);
  void health(const http::Request& rq, http::Responder& res);
  void version(const http::Request& rq, http::Responder& res);
  void tokenize(const http::Request& rq, http::Responder& res);
  void detokenize(const http::Request& rq, http::Responder& res);
  void metrics(const http::Request& rq, http::Responder& res);

  ServeLoop& loop_;
  const TextTokenizer& tok_;
  OpenAIConfig cfg_;
  std::string bos_text_, eos_text_;
  ChatTemplate chat_;
};

}  // namespace vmc
