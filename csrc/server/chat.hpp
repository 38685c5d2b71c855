// Chat prompt construction and the reasoning-content split of the native server.
//
// Same behaviour as the reference's HttpServer::build_chat_prompt (src/server/http_server.cpp:278-313)
// and the Python server (vm_c_b200/server/chat.py): render the checkpoint's Jinja chat template
// (tokenizer.chat_template) with `messages`, `add_generation_prompt`, `enable_thinking`,
// `bos_token`, `eos_token` and `raise_exception`; when there is no template, or it fails to parse or
// render, or renders nothing, build a ChatML prompt whose generation prompt opens a <think> block
// when thinking is enabled and inserts an empty one when it is disabled. The split of the completion
// into reasoning_content and content follows src/main.cpp:640-661.
#pragma once
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace vmc {

namespace jinja {
class Template;
}

struct ChatMessage {
  std::string role, content;
};

std::string chatml(const std::vector<ChatMessage>& messages, bool add_generation_prompt, bool enable_thinking);

class ChatTemplate {
 public:
  // Never throws: a template that does not parse is recorded and ChatML is used.
  ChatTemplate(const std::string& jinja_source, std::string bos_token, std::string eos_token);
  ~ChatTemplate();
  // `why`, when given, receives the reason a template fell back to ChatML (empty if it rendered).
  std::string render(const std::vector<ChatMessage>& messages, bool add_generation_prompt, bool enable_thinking,
                     std::string* why = nullptr) const;
  bool has_template() const { return tmpl_ != nullptr; }
  const std::string& parse_error() const { return error_; }

 private:
  std::unique_ptr<jinja::Template> tmpl_;
  std::string bos_, eos_, error_;
};

// (reasoning_content, content) of a complete completion.
std::pair<std::string, std::string> split_reasoning(const std::string& text, bool enable_thinking);

// Routes streamed deltas to reasoning_content until "</think>" is seen, then to content.
class ReasoningStream {
 public:
  explicit ReasoningStream(bool enable_thinking) : in_reasoning_(enable_thinking) {}
  std::pair<std::string, std::string> feed(const std::string& delta);

 private:
  bool in_reasoning_;
  bool after_end_ = false;
  std::string pending_;
};

}  // namespace vmc
