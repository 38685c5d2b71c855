// Chat prompt construction and the reasoning-content split of the native server.
//
// The reference renders the checkpoint's Jinja chat template with llama.cpp's vendored engine and
// falls back to a ChatML prompt (src/server/http_server.cpp:278-313); the generation prompt opens a
// <think> block when thinking is enabled and inserts an empty one when it is disabled. The split of
// the completion into reasoning_content and content follows src/main.cpp:640-661.
//
// This server renders the prompt formats of the template families it recognises from the
// checkpoint's template text (ChatML with and without Qwen3's thinking switch, Llama 3 header
// blocks, Mistral [INST] blocks) and ChatML otherwise.
#pragma once
#include <string>
#include <utility>
#include <vector>

namespace vmc {

struct ChatMessage {
  std::string role, content;
};

enum class ChatFormat { ChatML, Qwen3, Llama3, Mistral };

ChatFormat detect_chat_format(const std::string& jinja_template);
const char* chat_format_name(ChatFormat f);

std::string render_chat(ChatFormat f, const std::vector<ChatMessage>& messages, bool add_generation_prompt,
                        bool enable_thinking, const std::string& bos_token, const std::string& eos_token);

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
