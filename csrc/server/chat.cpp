// Chat prompt formats and reasoning split (see chat.hpp).
#include "chat.hpp"

namespace vmc {

namespace {

const std::string kThinkEnd = "</think>";

std::string lstrip_newlines(const std::string& s) {
  size_t i = 0;
  while (i < s.size() && (s[i] == '\r' || s[i] == '\n')) ++i;
  return s.substr(i);
}

std::string trim(const std::string& s) {
  const char* ws = " \t\r\n\v\f";
  const size_t b = s.find_first_not_of(ws);
  if (b == std::string::npos) return "";
  const size_t e = s.find_last_not_of(ws);
  return s.substr(b, e - b + 1);
}

bool chatml_role(const std::string& r) { return r == "system" || r == "user" || r == "assistant" || r == "tool"; }

}  // namespace

ChatFormat detect_chat_format(const std::string& t) {
  if (t.find("<|start_header_id|>") != std::string::npos) return ChatFormat::Llama3;
  if (t.find("<|im_start|>") != std::string::npos)
    return t.find("enable_thinking") != std::string::npos ? ChatFormat::Qwen3 : ChatFormat::ChatML;
  if (t.find("[INST]") != std::string::npos) return ChatFormat::Mistral;
  return ChatFormat::ChatML;
}

const char* chat_format_name(ChatFormat f) {
  switch (f) {
    case ChatFormat::Qwen3: return "qwen3";
    case ChatFormat::Llama3: return "llama3";
    case ChatFormat::Mistral: return "mistral";
    default: return "chatml";
  }
}

std::string render_chat(ChatFormat f, const std::vector<ChatMessage>& msgs, bool add_generation_prompt,
                        bool enable_thinking, const std::string& bos, const std::string& eos) {
  std::string out;
  switch (f) {
    case ChatFormat::ChatML:
      for (const auto& m : msgs)
        if (chatml_role(m.role)) out += "<|im_start|>" + m.role + "\n" + m.content + "<|im_end|>\n";
      if (add_generation_prompt) {
        out += "<|im_start|>assistant\n";
        out += enable_thinking ? "<think>\n" : "<think>\n\n</think>\n\n";
      }
      break;
    case ChatFormat::Qwen3: {
      // earlier assistant turns (before the last user message) lose their reasoning block
      size_t last_user = msgs.size();
      for (size_t i = 0; i < msgs.size(); ++i)
        if (msgs[i].role == "user") last_user = i;
      for (size_t i = 0; i < msgs.size(); ++i) {
        const auto& m = msgs[i];
        if (!chatml_role(m.role)) continue;
        std::string c = m.content;
        if (m.role == "assistant" && (last_user == msgs.size() || i < last_user)) {
          const size_t k = c.rfind(kThinkEnd);
          if (k != std::string::npos) c = lstrip_newlines(c.substr(k + kThinkEnd.size()));
        }
        out += "<|im_start|>" + m.role + "\n" + c + "<|im_end|>\n";
      }
      if (add_generation_prompt) {
        out += "<|im_start|>assistant\n";
        if (!enable_thinking) out += "<think>\n\n</think>\n\n";
      }
      break;
    }
    case ChatFormat::Llama3:
      for (size_t i = 0; i < msgs.size(); ++i) {
        if (i == 0) out += bos;
        out += "<|start_header_id|>" + msgs[i].role + "<|end_header_id|>\n\n" + trim(msgs[i].content) + "<|eot_id|>";
      }
      if (add_generation_prompt) out += "<|start_header_id|>assistant<|end_header_id|>\n\n";
      break;
    case ChatFormat::Mistral: {
      out += bos;
      std::string system;
      for (const auto& m : msgs) {
        if (m.role == "system") {
          system += (system.empty() ? "" : "\n\n") + m.content;
        } else if (m.role == "user") {
          out += "[INST] " + (system.empty() ? "" : system + "\n\n") + m.content + " [/INST]";
          system.clear();
        } else if (m.role == "assistant") {
          out += m.content + eos;
        }
      }
      break;
    }
  }
  return out;
}

std::pair<std::string, std::string> split_reasoning(const std::string& text, bool enable_thinking) {
  if (!enable_thinking) return {"", text};
  const size_t k = text.find(kThinkEnd);
  if (k == std::string::npos) return {"", text};
  return {text.substr(0, k), lstrip_newlines(text.substr(k + kThinkEnd.size()))};
}

std::pair<std::string, std::string> ReasoningStream::feed(const std::string& delta_in) {
  if (!in_reasoning_) {
    std::string delta = delta_in;
    if (after_end_) {
      delta = lstrip_newlines(delta);
      if (!delta.empty()) after_end_ = false;
    }
    return {"", delta};
  }
  pending_ += delta_in;
  const size_t k = pending_.find(kThinkEnd);
  if (k != std::string::npos) {
    std::string reasoning = pending_.substr(0, k);
    std::string rest = lstrip_newlines(pending_.substr(k + kThinkEnd.size()));
    pending_.clear();
    in_reasoning_ = false;
    after_end_ = rest.empty();
    return {reasoning, rest};
  }
  // keep a possible partial "</think>" at the end
  size_t keep = 0;
  for (size_t n = 1; n < kThinkEnd.size(); ++n)
    if (pending_.size() >= n && pending_.compare(pending_.size() - n, n, kThinkEnd, 0, n) == 0) keep = n;
  std::string out = pending_.substr(0, pending_.size() - keep);
  pending_.erase(0, pending_.size() - keep);
  return {out, ""};
}

}  // namespace vmc
