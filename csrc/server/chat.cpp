// Chat prompt formats and reasoning split (see chat.hpp).
#include "chat.hpp"

#include "jinja.hpp"

namespace vmc {

namespace {

const std::string kThinkEnd = "</think>";

std::string lstrip_newlines(const std::string& s) {
  size_t i = 0;
  while (i < s.size() && (s[i] == '\r' || s[i] == '\n')) ++i;
  return s.substr(i);
}

bool chatml_role(const std::string& r) { return r == "system" || r == "user" || r == "assistant" || r == "tool"; }

}  // namespace

std::string chatml(const std::vector<ChatMessage>& msgs, bool add_generation_prompt, bool enable_thinking) {
  std::string out;
  for (const auto& m : msgs)
    if (chatml_role(m.role)) out += "<|im_start|>" + m.role + "\n" + m.content + "<|im_end|>\n";
  if (add_generation_prompt) {
    out += "<|im_start|>assistant\n";
    out += enable_thinking ? "<think>\n" : "<think>\n\n</think>\n\n";
  }
  return out;
}

ChatTemplate::ChatTemplate(const std::string& src, std::string bos, std::string eos)
    : bos_(std::move(bos)), eos_(std::move(eos)) {
  if (src.empty()) return;
  try {
    tmpl_ = std::make_unique<jinja::Template>(src);
  } catch (const std::exception& e) {
    error_ = e.what();
  }
}

ChatTemplate::~ChatTemplate() = default;

std::string ChatTemplate::render(const std::vector<ChatMessage>& msgs, bool add_generation_prompt,
                                 bool enable_thinking, std::string* why) const {
  if (why) *why = tmpl_ ? "" : error_;
  if (tmpl_) {
    try {
      jinja::List ml;
      for (const auto& m : msgs)
        ml.push_back(jinja::Value::dict({{"role", jinja::Value::str(m.role)}, {"content", jinja::Value::str(m.content)}}));
      jinja::Value g = jinja::Value::dict();
      g.set("messages", jinja::Value::list(std::move(ml)));
      g.set("add_generation_prompt", jinja::Value::boolean(add_generation_prompt));
      g.set("enable_thinking", jinja::Value::boolean(enable_thinking));
      g.set("bos_token", jinja::Value::str(bos_));
      g.set("eos_token", jinja::Value::str(eos_));
      std::string s = tmpl_->render(g);
      if (!s.empty()) return s;
      if (why) *why = "the template rendered nothing";
    } catch (const std::exception& e) {  // raise_exception or an unsupported construct: ChatML
      if (why) *why = e.what();
    }
  }
  return chatml(msgs, add_generation_prompt, enable_thinking);
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
