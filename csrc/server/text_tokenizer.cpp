// GGUF text tokenizer and incremental detokenizer (see text_tokenizer.hpp).
#include "text_tokenizer.hpp"

#include <algorithm>
#include <stdexcept>

#include "gguf.hpp"
#include "unicode.hpp"

namespace vmc {

namespace {

const char* const kSpaceMark = "\xE2\x96\x81";  // U+2581, SentencePiece's space

struct Cps {
  std::vector<uint32_t> cp;
  std::vector<size_t> off;  // byte offset of each code point, plus the end
};

Cps decode_cps(const std::string& s) {
  Cps c;
  size_t i = 0;
  while (i < s.size()) {
    c.off.push_back(i);
    c.cp.push_back(uni::next(s, i));
  }
  c.off.push_back(s.size());
  return c;
}

bool is_nl(uint32_t c) { return c == '\r' || c == '\n'; }
bool is_other(uint32_t c) { return !(uni::char_class(c) & (uni::kLetter | uni::kNumber | uni::kSpace)); }

// Length (in code points) of an English contraction ('s 't 're 've 'm 'll 'd) at position i, 0 if none.
size_t contraction(const std::vector<uint32_t>& c, size_t i, bool fold_case) {
  if (c[i] != '\'') return 0;
  auto ch = [&](size_t k) -> uint32_t {
    if (k >= c.size()) return 0;
    uint32_t x = c[k];
    if (fold_case && x >= 'A' && x <= 'Z') x += 'a' - 'A';
    if (fold_case && x == 0x17F) x = 's';  // LATIN SMALL LETTER LONG S case-folds to 's'
    return x;
  };
  const uint32_t a = ch(i + 1), b = ch(i + 2);
  if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
  if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
  return 0;
}

// Shared tail of the expressions: `\s+(?!\S)|\s+` at i (i is whitespace).
size_t trailing_space(const std::vector<uint32_t>& c, size_t i) {
  size_t j = i;
  while (j < c.size() && uni::is_space(c[j])) ++j;
  if (j == c.size()) return j - i;      // runs to the end: nothing non-space follows
  if (j - i >= 2) return j - i - 1;     // leave the last space to prefix the next word
  return 1;                             // `\s+`
}

// 'gpt2': 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
size_t match_gpt2(const std::vector<uint32_t>& c, size_t i) {
  if (size_t n = contraction(c, i, false)) return n;
  const size_t n = c.size();
  const size_t s = (c[i] == ' ' && i + 1 < n) ? i + 1 : i;  // optional leading space
  for (int cls : {uni::kLetter, uni::kNumber}) {
    size_t b = (uni::char_class(c[s]) & cls) ? s : ((uni::char_class(c[i]) & cls) ? i : n);
    if (b < n) {
      size_t j = b;
      while (j < n && (uni::char_class(c[j]) & cls)) ++j;
      return j - i;
    }
  }
  {
    size_t b = is_other(c[s]) ? s : (is_other(c[i]) ? i : n);
    if (b < n) {
      size_t j = b;
      while (j < n && is_other(c[j])) ++j;
      return j - i;
    }
  }
  return trailing_space(c, i);
}

// 'llama-bpe' (digits = 3), 'qwen2' (digits = 1) and 'qwen35' (digits = 1, marks = true: combining
// marks join letters):
// (?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,D}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+
// with \p{L} read as [\p{L}\p{M}] in the word run and [^\s\p{L}\p{M}\p{N}] as "other" when marks.
size_t match_llama3(const std::vector<uint32_t>& c, size_t i, int digits, bool marks) {
  if (size_t n = contraction(c, i, true)) return n;
  const size_t n = c.size();
  const int word = marks ? (uni::kLetter | uni::kMark) : uni::kLetter;
  const auto is_word = [&](uint32_t x) { return (uni::char_class(x) & word) != 0; };
  const auto other = [&](uint32_t x) { return is_other(x) && !(marks && uni::is_mark(x)); };
  // [^\r\n\p{L}\p{N}]?\p{L}+
  {
    size_t b = n;
    if (is_word(c[i])) b = i;
    else if (!is_nl(c[i]) && !uni::is_letter(c[i]) && !uni::is_number(c[i]) && i + 1 < n && is_word(c[i + 1])) b = i + 1;
    if (b < n) {
      size_t j = b;
      while (j < n && is_word(c[j])) ++j;
      return j - i;
    }
  }
  // \p{N}{1,D}
  if (uni::is_number(c[i])) {
    size_t j = i;
    while (j < n && j - i < static_cast<size_t>(digits) && uni::is_number(c[j])) ++j;
    return j - i;
  }
  // ' ?[^\s\p{L}\p{N}]+[\r\n]*'
  {
    size_t b = n;
    if (c[i] == ' ' && i + 1 < n && other(c[i + 1])) b = i + 1;
    else if (other(c[i])) b = i;
    if (b < n) {
      size_t j = b;
      while (j < n && other(c[j])) ++j;
      while (j < n && is_nl(c[j])) ++j;
      return j - i;
    }
  }
  // \s*[\r\n]+ : the whitespace run up to and including its last newline
  {
    size_t j = i, last_nl = n;
    while (j < n && uni::is_space(c[j])) {
      if (is_nl(c[j])) last_nl = j;
      ++j;
    }
    if (last_nl < n) return last_nl + 1 - i;
  }
  return trailing_space(c, i);
}

}  // namespace

std::string TextTokenizer::pre_family(const std::string& pre) {
  // tokenizer.ggml.pre names that use one of the four expressions (GGUF vocabulary convention)
  static const std::pair<const char*, const char*> alias[] = {
      {"llama3", "llama-bpe"}, {"llama-v3", "llama-bpe"}, {"falcon3", "llama-bpe"}, {"falcon-h1", "llama-bpe"},
      {"pixtral", "llama-bpe"}, {"dbrx", "llama-bpe"}, {"smaug-bpe", "llama-bpe"}, {"deepseek-r1-qwen", "qwen2"},
      {"gpt-2", "gpt2"}, {"phi-2", "gpt2"}};
  for (const auto& a : alias)
    if (pre == a.first) return a.second;
  if (pre == "llama-bpe" || pre == "qwen2" || pre == "qwen35") return pre;
  return "gpt2";
}

std::vector<std::string> TextTokenizer::pre_split(const std::string& text, const std::string& family) {
  const Cps c = decode_cps(text);
  std::vector<std::string> out;
  size_t i = 0;
  while (i < c.cp.size()) {
    size_t len;
    if (family == "llama-bpe") len = match_llama3(c.cp, i, 3, false);
    else if (family == "qwen2") len = match_llama3(c.cp, i, 1, false);
    else if (family == "qwen35") len = match_llama3(c.cp, i, 1, true);
    else len = match_gpt2(c.cp, i);
    len = std::max<size_t>(1, len);
    out.emplace_back(text, c.off[i], c.off[i + len] - c.off[i]);
    i += len;
  }
  return out;
}

TextTokenizer::TextTokenizer(std::vector<std::string> tokens, std::vector<float> scores, std::vector<int> types,
                             const std::vector<std::string>& merges, const std::string& model, const std::string& pre,
                             int32_t bos_id, std::vector<int32_t> eos_ids, bool add_bos, bool add_space_prefix,
                             std::string chat_template, int32_t unk_id)
    : tokens_(std::move(tokens)),
      types_(std::move(types)),
      gpt2_(model == "gpt2"),
      pre_(pre),
      bos_(bos_id),
      eos_(std::move(eos_ids)),
      add_bos_(add_bos),
      add_space_prefix_(add_space_prefix),
      chat_template_(std::move(chat_template)) {
  if (tokens_.empty()) throw std::runtime_error("tokenizer: empty vocabulary");
  if (types_.empty()) types_.assign(tokens_.size(), NORMAL);
  if (scores.empty()) scores.assign(tokens_.size(), 0.f);
  core_ = std::make_unique<BpeTokenizer>(tokens_, scores, merges, gpt2_ ? "gpt2" : "llama");
  if (unk_id >= 0) core_->set_unk(unk_id);
  std::unordered_map<std::string, int32_t> sp;
  std::vector<std::string> order;
  for (size_t i = 0; i < tokens_.size(); ++i) {
    const int ty = i < types_.size() ? types_[i] : NORMAL;
    if ((ty == CONTROL || ty == USER) && !tokens_[i].empty()) {
      if (!sp.count(tokens_[i])) order.push_back(tokens_[i]);
      sp[tokens_[i]] = static_cast<int32_t>(i);  // a repeated piece maps to its last id
    }
  }
  std::stable_sort(order.begin(), order.end(), [](const std::string& a, const std::string& b) {
    return uni::length(a) > uni::length(b);
  });
  for (const auto& s : order) {
    by_first_[static_cast<unsigned char>(s[0])].push_back(static_cast<int>(specials_.size()));
    specials_.emplace_back(s, sp[s]);
  }
  // GPT-2's reversible byte <-> printable code point map
  int n = 0;
  for (int b = 0; b < 256; ++b) {
    const bool keep = (b >= '!' && b <= '~') || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    const uint32_t cp = keep ? static_cast<uint32_t>(b) : static_cast<uint32_t>(256 + n++);
    uni::append(byte_to_cp_[b], cp);
    cp_to_byte_[cp] = static_cast<uint8_t>(b);
  }
}

std::unique_ptr<TextTokenizer> TextTokenizer::from_gguf(const GgufFile& f) {
  if (!f.has("tokenizer.ggml.tokens")) throw std::runtime_error("GGUF has no tokenizer.ggml.tokens");
  std::vector<std::string> toks;
  for (const auto& t : f.get("tokenizer.ggml.tokens").as) toks.push_back(uni::sanitize(t));
  std::vector<float> scores;
  if (f.has("tokenizer.ggml.scores"))
    for (double s : f.get("tokenizer.ggml.scores").af) scores.push_back(static_cast<float>(s));
  std::vector<int> types;
  if (f.has("tokenizer.ggml.token_type"))
    for (int64_t t : f.get("tokenizer.ggml.token_type").ai) types.push_back(static_cast<int>(t));
  std::vector<std::string> merges;
  if (f.has("tokenizer.ggml.merges"))
    for (const auto& m : f.get("tokenizer.ggml.merges").as) merges.push_back(uni::sanitize(m));
  std::vector<int32_t> eos = {static_cast<int32_t>(f.get_int("tokenizer.ggml.eos_token_id", 2))};
  if (f.has("tokenizer.ggml.eot_token_id")) {
    const auto eot = static_cast<int32_t>(f.get_int("tokenizer.ggml.eot_token_id", -1));
    if (std::find(eos.begin(), eos.end(), eot) == eos.end()) eos.push_back(eot);
  }
  const auto flag = [&](const char* key, bool dflt) {
    if (!f.has(key)) return dflt;
    const GValue& v = f.get(key);
    return v.type == GValueType::BOOL ? v.b : f.get_int(key, dflt) != 0;
  };
  return std::make_unique<TextTokenizer>(
      std::move(toks), std::move(scores), std::move(types), merges, f.get_str("tokenizer.ggml.model", "llama"),
      f.get_str("tokenizer.ggml.pre", "gpt2"), static_cast<int32_t>(f.get_int("tokenizer.ggml.bos_token_id", 1)),
      std::move(eos), flag("tokenizer.ggml.add_bos_token", true), flag("tokenizer.ggml.add_space_prefix", true),
      f.get_str("tokenizer.chat_template", ""), static_cast<int32_t>(f.get_int("tokenizer.ggml.unknown_token_id", -1)));
}

std::vector<int32_t> TextTokenizer::encode_text(const std::string& text, bool first) const {
  if (text.empty()) return {};
  if (gpt2_) {
    const std::string fam = pre_family(pre_);
    std::vector<int32_t> out;
    for (const std::string& piece : pre_split(text, fam)) {
      std::string mapped;
      for (unsigned char b : piece) mapped += byte_to_cp_[b];
      const auto ids = core_->encode_piece(mapped);
      out.insert(out.end(), ids.begin(), ids.end());
    }
    return out;
  }
  std::string t;
  for (char ch : text) {
    if (ch == ' ') t += kSpaceMark;
    else t += ch;
  }
  if (first && add_space_prefix_ && t.compare(0, 3, kSpaceMark) != 0) t = kSpaceMark + t;
  return core_->encode_piece(t);
}

std::vector<int32_t> TextTokenizer::encode(const std::string& text, int add_bos, bool parse_special) const {
  const bool bos = add_bos < 0 ? add_bos_ : add_bos != 0;
  std::vector<int32_t> out;
  if (bos && bos_ >= 0) out.push_back(bos_);
  bool first = true;
  auto emit_text = [&](size_t b, size_t e) {
    if (e <= b) return;
    const auto ids = encode_text(text.substr(b, e - b), first);
    out.insert(out.end(), ids.begin(), ids.end());
    first = false;
  };
  size_t start = 0;
  if (parse_special && !specials_.empty()) {
    size_t p = 0;
    while (p < text.size()) {
      const std::pair<std::string, int32_t>* hit = nullptr;
      for (int k : by_first_[static_cast<unsigned char>(text[p])]) {
        const auto& s = specials_[k];
        if (text.compare(p, s.first.size(), s.first) == 0) {
          hit = &s;
          break;
        }
      }
      if (!hit) {
        ++p;
        continue;
      }
      emit_text(start, p);
      out.push_back(hit->second);
      first = false;
      p += hit->first.size();
      start = p;
    }
  }
  emit_text(start, text.size());
  return out;
}

std::string TextTokenizer::token_bytes(int32_t id) const {
  if (id < 0 || id >= vocab_size()) return "";
  const std::string& t = tokens_[id];
  const int ty = id < static_cast<int32_t>(types_.size()) ? types_[id] : NORMAL;
  if ((ty == BYTE || uni::length(t) == 6) && t.size() == 6 && t.compare(0, 3, "<0x") == 0 && t[5] == '>') {
    auto hex = [](char c) -> int {
      if (c >= '0' && c <= '9') return c - '0';
      if (c >= 'a' && c <= 'f') return c - 'a' + 10;
      if (c >= 'A' && c <= 'F') return c - 'A' + 10;
      return -1;
    };
    const int hi = hex(t[3]), lo = hex(t[4]);
    if (hi >= 0 && lo >= 0) return std::string(1, static_cast<char>(hi * 16 + lo));
  }
  if (gpt2_) {
    std::string out;
    size_t i = 0;
    while (i < t.size()) {
      const auto it = cp_to_byte_.find(uni::next(t, i));
      if (it == cp_to_byte_.end()) return t;
      out += static_cast<char>(it->second);
    }
    return out;
  }
  return t;
}

std::string TextTokenizer::post(const std::string& text) const {
  if (gpt2_) return text;
  std::string out;
  out.reserve(text.size());
  for (size_t i = 0; i < text.size();) {
    if (text.compare(i, 3, kSpaceMark) == 0) {
      out += ' ';
      i += 3;
    } else {
      out += text[i++];
    }
  }
  return out;
}

bool TextTokenizer::is_special(int32_t id) const {
  if (id < 0 || id >= static_cast<int32_t>(types_.size())) return false;
  return types_[id] == CONTROL || types_[id] == UNUSED;
}

std::string TextTokenizer::decode(const std::vector<int32_t>& ids, bool skip_special) const {
  std::string bytes;
  for (int32_t i : ids)
    if (!(skip_special && is_special(i))) bytes += token_bytes(i);
  return post(uni::sanitize(bytes));
}

IncrementalDetokenizer::IncrementalDetokenizer(const TextTokenizer& tok, std::vector<std::string> stop,
                                               bool skip_special)
    : tok_(tok), skip_special_(skip_special) {
  size_t longest = 1;
  for (auto& s : stop)
    if (!s.empty()) {
      longest = std::max(longest, uni::length(s));
      stop_.push_back(std::move(s));
    }
  hold_ = longest - 1;
}

std::string IncrementalDetokenizer::push(const std::vector<int32_t>& ids, bool final) {
  if (stopped_) return "";
  for (int32_t i : ids)
    if (!(skip_special_ && tok_.is_special(i))) buf_ += tok_.token_bytes(i);
  std::string s;
  buf_.erase(0, uni::decode_stream(buf_, final, s));  // holds only an incomplete trailing sequence
  text_ += tok_.post(s);
  for (const auto& st : stop_) {
    const size_t k = text_.find(st);
    if (k != std::string::npos) {
      std::string out = text_.substr(0, k);
      text_.clear();
      stopped_ = true;
      emitted_ += out;
      return out;
    }
  }
  std::string out;
  if (final || hold_ == 0) {
    out.swap(text_);
  } else {
    const size_t len = uni::length(text_);
    const size_t keep_from = uni::offset_of(text_, len > hold_ ? len - hold_ : 0);
    out = text_.substr(0, keep_from);
    text_.erase(0, keep_from);
  }
  emitted_ += out;
  return out;
}

}  // namespace vmc
