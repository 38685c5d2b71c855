// Native BPE cores of the GGUF tokenizers.
//
// Two merge procedures over the vocabulary stored in a GGUF file (tokenizer.ggml.*):
//  * "llama" (SentencePiece BPE): start from UTF-8 characters; repeatedly merge the adjacent pair
//    whose concatenation is a vocabulary token with the highest score; characters that never
//    become tokens fall back to the <0xXX> byte tokens.
//  * "gpt2" (byte-level BPE): start from the characters of one pre-tokenised word (already mapped
//    bytes -> printable code points); repeatedly merge the adjacent pair with the lowest merge
//    rank.
// Same capability as the reference's GgufTokenizer (src/tokenizer/gguf_tokenizer.cpp:39) and the
// llama_vocab tokenizer it is replaced by at run time (src/main.cpp:496-513). Both loops use a
// priority queue over candidate pairs with lazy invalidation (O(n log n) per word).
#include "tokenizer.hpp"

#include <queue>
#include <stdexcept>

namespace vmc {

namespace {

// Split a UTF-8 string into code-point substrings (invalid bytes become single-byte symbols).
std::vector<std::string> utf8_chars(const std::string& s) {
  std::vector<std::string> out;
  size_t i = 0;
  while (i < s.size()) {
    unsigned char c = static_cast<unsigned char>(s[i]);
    size_t n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 1;
    if (i + n > s.size()) n = 1;
    out.emplace_back(s.substr(i, n));
    i += n;
  }
  return out;
}

struct Sym {
  int prev, next;
  std::string text;
  bool alive;
};

struct Cand {
  double prio;  // larger = merge first
  int left;     // index of the left symbol
  size_t len_l, len_r;
  bool operator<(const Cand& o) const {
    if (prio != o.prio) return prio < o.prio;
    return left > o.left;  // ties: leftmost first
  }
};

}  // namespace

BpeTokenizer::BpeTokenizer(const std::vector<std::string>& tokens, const std::vector<float>& scores,
                           const std::vector<std::string>& merges, const std::string& model)
    : tokens_(tokens), scores_(scores), spm_(model != "gpt2") {
  for (size_t i = 0; i < tokens_.size(); ++i) tok_to_id_.emplace(tokens_[i], static_cast<int32_t>(i));
  for (size_t r = 0; r < merges.size(); ++r) {
    const auto& m = merges[r];
    size_t sp = m.find(' ', 1);
    if (sp == std::string::npos) continue;
    merge_rank_.emplace(m.substr(0, sp) + '\x01' + m.substr(sp + 1), static_cast<int>(r));
  }
  for (int b = 0; b < 256; ++b) {
    char buf[8];
    snprintf(buf, sizeof(buf), "<0x%02X>", b);
    auto it = tok_to_id_.find(buf);
    byte_tok_[b] = it == tok_to_id_.end() ? -1 : it->second;
  }
}

int32_t BpeTokenizer::token_id(const std::string& piece) const {
  auto it = tok_to_id_.find(piece);
  return it == tok_to_id_.end() ? -1 : it->second;
}

std::vector<int32_t> BpeTokenizer::encode_piece(const std::string& text) const {
  std::vector<int32_t> out;
  if (text.empty()) return out;
  auto chars = utf8_chars(text);
  std::vector<Sym> syms(chars.size());
  for (size_t i = 0; i < chars.size(); ++i) {
    syms[i] = {static_cast<int>(i) - 1, i + 1 < chars.size() ? static_cast<int>(i + 1) : -1, chars[i], true};
  }
  std::priority_queue<Cand> pq;
  auto try_add = [&](int l) {
    if (l < 0) return;
    int r = syms[l].next;
    if (r < 0) return;
    if (spm_) {
      auto it = tok_to_id_.find(syms[l].text + syms[r].text);
      if (it == tok_to_id_.end()) return;
      double sc = it->second < static_cast<int32_t>(scores_.size()) ? scores_[it->second] : 0.0;
      pq.push({sc, l, syms[l].text.size(), syms[r].text.size()});
    } else {
      auto it = merge_rank_.find(syms[l].text + '\x01' + syms[r].text);
      if (it == merge_rank_.end()) return;
      pq.push({-static_cast<double>(it->second), l, syms[l].text.size(), syms[r].text.size()});
    }
  };
  for (size_t i = 0; i + 1 < syms.size(); ++i) try_add(static_cast<int>(i));
  while (!pq.empty()) {
    Cand c = pq.top();
    pq.pop();
    Sym& L = syms[c.left];
    if (!L.alive || L.next < 0) continue;
    Sym& R = syms[L.next];
    if (L.text.size() != c.len_l || R.text.size() != c.len_r) continue;  // stale candidate
    L.text += R.text;
    R.alive = false;
    L.next = R.next;
    if (R.next >= 0) syms[R.next].prev = c.left;
    try_add(L.prev);
    try_add(c.left);
  }
  for (int i = 0; i >= 0 && i < static_cast<int>(syms.size()); i = syms[i].next) {
    const Sym& s = syms[i];
    auto it = tok_to_id_.find(s.text);
    if (it != tok_to_id_.end()) {
      out.push_back(it->second);
    } else {
      for (unsigned char b : s.text) {
        if (byte_tok_[b] >= 0) out.push_back(byte_tok_[b]);
        else if (unk_ >= 0) out.push_back(unk_);
      }
    }
  }
  return out;
}

}  // namespace vmc
