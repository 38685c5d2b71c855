// Native BPE merge core of the GGUF tokenizers (see tokenizer.cpp).
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace vmc {

class BpeTokenizer {
 public:
  // model: "llama" (SentencePiece-style, score-driven merges) or "gpt2" (rank-driven merges).
  BpeTokenizer(const std::vector<std::string>& tokens, const std::vector<float>& scores,
               const std::vector<std::string>& merges, const std::string& model);
  // Tokenise one piece of already normalised / pre-tokenised text.
  std::vector<int32_t> encode_piece(const std::string& text) const;
  int32_t token_id(const std::string& piece) const;
  void set_unk(int32_t id) { unk_ = id; }
  size_t vocab_size() const { return tokens_.size(); }

 private:
  std::vector<std::string> tokens_;
  std::vector<float> scores_;
  bool spm_;
  std::unordered_map<std::string, int32_t> tok_to_id_;
  std::unordered_map<std::string, int> merge_rank_;
  int32_t byte_tok_[256];
  int32_t unk_ = -1;
};

}  // namespace vmc
