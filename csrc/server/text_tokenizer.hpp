// Text tokenizer of a GGUF vocabulary, incremental detokenizer with stop strings.
//
// Same behaviour as the Python server's tokenizer (vm_c_b200/server/tokenizer.py) and the reference's
// stack it stands for: GgufTokenizer (src/tokenizer/gguf_tokenizer.cpp:39, GPT-2 byte-level BPE), the
// llama_vocab tokenizer it is replaced by at run time (src/main.cpp:15-73, 496-513; SentencePiece-BPE
// with byte fallback) and the incremental detokenizer
// (include/vm_c/tokenizer/incremental_detokenizer.hpp:11-55). The merge loops are the shared native
// core (csrc/host/tokenizer.cpp); the pre-tokenisers of the "gpt2", "llama-bpe", "qwen2" and "qwen35"
// vocabulary families are written as scanners that split text exactly as the published regular
// expressions do.
#pragma once
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "tokenizer.hpp"

namespace vmc {

class GgufFile;

class TextTokenizer {
 public:
  enum TokenType : int { NORMAL = 1, UNKNOWN = 2, CONTROL = 3, USER = 4, UNUSED = 5, BYTE = 6 };

  TextTokenizer(std::vector<std::string> tokens, std::vector<float> scores, std::vector<int> types,
                const std::vector<std::string>& merges, const std::string& model, const std::string& pre,
                int32_t bos_id, std::vector<int32_t> eos_ids, bool add_bos, bool add_space_prefix = true,
                std::string chat_template = "", int32_t unk_id = -1);
  static std::unique_ptr<TextTokenizer> from_gguf(const GgufFile& f);

  // add_bos: -1 uses the vocabulary's default.
  std::vector<int32_t> encode(const std::string& text, int add_bos = -1, bool parse_special = true) const;
  std::string decode(const std::vector<int32_t>& ids, bool skip_special = true) const;
  // Raw bytes of one token (byte tokens and GPT-2 byte mapping undone).
  std::string token_bytes(int32_t id) const;
  // SentencePiece vocabularies mark spaces with U+2581; decoded text gets plain spaces back.
  std::string post(const std::string& text) const;
  bool is_special(int32_t id) const;

  int32_t vocab_size() const { return static_cast<int32_t>(tokens_.size()); }
  const std::string& token(int32_t id) const { return tokens_.at(id); }
  int32_t bos_id() const { return bos_; }
  const std::vector<int32_t>& eos_ids() const { return eos_; }
  bool add_bos() const { return add_bos_; }
  const std::string& chat_template() const { return chat_template_; }
  bool byte_level() const { return gpt2_; }

  // The pre-tokeniser alone: the pieces one family's expression splits `text` into.
  static std::vector<std::string> pre_split(const std::string& text, const std::string& family);
  // The expression family ("gpt2", "llama-bpe", "qwen2", "qwen35") of a tokenizer.ggml.pre name.
  static std::string pre_family(const std::string& pre);

 private:
  std::vector<int32_t> encode_text(const std::string& text, bool first) const;

  std::vector<std::string> tokens_;
  std::vector<int> types_;
  bool gpt2_;
  std::string pre_;
  int32_t bos_;
  std::vector<int32_t> eos_;
  bool add_bos_, add_space_prefix_;
  std::string chat_template_;
  std::unique_ptr<BpeTokenizer> core_;
  std::vector<std::pair<std::string, int32_t>> specials_;  // longest first
  std::vector<int> by_first_[256];                         // specials_ indices by first byte
  std::string byte_to_cp_[256];                                 // GPT-2 byte -> printable code point
  std::unordered_map<uint32_t, uint8_t> cp_to_byte_;
};

// Streams text deltas for generated tokens; holds back the bytes of an incomplete trailing UTF-8
// sequence (ill-formed bytes are replaced by U+FFFD at once) and text that may be the start of a stop
// string.
class IncrementalDetokenizer {
 public:
  IncrementalDetokenizer(const TextTokenizer& tok, std::vector<std::string> stop, bool skip_special = true);
  // Appends tokens, returns the text that can be emitted now.
  std::string push(const std::vector<int32_t>& ids, bool final = false);
  bool stopped() const { return stopped_; }
  const std::string& emitted() const { return emitted_; }

 private:
  const TextTokenizer& tok_;
  std::vector<std::string> stop_;
  bool skip_special_;
  std::string buf_, text_, emitted_;
  bool stopped_ = false;
  size_t hold_ = 0;  // code points
};

}  // namespace vmc
