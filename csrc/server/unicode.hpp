// UTF-8 helpers and the Unicode character classes the pre-tokenisers need.
//
// Classes (letter = general category L*, number = N*, mark = M*, space = the `\s` class of Unicode
// regular expressions) come from a range table that the build generates from the Python `regex` module the
// Python tokenizer uses, so both tokenizers split text identically.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace vmc::uni {

enum : int { kLetter = 1, kNumber = 2, kSpace = 4, kMark = 8 };

// Class bits of code point `cp` (0 for "other").
int char_class(uint32_t cp);
inline bool is_letter(uint32_t cp) { return char_class(cp) & kLetter; }
inline bool is_number(uint32_t cp) { return char_class(cp) & kNumber; }
inline bool is_space(uint32_t cp) { return char_class(cp) & kSpace; }
inline bool is_mark(uint32_t cp) { return char_class(cp) & kMark; }

// Decodes the code point at s[i] and advances i. A byte that does not start a well-formed
// sequence decodes as U+FFFD and advances by one.
uint32_t next(const std::string& s, size_t& i);
void append(std::string& out, uint32_t cp);
// Number of code points of well-formed UTF-8 text.
size_t length(const std::string& s);
// Byte offset of the first `n` code points of well-formed UTF-8 text (s.size() if shorter).
size_t offset_of(const std::string& s, size_t n);

// Length of the longest prefix of `s` that is well-formed UTF-8 (what a strict decoder accepts).
size_t valid_prefix(const std::string& s);
// Decodes bytes replacing each maximal ill-formed subpart by U+FFFD (the Unicode-recommended
// practice; the same output as Python's bytes.decode("utf-8", "replace")).
std::string sanitize(const std::string& s);
// Streaming form of sanitize(): appends the decoded text of `in` to `out` and returns how many bytes
// were consumed. Unless `final`, an incomplete sequence at the end (one more byte could still
// complete it) is left unconsumed; everything else, ill-formed bytes included, is decoded at once
// (Python's incremental UTF-8 decoder with errors="replace").
size_t decode_stream(const std::string& in, bool final, std::string& out);

}  // namespace vmc::uni
