// JSON parser and writer (see json.hpp).
#include "json.hpp"

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>

namespace vmc::json {

namespace {

[[noreturn]] void type_error(const char* want) { throw std::runtime_error(std::string("JSON value is not ") + want); }

void put_utf8(std::string& out, uint32_t cp) {
  if (cp < 0x80) {
    out += static_cast<char>(cp);
  } else if (cp < 0x800) {
    out += static_cast<char>(0xC0 | (cp >> 6));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    out += static_cast<char>(0xE0 | (cp >> 12));
    out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  } else {
    out += static_cast<char>(0xF0 | (cp >> 18));
    out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
    out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
    out += static_cast<char>(0x80 | (cp & 0x3F));
  }
}

// Length of the well-formed UTF-8 sequence at s[i] (1-4), or 0 if it is not well formed
// (overlong forms, surrogates and code points above U+10FFFF are rejected).
size_t utf8_len(const std::string& s, size_t i) {
  const auto b = [&](size_t k) { return static_cast<unsigned char>(s[k]); };
  const unsigned char c = b(i);
  if (c < 0x80) return 1;
  size_t n;
  uint32_t cp;
  if ((c & 0xE0) == 0xC0) {
    n = 2;
    cp = c & 0x1F;
  } else if ((c & 0xF0) == 0xE0) {
    n = 3;
    cp = c & 0x0F;
  } else if ((c & 0xF8) == 0xF0) {
    n = 4;
    cp = c & 0x07;
  } else {
    return 0;
  }
  if (i + n > s.size()) return 0;
  for (size_t k = 1; k < n; ++k) {
    if ((b(i + k) & 0xC0) != 0x80) return 0;
    cp = (cp << 6) | (b(i + k) & 0x3F);
  }
  static const uint32_t min_cp[5] = {0, 0, 0x80, 0x800, 0x10000};
  if (cp < min_cp[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return 0;
  return n;
}

class Parser {
 public:
  Parser(const std::string& s, int max_depth) : s_(s), max_depth_(max_depth) {}

  Value document() {
    ws();
    Value v = value(0);
    ws();
    if (p_ != s_.size()) fail("trailing characters after the JSON value");
    return v;
  }

 private:
  [[noreturn]] void fail(const std::string& msg) const {
    throw ParseError("invalid JSON at offset " + std::to_string(p_) + ": " + msg, p_);
  }
  void ws() {
    while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\t' || s_[p_] == '\n' || s_[p_] == '\r')) ++p_;
  }
  char peek() const { return p_ < s_.size() ? s_[p_] : '\0'; }
  void expect(char c) {
    if (peek() != c) fail(std::string("expected '") + c + "'");
    ++p_;
  }
  void literal(const char* w) {
    const size_t n = strlen(w);
    if (s_.compare(p_, n, w) != 0) fail(std::string("expected ") + w);
    p_ += n;
  }

  Value value(int depth) {
    if (depth > max_depth_) fail("nesting deeper than " + std::to_string(max_depth_));
    switch (peek()) {
      case '{': return object(depth);
      case '[': return array(depth);
      case '"': return Value(string());
      case 't': literal("true"); return Value(true);
      case 'f': literal("false"); return Value(false);
      case 'n': literal("null"); return Value();
      default: return number();
    }
  }

  Value object(int depth) {
    expect('{');
    Value v = Value::object();
    ws();
    if (peek() == '}') {
      ++p_;
      return v;
    }
    for (;;) {
      ws();
      if (peek() != '"') fail("expected a member name");
      std::string k = string();
      ws();
      expect(':');
      ws();
      v.set(k, value(depth + 1));
      ws();
      if (peek() == ',') {
        ++p_;
        continue;
      }
      expect('}');
      return v;
    }
  }

  Value array(int depth) {
    expect('[');
    Value v = Value::array();
    ws();
    if (peek() == ']') {
      ++p_;
      return v;
    }
    for (;;) {
      ws();
      v.push(value(depth + 1));
      ws();
      if (peek() == ',') {
        ++p_;
        continue;
      }
      expect(']');
      return v;
    }
  }

  uint32_t hex4() {
    if (p_ + 4 > s_.size()) fail("truncated \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = s_[p_++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= c - '0';
      else if (c >= 'a' && c <= 'f') v |= c - 'a' + 10;
      else if (c >= 'A' && c <= 'F') v |= c - 'A' + 10;
      else fail("bad hex digit in \\u escape");
    }
    return v;
  }

  std::string string() {
    expect('"');
    std::string out;
    for (;;) {
      if (p_ >= s_.size()) fail("unterminated string");
      const unsigned char c = static_cast<unsigned char>(s_[p_]);
      if (c == '"') {
        ++p_;
        return out;
      }
      if (c < 0x20) fail("control character in string");
      if (c == '\\') {
        ++p_;
        if (p_ >= s_.size()) fail("unterminated escape");
        const char e = s_[p_++];
        switch (e) {
          case '"': out += '"'; break;
          case '\\': out += '\\'; break;
          case '/': out += '/'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'n': out += '\n'; break;
          case 'r': out += '\r'; break;
          case 't': out += '\t'; break;
          case 'u': {
            uint32_t cp = hex4();
            if (cp >= 0xD800 && cp <= 0xDBFF) {  // high surrogate: a low one must follow
              if (p_ + 6 <= s_.size() && s_[p_] == '\\' && s_[p_ + 1] == 'u') {
                const size_t save = p_;
                p_ += 2;
                const uint32_t lo = hex4();
                if (lo >= 0xDC00 && lo <= 0xDFFF) {
                  cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                } else {
                  p_ = save;
                  cp = 0xFFFD;
                }
              } else {
                cp = 0xFFFD;
              }
            } else if (cp >= 0xDC00 && cp <= 0xDFFF) {
              cp = 0xFFFD;  // lone low surrogate
            }
            put_utf8(out, cp);
            break;
          }
          default: fail("unknown escape");
        }
        continue;
      }
      const size_t n = utf8_len(s_, p_);
      if (n == 0) fail("invalid UTF-8 in string");
      out.append(s_, p_, n);
      p_ += n;
    }
  }

  Value number() {
    const size_t b = p_;
    if (peek() == '-') ++p_;
    if (peek() == '0') {
      ++p_;
    } else if (peek() >= '1' && peek() <= '9') {
      while (peek() >= '0' && peek() <= '9') ++p_;
    } else {
      fail("unexpected character");
    }
    bool integral = true;
    if (peek() == '.') {
      integral = false;
      ++p_;
      if (!(peek() >= '0' && peek() <= '9')) fail("digit expected after '.'");
      while (peek() >= '0' && peek() <= '9') ++p_;
    }
    if (peek() == 'e' || peek() == 'E') {
      integral = false;
      ++p_;
      if (peek() == '+' || peek() == '-') ++p_;
      if (!(peek() >= '0' && peek() <= '9')) fail("digit expected in exponent");
      while (peek() >= '0' && peek() <= '9') ++p_;
    }
    const std::string tok = s_.substr(b, p_ - b);
    if (integral) {
      errno = 0;
      char* end = nullptr;
      const long long v = strtoll(tok.c_str(), &end, 10);
      if (errno == 0 && end && *end == '\0') return Value(static_cast<int64_t>(v));
    }
    return Value(strtod(tok.c_str(), nullptr));
  }

  const std::string& s_;
  size_t p_ = 0;
  int max_depth_;
};

void dump_string(std::string& out, const std::string& s) {
  out += '"';
  size_t i = 0;
  while (i < s.size()) {
    const unsigned char c = static_cast<unsigned char>(s[i]);
    if (c == '"') {
      out += "\\\"";
    } else if (c == '\\') {
      out += "\\\\";
    } else if (c == '\n') {
      out += "\\n";
    } else if (c == '\r') {
      out += "\\r";
    } else if (c == '\t') {
      out += "\\t";
    } else if (c < 0x20 || c == 0x7F) {
      char buf[8];
      snprintf(buf, sizeof(buf), "\\u%04x", c);
      out += buf;
    } else if (c < 0x80) {
      out += static_cast<char>(c);
    } else {
      const size_t n = utf8_len(s, i);
      if (n == 0) {
        out += "\xEF\xBF\xBD";  // U+FFFD for a byte that does not start a well-formed sequence
        ++i;
        continue;
      }
      out.append(s, i, n);
      i += n;
      continue;
    }
    ++i;
  }
  out += '"';
}

void dump_value(std::string& out, const Value& v) {
  switch (v.type()) {
    case Value::Type::Null: out += "null"; break;
    case Value::Type::Bool: out += v.as_bool() ? "true" : "false"; break;
    case Value::Type::Int: out += std::to_string(v.as_int()); break;
    case Value::Type::Double: {
      const double d = v.as_double();
      if (!std::isfinite(d)) {
        out += "null";  // JSON has no NaN / infinity
      } else {
        char buf[32];
        snprintf(buf, sizeof(buf), "%.17g", d);
        // keep the value a JSON number that reads back as a double
        out += buf;
      }
      break;
    }
    case Value::Type::String: dump_string(out, v.as_string()); break;
    case Value::Type::Array: {
      out += '[';
      bool first = true;
      for (const Value& e : v.as_array()) {
        if (!first) out += ", ";
        first = false;
        dump_value(out, e);
      }
      out += ']';
      break;
    }
    case Value::Type::Object: {
      out += '{';
      bool first = true;
      for (const auto& m : v.as_object()) {
        if (!first) out += ", ";
        first = false;
        dump_string(out, m.first);
        out += ": ";
        dump_value(out, m.second);
      }
      out += '}';
      break;
    }
  }
}

}  // namespace

bool Value::as_bool() const {
  if (t_ != Type::Bool) type_error("a boolean");
  return b_;
}

int64_t Value::as_int() const {
  if (t_ == Type::Int) return i_;
  if (t_ == Type::Double && std::floor(d_) == d_ && std::fabs(d_) < 9.2e18) return static_cast<int64_t>(d_);
  type_error("an integer");
}

double Value::as_double() const {
  if (t_ == Type::Int) return static_cast<double>(i_);
  if (t_ == Type::Double) return d_;
  type_error("a number");
}

const std::string& Value::as_string() const {
  if (t_ != Type::String) type_error("a string");
  return s_;
}

const Value::Array& Value::as_array() const {
  if (t_ != Type::Array) type_error("an array");
  return a_;
}

Value::Array& Value::as_array() {
  if (t_ != Type::Array) type_error("an array");
  return a_;
}

const Value::Object& Value::as_object() const {
  if (t_ != Type::Object) type_error("an object");
  return o_;
}

const Value* Value::get(const std::string& key) const {
  if (t_ != Type::Object) return nullptr;
  for (const auto& m : o_)
    if (m.first == key) return &m.second;
  return nullptr;
}

Value& Value::operator[](const std::string& key) {
  if (t_ == Type::Null) t_ = Type::Object;
  if (t_ != Type::Object) type_error("an object");
  for (auto& m : o_)
    if (m.first == key) return m.second;
  o_.emplace_back(key, Value());
  return o_.back().second;
}

Value& Value::set(const std::string& key, Value v) {
  Value& slot = (*this)[key];
  slot = std::move(v);
  return *this;
}

Value& Value::push(Value v) {
  if (t_ == Type::Null) t_ = Type::Array;
  if (t_ != Type::Array) type_error("an array");
  a_.push_back(std::move(v));
  return *this;
}

size_t Value::size() const {
  if (t_ == Type::Array) return a_.size();
  if (t_ == Type::Object) return o_.size();
  if (t_ == Type::String) return s_.size();
  return 0;
}

bool Value::get_bool(const std::string& key, bool dflt) const {
  const Value* v = get(key);
  return v && !v->is_null() ? v->as_bool() : dflt;
}

int64_t Value::get_int(const std::string& key, int64_t dflt) const {
  const Value* v = get(key);
  return v && !v->is_null() ? v->as_int() : dflt;
}

double Value::get_double(const std::string& key, double dflt) const {
  const Value* v = get(key);
  return v && !v->is_null() ? v->as_double() : dflt;
}

std::string Value::get_string(const std::string& key, const std::string& dflt) const {
  const Value* v = get(key);
  return v && !v->is_null() ? v->as_string() : dflt;
}

Value parse(const std::string& text, int max_depth) { return Parser(text, max_depth).document(); }

std::string dump(const Value& v) {
  std::string out;
  dump_value(out, v);
  return out;
}

std::string quote(const std::string& s) {
  std::string out;
  dump_string(out, s);
  return out;
}

}  // namespace vmc::json
