// Minimal JSON document model for the native OpenAI server: parse (RFC 8259, UTF-8, \u escapes with
// surrogate pairs, nesting depth bounded) and serialise (control characters escaped, invalid UTF-8
// replaced by U+FFFD so the output is always valid JSON). Objects keep insertion order; values copy
// deeply. Integers that fit in int64 stay exact (token ids, seeds); other numbers are doubles.
//
// The reference links nlohmann_json for the same purpose (CMakeLists.txt:81-125, used by
// src/server/http_server.cpp); this is a small self-contained replacement.
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace vmc::json {

class ParseError : public std::runtime_error {
 public:
  ParseError(const std::string& what, size_t offset) : std::runtime_error(what), offset_(offset) {}
  size_t offset() const { return offset_; }

 private:
  size_t offset_;
};

class Value {
 public:
  enum class Type { Null, Bool, Int, Double, String, Array, Object };
  using Array = std::vector<Value>;
  using Member = std::pair<std::string, Value>;
  using Object = std::vector<Member>;

  Value() = default;
  Value(std::nullptr_t) {}
  Value(bool b) : t_(Type::Bool), b_(b) {}
  Value(int v) : t_(Type::Int), i_(v) {}
  Value(int64_t v) : t_(Type::Int), i_(v) {}
  Value(double v) : t_(Type::Double), d_(v) {}
  Value(const char* s) : t_(Type::String), s_(s) {}
  Value(std::string s) : t_(Type::String), s_(std::move(s)) {}
  Value(Array a) : t_(Type::Array), a_(std::move(a)) {}
  static Value object() {
    Value v;
    v.t_ = Type::Object;
    return v;
  }
  static Value array() { return Value(Array{}); }

  Type type() const { return t_; }
  bool is_null() const { return t_ == Type::Null; }
  bool is_bool() const { return t_ == Type::Bool; }
  bool is_number() const { return t_ == Type::Int || t_ == Type::Double; }
  bool is_int() const { return t_ == Type::Int; }
  bool is_string() const { return t_ == Type::String; }
  bool is_array() const { return t_ == Type::Array; }
  bool is_object() const { return t_ == Type::Object; }

  bool as_bool() const;
  int64_t as_int() const;     // numbers only (a double must be integral)
  double as_double() const;   // numbers only
  const std::string& as_string() const;
  const Array& as_array() const;
  Array& as_array();
  const Object& as_object() const;

  // Object access. get() returns nullptr for a missing key (or a non-object); operator[] inserts.
  const Value* get(const std::string& key) const;
  Value& operator[](const std::string& key);
  Value& set(const std::string& key, Value v);
  // Array append.
  Value& push(Value v);
  size_t size() const;

  // Convenience lookups with a default for missing or null members (type errors still throw).
  bool get_bool(const std::string& key, bool dflt) const;
  int64_t get_int(const std::string& key, int64_t dflt) const;
  double get_double(const std::string& key, double dflt) const;
  std::string get_string(const std::string& key, const std::string& dflt) const;

 private:
  Type t_ = Type::Null;
  bool b_ = false;
  int64_t i_ = 0;
  double d_ = 0;
  std::string s_;
  Array a_;
  Object o_;
};

Value parse(const std::string& text, int max_depth = 128);
std::string dump(const Value& v);
// A JSON string literal (quotes included) of `s`.
std::string quote(const std::string& s);

}  // namespace vmc::json
