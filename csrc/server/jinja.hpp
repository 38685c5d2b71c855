// A Jinja2 template interpreter for chat templates.
//
// The reference renders the checkpoint's `tokenizer.chat_template` with llama.cpp's vendored Jinja
// engine (include/vm_c/tokenizer/jinja_template.hpp:37); the Python server uses jinja2 with
// trim_blocks and lstrip_blocks. This is the subset chat templates use, with jinja2's semantics:
//  * tags {{ }}, {% %}, {# #} with `-` / `+` whitespace control, trim_blocks, lstrip_blocks, the
//    trailing newline of the source dropped;
//  * statements: if / elif / else, for (tuple targets, `loop.*`, an inline `if` filter, else),
//    set (names, namespace attributes, block set), macro with defaults, break / continue;
//  * expressions: literals, lists, dicts, attribute / item / slice access, calls with keyword
//    arguments, the arithmetic, comparison, `in`, `is` test, `~`, logical and conditional
//    operators, filters;
//  * the string, list and dict methods templates call (strip, split, startswith, items, get, ...),
//    namespace(), range(), raise_exception(); common filters and tests.
// Undefined values print as nothing, are false, iterate as empty and propagate through attribute
// and item access. Anything outside the subset raises TemplateError, and the caller falls back to
// ChatML as the reference does when its engine fails.
#pragma once
#include <cstdint>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace vmc::json {
class Value;
}

namespace vmc::jinja {

class TemplateError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};

struct Value;
using List = std::vector<Value>;
using Dict = std::vector<std::pair<std::string, Value>>;
using Args = std::vector<Value>;
using Kwargs = std::vector<std::pair<std::string, Value>>;
using Func = std::function<Value(const Args&, const Kwargs&)>;

// A Python-like value. Lists and dicts are shared by reference, as in Python (a namespace is a dict
// whose attributes can be assigned).
struct Value {
  enum Type { Undefined, None, Bool, Int, Float, Str, ListT, DictT, Callable };
  Type t = Undefined;
  bool b = false;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::shared_ptr<List> l;
  std::shared_ptr<Dict> d;
  std::shared_ptr<Func> fn;
  bool is_namespace = false;
  bool is_tuple = false;   // a list printed as a Python tuple
  bool is_markup = false;  // a string that is jinja2 Markup (tojson, safe, escape results)

  Value() = default;
  static Value none() { Value v; v.t = None; return v; }
  static Value boolean(bool x) { Value v; v.t = Bool; v.b = x; return v; }
  static Value integer(int64_t x) { Value v; v.t = Int; v.i = x; return v; }
  static Value number(double x) { Value v; v.t = Float; v.f = x; return v; }
  static Value str(std::string x) { Value v; v.t = Str; v.s = std::move(x); return v; }
  static Value list(List x = {}) { Value v; v.t = ListT; v.l = std::make_shared<List>(std::move(x)); return v; }
  static Value dict(Dict x = {}) { Value v; v.t = DictT; v.d = std::make_shared<Dict>(std::move(x)); return v; }
  static Value func(Func f) { Value v; v.t = Callable; v.fn = std::make_shared<Func>(std::move(f)); return v; }

  bool truthy() const;
  const Value* get(const std::string& key) const;  // dict member or nullptr
  void set(const std::string& key, Value v);       // dict member (inserted or replaced)
};

// Python str() of a value (what {{ }} prints).
std::string to_str(const Value& v);
Value from_json(const json::Value& v);

class Template {
 public:
  // Parses the source; throws TemplateError on a syntax error or an unsupported construct.
  explicit Template(const std::string& source);
  ~Template();
  Template(Template&&) noexcept;
  Template& operator=(Template&&) noexcept;
  // Renders with `globals` (a dict); throws TemplateError (raise_exception included).
  std::string render(const Value& globals) const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};

}  // namespace vmc::jinja
