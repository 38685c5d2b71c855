// Jinja2 chat-template interpreter (see jinja.hpp).
#include "jinja.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "json.hpp"
#include "unicode.hpp"

namespace vmc::jinja {

// ---- values ---------------------------------------------------------------------------------------

bool Value::truthy() const {
  switch (t) {
    case Undefined:
    case None: return false;
    case Bool: return b;
    case Int: return i != 0;
    case Float: return f != 0;
    case Str: return !s.empty();
    case ListT: return !l->empty();
    case DictT: return !d->empty();
    case Callable: return true;
  }
  return false;
}

const Value* Value::get(const std::string& key) const {
  if (t != DictT) return nullptr;
  for (const auto& kv : *d)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

void Value::set(const std::string& key, Value v) {
  for (auto& kv : *d)
    if (kv.first == key) {
      kv.second = std::move(v);
      return;
    }
  d->emplace_back(key, std::move(v));
}

namespace {

[[noreturn]] void fail(const std::string& m) { throw TemplateError(m); }

// Attribute and item access on an undefined value fails, as with jinja2's default Undefined; a missing
// key or attribute of a defined value is undefined.
[[noreturn]] void undefined_access(const std::string& what) { fail("undefined value has no " + what); }

std::string float_repr(double x) {
  if (std::isnan(x)) return "nan";
  if (std::isinf(x)) return x > 0 ? "inf" : "-inf";
  char buf[40];
  for (int p = 1; p <= 17; ++p) {  // shortest representation that reads back exactly
    snprintf(buf, sizeof(buf), "%.*g", p, x);
    if (strtod(buf, nullptr) == x) break;
  }
  std::string s = buf;
  if (s.find_first_of(".en") == std::string::npos) s += ".0";
  return s;
}

std::string str_repr(const std::string& s) {
  const char q = (s.find('\'') != std::string::npos && s.find('"') == std::string::npos) ? '"' : '\'';
  std::string out(1, q);
  for (unsigned char c : s) {
    if (c == '\\') out += "\\\\";
    else if (c == static_cast<unsigned char>(q)) out += std::string("\\") + q;
    else if (c == '\n') out += "\\n";
    else if (c == '\r') out += "\\r";
    else if (c == '\t') out += "\\t";
    else if (c < 0x20 || c == 0x7F) {
      char b[8];
      snprintf(b, sizeof(b), "\\x%02x", c);
      out += b;
    } else {
      out += static_cast<char>(c);
    }
  }
  return out + q;
}

std::string repr(const Value& v) {
  switch (v.t) {
    case Value::Str: return v.is_markup ? "Markup(" + str_repr(v.s) + ")" : str_repr(v.s);
    case Value::ListT: {
      std::string o = v.is_tuple ? "(" : "[";
      for (size_t k = 0; k < v.l->size(); ++k) o += (k ? ", " : "") + repr((*v.l)[k]);
      if (v.is_tuple) return o + (v.l->size() == 1 ? ",)" : ")");
      return o + "]";
    }
    case Value::Undefined: return "Undefined";
    case Value::DictT: {
      std::string o = "{";
      bool first = true;
      for (const auto& kv : *v.d) {
        o += (first ? "" : ", ") + str_repr(kv.first) + ": " + repr(kv.second);
        first = false;
      }
      return o + "}";
    }
    default: return to_str(v);
  }
}

// jinja2's Markup: what tojson, safe and escape return. `markup + str` escapes the str; its repr is
// Markup('...').
Value markup(std::string x) {
  Value v = Value::str(std::move(x));
  v.is_markup = true;
  return v;
}

bool is_num(const Value& v) { return v.t == Value::Int || v.t == Value::Float || v.t == Value::Bool; }
double num(const Value& v) { return v.t == Value::Float ? v.f : static_cast<double>(v.t == Value::Bool ? v.b : v.i); }
int64_t as_int(const Value& v) {
  if (v.t == Value::Int) return v.i;
  if (v.t == Value::Bool) return v.b;
  if (v.t == Value::Float) return static_cast<int64_t>(v.f);
  fail("an integer is required");
}

bool equal(const Value& a, const Value& b) {
  if (is_num(a) && is_num(b)) return num(a) == num(b);
  if (a.t != b.t) return (a.t == Value::Undefined && b.t == Value::Undefined);
  switch (a.t) {
    case Value::Undefined:
    case Value::None: return true;
    case Value::Str: return a.s == b.s;
    case Value::ListT:
      if (a.l->size() != b.l->size()) return false;
      for (size_t k = 0; k < a.l->size(); ++k)
        if (!equal((*a.l)[k], (*b.l)[k])) return false;
      return true;
    case Value::DictT:
      if (a.d->size() != b.d->size()) return false;
      for (const auto& kv : *a.d) {
        const Value* o = b.get(kv.first);
        if (!o || !equal(kv.second, *o)) return false;
      }
      return true;
    default: return a.fn == b.fn;
  }
}

int compare(const Value& a, const Value& b) {
  if (is_num(a) && is_num(b)) {
    const double x = num(a), y = num(b);
    return x < y ? -1 : x > y ? 1 : 0;
  }
  if (a.t == Value::Str && b.t == Value::Str) return a.s < b.s ? -1 : a.s > b.s ? 1 : 0;
  if (a.t == Value::ListT && b.t == Value::ListT) {
    for (size_t k = 0; k < std::min(a.l->size(), b.l->size()); ++k)
      if (int c = compare((*a.l)[k], (*b.l)[k])) return c;
    return a.l->size() < b.l->size() ? -1 : a.l->size() > b.l->size() ? 1 : 0;
  }
  fail("values of these types cannot be ordered");
}

// Code points of a string as one-character strings (string iteration and indexing).
std::vector<std::string> chars(const std::string& s) {
  std::vector<std::string> out;
  size_t i = 0;
  while (i < s.size()) {
    const size_t b = i;
    uni::next(s, i);
    out.emplace_back(s, b, i - b);
  }
  return out;
}

List iterate(const Value& v) {
  switch (v.t) {
    case Value::Undefined: return {};
    case Value::ListT: return *v.l;
    case Value::DictT: {
      List out;
      for (const auto& kv : *v.d) out.push_back(Value::str(kv.first));
      return out;
    }
    case Value::Str: {
      List out;
      for (auto& c : chars(v.s)) out.push_back(Value::str(c));
      return out;
    }
    default: fail("value is not iterable");
  }
}

bool contains(const Value& hay, const Value& needle) {
  if (hay.t == Value::Str) {
    if (needle.t != Value::Str) fail("'in <string>' requires a string");
    return hay.s.find(needle.s) != std::string::npos;
  }
  if (hay.t == Value::DictT) return needle.t == Value::Str && hay.get(needle.s) != nullptr;
  if (hay.t == Value::ListT) {
    for (const Value& x : *hay.l)
      if (equal(x, needle)) return true;
    return false;
  }
  if (hay.t == Value::Undefined) return false;
  fail("argument of type is not iterable");
}

const char* const kWs = " \t\n\r\f\v";

std::string strip_chars(const std::string& s, const std::string& cs, bool left, bool right) {
  size_t b = 0, e = s.size();
  if (left) b = s.find_first_not_of(cs);
  if (b == std::string::npos) return "";
  if (right) e = s.find_last_not_of(cs) + 1;
  return s.substr(b, e - b);
}

std::string ascii_upper(std::string s) {
  for (char& c : s)
    if (c >= 'a' && c <= 'z') c = static_cast<char>(c - 32);
  return s;
}
std::string ascii_lower(std::string s) {
  for (char& c : s)
    if (c >= 'A' && c <= 'Z') c = static_cast<char>(c + 32);
  return s;
}

std::string replace_all(const std::string& s, const std::string& a, const std::string& b, int64_t count = -1) {
  if (a.empty()) return s;
  std::string out;
  size_t p = 0;
  int64_t n = 0;
  while (count < 0 || n < count) {
    const size_t k = s.find(a, p);
    if (k == std::string::npos) break;
    out += s.substr(p, k - p) + b;
    p = k + a.size();
    ++n;
  }
  return out + s.substr(p);
}

// Python's json.dumps with sort_keys=True and jinja2's HTML-safe escaping of < > & '.
void tojson(std::string& o, const Value& v, int indent, int level) {
  auto nl = [&](int lv) {
    if (indent < 0) return;
    o += '\n';
    o.append(static_cast<size_t>(indent * lv), ' ');
  };
  switch (v.t) {
    case Value::Undefined: fail("Object of type Undefined is not JSON serializable");
    case Value::None: o += "null"; return;
    case Value::Bool: o += v.b ? "true" : "false"; return;
    case Value::Int: o += std::to_string(v.i); return;
    case Value::Float: o += float_repr(v.f); return;
    case Value::Str: {
      o += '"';
      size_t i = 0;
      while (i < v.s.size()) {
        const uint32_t c = uni::next(v.s, i);
        char b[16];
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c == '\n') o += "\\n";
        else if (c == '\r') o += "\\r";
        else if (c == '\t') o += "\\t";
        else if (c == '\b') o += "\\b";
        else if (c == '\f') o += "\\f";
        else if (c == '<' || c == '>' || c == '&' || c == '\'' || c < 0x20 || c >= 0x7F) {
          if (c >= 0x10000) {  // ensure_ascii: a surrogate pair
            const uint32_t x = c - 0x10000;
            snprintf(b, sizeof(b), "\\u%04x\\u%04x", 0xD800 + (x >> 10), 0xDC00 + (x & 0x3FF));
          } else {
            snprintf(b, sizeof(b), "\\u%04x", c);
          }
          o += b;
        } else {
          o += static_cast<char>(c);
        }
      }
      o += '"';
      return;
    }
    case Value::ListT: {
      o += '[';
      for (size_t k = 0; k < v.l->size(); ++k) {
        if (k) o += indent < 0 ? ", " : ",";
        nl(level + 1);
        tojson(o, (*v.l)[k], indent, level + 1);
      }
      if (!v.l->empty()) nl(level);
      o += ']';
      return;
    }
    case Value::DictT: {
      std::vector<const std::pair<std::string, Value>*> kv;
      for (const auto& x : *v.d) kv.push_back(&x);
      std::sort(kv.begin(), kv.end(), [](auto* a, auto* b) { return a->first < b->first; });
      o += '{';
      for (size_t k = 0; k < kv.size(); ++k) {
        if (k) o += indent < 0 ? ", " : ",";
        nl(level + 1);
        tojson(o, Value::str(kv[k]->first), indent, level + 1);
        o += ": ";
        tojson(o, kv[k]->second, indent, level + 1);
      }
      if (!kv.empty()) nl(level);
      o += '}';
      return;
    }
    case Value::Callable: fail("a callable is not JSON serialisable");
  }
}

// ---- source chunks ---------------------------------------------------------------------------------

struct Chunk {
  enum Kind { Text, Var, Block } kind;
  std::string s;  // text, or the tag's inner source
  int line;
};

std::vector<Chunk> chunk_source(std::string src) {
  // keep_trailing_newline=False: one trailing newline of the source is dropped
  if (src.size() >= 1 && src.back() == '\n') src.pop_back();
  std::vector<Chunk> out;
  size_t pos = 0;
  bool line_starting = true;
  int line = 1;
  auto count_lines = [&](size_t a, size_t b) {
    for (size_t k = a; k < b && k < src.size(); ++k)
      if (src[k] == '\n') ++line;
  };
  while (pos <= src.size()) {
    size_t idx = std::string::npos;
    for (const char* open : {"{{", "{%", "{#"}) idx = std::min(idx, src.find(open, pos));
    if (idx == std::string::npos) {
      if (pos < src.size()) out.push_back({Chunk::Text, src.substr(pos), line});
      break;
    }
    std::string text = src.substr(pos, idx - pos);
    const char kind = src[idx + 1];
    size_t inner = idx + 2;
    const char sign = inner < src.size() ? src[inner] : '\0';
    if (sign == '-' || sign == '+') ++inner;
    // closing delimiter, skipping string literals inside expression tags
    const std::string close = kind == '{' ? "}}" : kind == '%' ? "%}" : "#}";
    size_t c = inner;
    char quote = 0;
    while (c + 1 < src.size()) {
      const char ch = src[c];
      if (kind != '#') {
        if (quote) {
          if (ch == '\\') {
            c += 2;
            continue;
          }
          if (ch == quote) quote = 0;
          ++c;
          continue;
        }
        if (ch == '\'' || ch == '"') {
          quote = ch;
          ++c;
          continue;
        }
      }
      if (src.compare(c, 2, close) == 0) break;
      ++c;
    }
    if (c + 1 >= src.size()) fail("unclosed tag at line " + std::to_string(line));
    size_t end_inner = c;
    const bool strip_after = end_inner > inner && src[end_inner - 1] == '-';
    const bool keep_after = kind != '{' && !strip_after && end_inner > inner && src[end_inner - 1] == '+';
    if (strip_after || keep_after) --end_inner;
    // whitespace control of the text before the tag
    if (sign == '-') {
      text = strip_chars(text, kWs, false, true);
    } else if (sign != '+' && kind != '{') {  // lstrip_blocks
      const size_t nlp = text.rfind('\n');
      const size_t lp = nlp == std::string::npos ? 0 : nlp + 1;
      if ((lp > 0 || line_starting) && lp < text.size() &&
          text.find_first_not_of(kWs, lp) == std::string::npos)
        text.erase(lp);
    }
    if (!text.empty()) out.push_back({Chunk::Text, text, line});
    count_lines(pos, idx);
    if (kind != '#') out.push_back({kind == '{' ? Chunk::Var : Chunk::Block, src.substr(inner, end_inner - inner), line});
    count_lines(idx, c + 2);
    pos = c + 2;
    if (strip_after) {
      const size_t np = src.find_first_not_of(kWs, pos);
      const size_t stop = np == std::string::npos ? src.size() : np;
      count_lines(pos, stop);
      pos = stop;
    } else if (kind != '{' && !keep_after && pos < src.size() && src[pos] == '\n') {  // trim_blocks
      ++pos;
      ++line;
    }
    line_starting = pos > 0 && src[pos - 1] == '\n';
    if (pos >= src.size()) break;
  }
  return out;
}

// ---- expression tokens -----------------------------------------------------------------------------

struct Tok {
  enum Kind { Name, String, Int, Float, Op, End } k;
  std::string s;
  int64_t i = 0;
  double f = 0;
};

std::vector<Tok> lex(const std::string& src) {
  std::vector<Tok> out;
  size_t p = 0;
  while (p < src.size()) {
    const char c = src[p];
    if (strchr(kWs, c)) {
      ++p;
      continue;
    }
    if (isalpha(static_cast<unsigned char>(c)) || c == '_') {
      size_t e = p;
      while (e < src.size() && (isalnum(static_cast<unsigned char>(src[e])) || src[e] == '_')) ++e;
      out.push_back({Tok::Name, src.substr(p, e - p)});
      p = e;
      continue;
    }
    if (isdigit(static_cast<unsigned char>(c))) {
      size_t e = p;
      bool is_float = false;
      while (e < src.size() && (isdigit(static_cast<unsigned char>(src[e])) || src[e] == '_')) ++e;
      if (e + 1 < src.size() && src[e] == '.' && isdigit(static_cast<unsigned char>(src[e + 1]))) {
        is_float = true;
        ++e;
        while (e < src.size() && isdigit(static_cast<unsigned char>(src[e]))) ++e;
      }
      if (e < src.size() && (src[e] == 'e' || src[e] == 'E')) {
        size_t x = e + 1;
        if (x < src.size() && (src[x] == '+' || src[x] == '-')) ++x;
        if (x < src.size() && isdigit(static_cast<unsigned char>(src[x]))) {
          is_float = true;
          e = x;
          while (e < src.size() && isdigit(static_cast<unsigned char>(src[e]))) ++e;
        }
      }
      std::string t = src.substr(p, e - p);
      t.erase(std::remove(t.begin(), t.end(), '_'), t.end());
      Tok tk{is_float ? Tok::Float : Tok::Int, t};
      if (is_float) tk.f = strtod(t.c_str(), nullptr);
      else tk.i = strtoll(t.c_str(), nullptr, 10);
      out.push_back(tk);
      p = e;
      continue;
    }
    if (c == '\'' || c == '"') {
      std::string v;
      size_t e = p + 1;
      for (;;) {
        if (e >= src.size()) fail("unterminated string literal");
        const char ch = src[e];
        if (ch == c) break;
        if (ch == '\\' && e + 1 < src.size()) {
          const char x = src[e + 1];
          e += 2;
          switch (x) {
            case 'n': v += '\n'; break;
            case 't': v += '\t'; break;
            case 'r': v += '\r'; break;
            case '0': v += '\0'; break;
            case 'b': v += '\b'; break;
            case 'f': v += '\f'; break;
            case '\\': v += '\\'; break;
            case '\'': v += '\''; break;
            case '"': v += '"'; break;
            case '\n': break;
            case 'x':
            case 'u':
            case 'U': {
              const int n = x == 'x' ? 2 : x == 'u' ? 4 : 8;
              if (e + n > src.size()) fail("truncated escape");
              const uint32_t cp = static_cast<uint32_t>(strtoul(src.substr(e, n).c_str(), nullptr, 16));
              uni::append(v, cp);
              e += n;
              break;
            }
            default:
              v += '\\';
              v += x;
          }
          continue;
        }
        v += ch;
        ++e;
      }
      out.push_back({Tok::String, v});
      p = e + 1;
      continue;
    }
    static const char* const ops[] = {"**", "//", "==", "!=", "<=", ">=", "+", "-", "*", "/", "%", "~", "<", ">",
                                      "(", ")", "[", "]", "{", "}", ",", ".", ":", "|", "="};
    bool ok = false;
    for (const char* op : ops)
      if (src.compare(p, strlen(op), op) == 0) {
        out.push_back({Tok::Op, op});
        p += strlen(op);
        ok = true;
        break;
      }
    if (!ok) fail(std::string("unexpected character '") + c + "' in tag");
  }
  out.push_back({Tok::End, ""});
  return out;
}

// ---- filters and tests this interpreter provides ---------------------------------------------------

struct FilterSpec {
  const char* name;
  std::vector<const char*> kwargs;
  size_t min_args = 0;
  int max_args = 0;  // positional arguments after the value; -1: any
};

const std::vector<FilterSpec>& filter_specs() {
  static const std::vector<FilterSpec> v = {
      {"trim", {"chars"}, 0, 1}, {"strip", {"chars"}, 0, 1}, {"length", {}}, {"count", {}},
      {"tojson", {"indent"}, 0, 1}, {"upper", {}}, {"lower", {}}, {"title", {}}, {"capitalize", {}}, {"first", {}},
      {"last", {}}, {"join", {"d", "attribute"}, 0, 2}, {"default", {"default_value", "boolean"}, 0, 2},
      {"d", {"default_value", "boolean"}, 0, 2}, {"list", {}}, {"int", {"default", "base"}, 0, 2},
      {"float", {"default"}, 0, 1}, {"string", {}}, {"items", {}}, {"reverse", {}},
      {"replace", {"old", "new", "count"}, 2, 3}, {"safe", {}}, {"e", {}}, {"escape", {}}, {"abs", {}},
      {"map", {"attribute", "default"}, 0, -1}, {"selectattr", {}, 1, -1}, {"rejectattr", {}, 1, -1},
      {"select", {}, 0, -1}, {"reject", {}, 0, -1}, {"indent", {"width", "first", "blank"}, 0, 3}, {"unique", {}}};
  return v;
}

const FilterSpec* find_filter(const std::string& n) {
  for (const auto& f : filter_specs())
    if (n == f.name) return &f;
  return nullptr;
}

bool known_test(const std::string& n) {
  static const char* const names[] = {"defined", "undefined", "none", "string", "number", "integer", "float",
                                      "boolean", "true", "false", "mapping", "iterable", "sequence", "callable",
                                      "lower", "upper", "odd", "even", "divisibleby", "equalto", "eq", "==",
                                      "sameas", "ne", "!=", "lt", "lessthan", "<", "le", "<=", "gt", "greaterthan",
                                      ">", "ge", ">=", "in"};
  for (const char* x : names)
    if (n == x) return true;
  return false;
}

// ---- syntax tree -----------------------------------------------------------------------------------

enum class EK { Lit, Name, List, Dict, Attr, Item, Slice, Call, Filter, Test, Neg, Pos, Bin, Cmp, And, Or, Not, Cond,
                Splat, KwSplat };  // Splat / KwSplat: `*args` / `**kwargs` of a call

struct Expr;
using EP = std::unique_ptr<Expr>;

struct Expr {
  EK k;
  bool tuple = false;  // EK::List written as a tuple
  std::string name;
  Value lit;
  std::vector<EP> a;
  std::vector<std::pair<std::string, EP>> kw;
  std::vector<std::string> ops;  // comparison chain: a[0] ops[0] a[1] ops[1] a[2] ...
  bool negate = false;
};

EP mk(EK k, std::string name = "") {
  EP e = std::make_unique<Expr>();
  e->k = k;
  e->name = std::move(name);
  return e;
}

enum class SK { Text, Out, If, For, Set, SetAttr, SetBlock, Macro, Break, Continue };

struct Stmt {
  explicit Stmt(SK kind) : k(kind) {}
  SK k;
  std::string text;
  EP e;
  std::vector<std::pair<EP, std::vector<Stmt>>> branches;
  std::vector<std::string> targets;
  EP filter;
  std::vector<Stmt> body, else_body;
  std::vector<EP> defaults;  // macro parameter defaults (null: required)
};

class Parser {
 public:
  explicit Parser(std::vector<Tok> t) : t_(std::move(t)) {}
  bool at_end() const { return t_[p_].k == Tok::End; }
  const Tok& peek(size_t o = 0) const { return t_[std::min(p_ + o, t_.size() - 1)]; }
  bool is_op(const char* s, size_t o = 0) const { return peek(o).k == Tok::Op && peek(o).s == s; }
  bool is_name(const char* s, size_t o = 0) const { return peek(o).k == Tok::Name && peek(o).s == s; }
  void expect_op(const char* s) {
    if (!is_op(s)) fail(std::string("expected '") + s + "' but found '" + peek().s + "'");
    ++p_;
  }
  std::string name() {
    if (peek().k != Tok::Name) fail("expected a name, found '" + peek().s + "'");
    return t_[p_++].s;
  }
  void skip() { ++p_; }
  void expect_end() {
    if (!at_end()) fail("unexpected '" + peek().s + "' at the end of a tag");
  }
  // The end of a tag that opens a body; jinja2 allows a colon there for Python compatibility.
  void expect_body_start() {
    if (is_op(":")) skip();
    expect_end();
  }

  EP expression() { return condexpr(); }
  EP expression_no_cond() { return or_expr(); }

  // expression list without parentheses (`set` values, `if` tests): a, b -> list. `if` / `elif` tests
  // take no conditional expression at their top level (jinja2 parses them with_condexpr=False).
  EP tuple_or_expr(bool with_cond = true) {
    EP e = with_cond ? expression() : expression_no_cond();
    if (!is_op(",")) return e;
    EP l = mk(EK::List);
    l->tuple = true;
    l->a.push_back(std::move(e));
    while (is_op(",")) {
      skip();
      if (at_end()) break;
      l->a.push_back(with_cond ? expression() : expression_no_cond());
    }
    return l;
  }

 private:
  EP condexpr() {
    EP e = or_expr();
    while (is_name("if")) {
      skip();
      EP c = mk(EK::Cond);
      EP cond = or_expr();
      EP other;
      if (is_name("else")) {
        skip();
        other = condexpr();
      }
      c->a.push_back(std::move(e));
      c->a.push_back(std::move(cond));
      c->a.push_back(std::move(other));
      e = std::move(c);
    }
    return e;
  }
  EP or_expr() {
    EP e = and_expr();
    while (is_name("or")) {
      skip();
      EP n = mk(EK::Or);
      n->a.push_back(std::move(e));
      n->a.push_back(and_expr());
      e = std::move(n);
    }
    return e;
  }
  EP and_expr() {
    EP e = not_expr();
    while (is_name("and")) {
      skip();
      EP n = mk(EK::And);
      n->a.push_back(std::move(e));
      n->a.push_back(not_expr());
      e = std::move(n);
    }
    return e;
  }
  EP not_expr() {
    if (is_name("not")) {
      skip();
      EP n = mk(EK::Not);
      n->a.push_back(not_expr());
      return n;
    }
    return compare();
  }
  EP compare() {
    EP e = math1();
    EP chain;  // `a < b < c` is `a < b and b < c`, as in Python
    for (;;) {
      std::string op;
      if (peek().k == Tok::Op && (peek().s == "==" || peek().s == "!=" || peek().s == "<" || peek().s == ">" ||
                                  peek().s == "<=" || peek().s == ">=")) {
        op = peek().s;
        skip();
      } else if (is_name("in")) {
        op = "in";
        skip();
      } else if (is_name("not") && is_name("in", 1)) {
        op = "notin";
        skip();
        skip();
      } else {
        return chain ? std::move(chain) : std::move(e);
      }
      if (!chain) {
        chain = mk(EK::Cmp);
        chain->a.push_back(std::move(e));
      }
      chain->ops.push_back(op);
      chain->a.push_back(math1());
    }
  }
  EP binary(EP l, const std::string& op, EP r) {
    EP n = mk(EK::Bin, op);
    n->a.push_back(std::move(l));
    n->a.push_back(std::move(r));
    return n;
  }
  EP math1() {
    EP e = concat();
    while (is_op("+") || is_op("-")) {
      const std::string op = peek().s;
      skip();
      e = binary(std::move(e), op, concat());
    }
    return e;
  }
  EP concat() {
    EP e = math2();
    while (is_op("~")) {
      skip();
      e = binary(std::move(e), "~", math2());
    }
    return e;
  }
  EP math2() {
    EP e = power();
    while (is_op("*") || is_op("/") || is_op("//") || is_op("%")) {
      const std::string op = peek().s;
      skip();
      e = binary(std::move(e), op, power());
    }
    return e;
  }
  EP power() {
    EP e = unary(true);
    while (is_op("**")) {
      skip();
      e = binary(std::move(e), "**", unary(true));
    }
    return e;
  }
  EP unary(bool with_filter) {
    EP e;
    if (is_op("-") || is_op("+")) {
      const bool neg = is_op("-");
      skip();
      e = mk(neg ? EK::Neg : EK::Pos);
      e->a.push_back(unary(false));
    } else {
      e = primary();
    }
    e = postfix(std::move(e));
    if (with_filter) e = filter_expr(std::move(e));
    return e;
  }
  EP primary() {
    const Tok& t = peek();
    if (t.k == Tok::Name) {
      const std::string n = t.s;
      skip();
      EP e = mk(EK::Lit);
      if (n == "true" || n == "True") e->lit = Value::boolean(true);
      else if (n == "false" || n == "False") e->lit = Value::boolean(false);
      else if (n == "none" || n == "None") e->lit = Value::none();
      else return mk(EK::Name, n);
      return e;
    }
    if (t.k == Tok::String) {
      std::string s;
      while (peek().k == Tok::String) {  // adjacent literals concatenate
        s += peek().s;
        skip();
      }
      EP e = mk(EK::Lit);
      e->lit = Value::str(s);
      return e;
    }
    if (t.k == Tok::Int || t.k == Tok::Float) {
      EP e = mk(EK::Lit);
      e->lit = t.k == Tok::Int ? Value::integer(t.i) : Value::number(t.f);
      skip();
      return e;
    }
    if (is_op("(")) {
      skip();
      if (is_op(")")) {
        skip();
        EP t0 = mk(EK::List);
        t0->tuple = true;
        return t0;
      }
      EP e = expression();
      if (is_op(",")) {
        EP l = mk(EK::List);
        l->tuple = true;
        l->a.push_back(std::move(e));
        while (is_op(",")) {
          skip();
          if (is_op(")")) break;
          l->a.push_back(expression());
        }
        e = std::move(l);
      }
      expect_op(")");
      return e;
    }
    if (is_op("[")) {
      skip();
      EP l = mk(EK::List);
      while (!is_op("]")) {
        l->a.push_back(expression());
        if (!is_op(",")) break;
        skip();
      }
      expect_op("]");
      return l;
    }
    if (is_op("{")) {
      skip();
      EP d = mk(EK::Dict);
      while (!is_op("}")) {
        d->a.push_back(expression());
        expect_op(":");
        d->a.push_back(expression());
        if (!is_op(",")) break;
        skip();
      }
      expect_op("}");
      return d;
    }
    fail("unexpected '" + t.s + "' in expression");
  }
  void call_args(Expr& n) {
    expect_op("(");
    while (!is_op(")")) {
      if (is_op("*") || is_op("**")) {
        EP sp = mk(is_op("*") ? EK::Splat : EK::KwSplat);
        skip();
        sp->a.push_back(expression());
        if (sp->k == EK::Splat) n.a.push_back(std::move(sp));
        else n.kw.emplace_back("**", std::move(sp));
      } else if (peek().k == Tok::Name && is_op("=", 1)) {
        std::string k = name();
        skip();
        n.kw.emplace_back(k, expression());
      } else {
        if (!n.kw.empty()) fail("invalid syntax for function call expression");
        n.a.push_back(expression());
      }
      if (!is_op(",")) break;
      skip();
    }
    expect_op(")");
  }
  EP postfix(EP e) {
    for (;;) {
      if (is_op(".")) {
        skip();
        EP n;
        if (peek().k == Tok::Int) {  // `x.0` is item 0
          n = mk(EK::Item);
          n->a.push_back(std::move(e));
          EP key = mk(EK::Lit);
          key->lit = Value::integer(peek().i);
          skip();
          n->a.push_back(std::move(key));
          e = std::move(n);
          continue;
        }
        n = mk(EK::Attr, name());
        n->a.push_back(std::move(e));
        e = std::move(n);
      } else if (is_op("[")) {
        skip();
        EP idx[3];
        bool slice = false;
        for (int part = 0; part < 3; ++part) {
          if (!is_op(":") && !is_op("]")) idx[part] = expression();
          if (is_op(":") && part < 2) {
            slice = true;
            skip();
          } else {
            break;
          }
        }
        if (!slice && is_op(",")) {  // a tuple key (`x[1, 2]`): never a key of these values
          EP t = mk(EK::List);
          t->tuple = true;
          if (idx[0]) t->a.push_back(std::move(idx[0]));
          while (is_op(",")) {  // no trailing comma in a subscript (jinja2 rejects it)
            skip();
            t->a.push_back(expression());
          }
          idx[0] = std::move(t);
        }
        expect_op("]");
        EP n = mk(slice ? EK::Slice : EK::Item);
        n->a.push_back(std::move(e));
        if (slice) {
          for (auto& x : idx) n->a.push_back(std::move(x));
        } else {
          if (!idx[0]) idx[0] = mk(EK::Lit);  // `x[]`: an undefined key, as jinja2 evaluates it
          n->a.push_back(std::move(idx[0]));
        }
        e = std::move(n);
      } else if (is_op("(")) {
        EP n = mk(EK::Call);
        n->a.push_back(std::move(e));
        call_args(*n);
        e = std::move(n);
      } else {
        return e;
      }
    }
  }
  EP filter_expr(EP e) {
    for (;;) {
      if (is_op("|")) {
        skip();
        std::string f = name();
        while (is_op(".")) {  // dotted filter names are not used by chat templates
          skip();
          f += "." + name();
        }
        EP n = mk(EK::Filter, f);
        n->a.push_back(std::move(e));
        if (is_op("(")) call_args(*n);
        e = std::move(n);
      } else if (is_name("is")) {
        skip();
        bool neg = false;
        if (is_name("not")) {
          neg = true;
          skip();
        }
        std::string tn;
        if (peek().k == Tok::Name) {
          tn = name();
          while (is_op(".")) {  // dotted test names parse (and are unknown)
            skip();
            tn += "." + name();
          }
        } else if (is_op("==") || is_op("!=") || is_op("<") || is_op(">") || is_op("<=") || is_op(">=")) {
          tn = peek().s;
          skip();
        } else {
          fail("expected a test name after 'is'");
        }
        EP n = mk(EK::Test, tn);
        n->negate = neg;
        n->a.push_back(std::move(e));
        if (is_op("(")) {
          call_args(*n);
        } else if (peek().k == Tok::String || peek().k == Tok::Int || peek().k == Tok::Float || is_op("[") ||
                   is_op("{") || (peek().k == Tok::Name && !is_name("and") && !is_name("or") && !is_name("else"))) {
          // `x is divisibleby 3`, `x is sameas none` (jinja2 takes one primary with its postfix here)
          if (is_name("is")) fail("tests cannot be chained with 'is'");
          n->a.push_back(postfix(primary()));
        }
        e = std::move(n);
      } else if (is_op("(")) {
        EP n = mk(EK::Call);
        n->a.push_back(std::move(e));
        call_args(*n);
        e = std::move(n);
      } else {
        return e;
      }
    }
  }

  std::vector<Tok> t_;
  size_t p_ = 0;
};

// Statement tree from the chunks.
class Builder {
 public:
  explicit Builder(std::vector<Chunk> c) : c_(std::move(c)) {}

  std::vector<Stmt> build() {
    std::string term;
    auto body = block({}, term);
    if (!term.empty()) fail("unexpected {% " + term + " %}");
    check(body, false);
    return body;
  }

 private:
  // Parses statements until a block tag whose keyword is in `ends`; returns that keyword in `term`
  // (the tag's parser is left in `last_` for elif / else conditions).
  std::vector<Stmt> block(const std::vector<std::string>& ends, std::string& term) {
    std::vector<Stmt> out;
    while (i_ < c_.size()) {
      const Chunk& ch = c_[i_++];
      if (ch.kind == Chunk::Text) {
        Stmt s(SK::Text);
        s.text = ch.s;
        out.push_back(std::move(s));
        continue;
      }
      auto p = std::make_unique<Parser>(lex(ch.s));
      if (ch.kind == Chunk::Var) {
        Stmt s(SK::Out);
        s.e = p->tuple_or_expr();
        p->expect_end();
        out.push_back(std::move(s));
        continue;
      }
      const std::string kw = p->name();
      if (std::find(ends.begin(), ends.end(), kw) != ends.end()) {
        term = kw;
        last_ = std::move(p);
        return out;
      }
      try {
        out.push_back(statement(kw, *p));
      } catch (const TemplateError& e) {
        fail(std::string(e.what()) + " (line " + std::to_string(ch.line) + ")");
      }
    }
    if (!ends.empty()) fail("missing {% " + ends[0] + " %}");
    term.clear();
    return out;
  }

  Stmt statement(const std::string& kw, Parser& p) {
    if (kw == "if") {
      Stmt s(SK::If);
      EP cond = p.tuple_or_expr(false);
      p.expect_body_start();
      for (;;) {
        std::string term;
        auto body = block({"elif", "else", "endif"}, term);
        s.branches.emplace_back(std::move(cond), std::move(body));
        if (term == "endif") {
          last_->expect_end();
          return s;
        }
        if (term == "else") {
          last_->expect_body_start();
          std::string t2;
          auto eb = block({"endif"}, t2);
          last_->expect_end();
          s.branches.emplace_back(nullptr, std::move(eb));
          return s;
        }
        cond = last_->tuple_or_expr(false);  // elif
        last_->expect_body_start();
      }
    }
    if (kw == "for") {
      Stmt s(SK::For);
      s.targets.push_back(p.name());
      while (p.is_op(",")) {
        p.skip();
        s.targets.push_back(p.name());
      }
      if (!p.is_name("in")) fail("expected 'in' in for");
      p.skip();
      s.e = p.tuple_or_expr(false);
      if (p.is_name("if")) {
        p.skip();
        s.filter = p.expression();
      }
      if (p.is_name("recursive")) fail("recursive loops are not supported");
      p.expect_body_start();
      std::string term;
      s.body = block({"else", "endfor"}, term);
      if (term == "endfor") last_->expect_end();
      if (term == "else") {
        last_->expect_body_start();
        std::string t2;
        s.else_body = block({"endfor"}, t2);
        last_->expect_end();
      }
      return s;
    }
    if (kw == "set") {
      std::string first = p.name();
      if (p.is_op(".")) {  // namespace attribute
        p.skip();
        Stmt s(SK::SetAttr);
        s.targets = {first, p.name()};
        p.expect_op("=");
        s.e = p.tuple_or_expr();
        p.expect_end();
        return s;
      }
      Stmt s(SK::Set);
      s.targets.push_back(first);
      while (p.is_op(",")) {
        p.skip();
        s.targets.push_back(p.name());
      }
      if (p.at_end() || (p.is_op(":") && p.peek(1).k == Tok::End)) {  // block set
        p.expect_body_start();
        s.k = SK::SetBlock;
        std::string term;
        s.body = block({"endset"}, term);
        last_->expect_end();
        return s;
      }
      p.expect_op("=");
      s.e = p.tuple_or_expr();
      p.expect_end();
      return s;
    }
    if (kw == "macro") {
      Stmt s(SK::Macro);
      s.text = p.name();
      p.expect_op("(");
      while (!p.is_op(")")) {
        s.targets.push_back(p.name());
        if (p.is_op("=")) {
          p.skip();
          s.defaults.push_back(p.expression());
        } else {
          s.defaults.push_back(nullptr);
        }
        if (!p.is_op(",")) break;
        p.skip();
      }
      p.expect_op(")");
      p.expect_body_start();
      std::string term;
      s.body = block({"endmacro"}, term);
      last_->expect_end();
      return s;
    }
    if (kw == "break" || kw == "continue") {
      p.expect_end();
      return Stmt(kw == "break" ? SK::Break : SK::Continue);
    }
    fail("unsupported tag {% " + kw + " %}");
  }

  // jinja2 rejects an unknown filter or test when it compiles the template, except in "soft" code: an
  // `if` statement's tests and branches, a conditional expression and the right operand of `and` /
  // `or`, where the error is raised only if that code runs. Loop, macro and set-block bodies are never
  // soft.
  static void check(const Expr& e, bool soft) {
    const bool s2 = soft || e.k == EK::Cond;
    if (!s2 && e.k == EK::Filter && !find_filter(e.name)) fail("no filter named '" + e.name + "'");
    if (!s2 && e.k == EK::Test && !known_test(e.name)) fail("no test named '" + e.name + "'");
    for (size_t k = 0; k < e.a.size(); ++k)  // the right operand of and / or may not run: soft
      if (e.a[k]) check(*e.a[k], s2 || ((e.k == EK::And || e.k == EK::Or) && k == 1));
    for (const auto& kv : e.kw) check(*kv.second, s2);
  }
  static void check(const std::vector<Stmt>& body, bool soft) {
    for (const Stmt& st : body) {
      if (st.e) check(*st.e, soft);
      switch (st.k) {
        case SK::If:
          for (const auto& br : st.branches) {
            if (br.first) check(*br.first, true);
            check(br.second, true);
          }
          break;
        case SK::For:
          if (st.filter) check(*st.filter, false);
          check(st.body, false);
          check(st.else_body, false);
          break;
        case SK::SetBlock:
        case SK::Macro:
          for (const auto& d : st.defaults)
            if (d) check(*d, false);
          check(st.body, false);
          break;
        default: break;
      }
    }
  }

  std::vector<Chunk> c_;
  size_t i_ = 0;
  std::unique_ptr<Parser> last_;
};

// ---- evaluation ------------------------------------------------------------------------------------

enum class Flow { Normal, Break, Continue };

struct Ctx {
  std::vector<std::vector<std::pair<std::string, Value>>> scopes;
  int64_t budget = 20000000;  // evaluation steps before a runaway template is stopped
  int depth = 0;
  size_t max_out = 16u << 20;

  Value lookup(const std::string& n) const {
    for (size_t k = scopes.size(); k-- > 0;)
      for (const auto& kv : scopes[k])
        if (kv.first == n) return kv.second;
    return Value();
  }
  void assign(const std::string& n, Value v) {
    auto& s = scopes.back();
    for (auto& kv : s)
      if (kv.first == n) {
        kv.second = std::move(v);
        return;
      }
    s.emplace_back(n, std::move(v));
  }
  void tick() {
    if (--budget < 0) fail("template evaluation exceeded its step budget");
  }
};

const Value* kwarg(const Kwargs& kw, const char* name) {
  for (const auto& kv : kw)
    if (kv.first == name) return &kv.second;
  return nullptr;
}

// Positional argument k, else keyword `name`, else nullptr.
const Value* arg(const Args& a, const Kwargs& kw, size_t k, const char* name) {
  if (k < a.size()) return &a[k];
  return kwarg(kw, name);
}

std::string arg_str(const Args& a, const Kwargs& kw, size_t k, const char* name, const std::string& dflt) {
  const Value* v = arg(a, kw, k, name);
  if (!v || v->t == Value::None || v->t == Value::Undefined) return dflt;
  if (v->t != Value::Str) fail(std::string("argument '") + name + "' must be a string");
  return v->s;
}

Value slice_of(const Value& obj, const Value* st, const Value* sp, const Value* stepv) {
  std::vector<Value> items;
  bool is_str = obj.t == Value::Str;
  if (is_str) {
    for (auto& c : chars(obj.s)) items.push_back(Value::str(c));
  } else if (obj.t == Value::ListT) {
    items = *obj.l;
  } else if (obj.t == Value::Undefined) {
    undefined_access("items");
  } else {
    fail("value cannot be sliced");
  }
  const int64_t n = static_cast<int64_t>(items.size());
  const int64_t step = stepv && stepv->t != Value::None ? as_int(*stepv) : 1;
  if (step == 0) fail("slice step cannot be zero");
  auto norm = [&](const Value* v, int64_t dflt, bool is_stop) -> int64_t {
    if (!v || v->t == Value::None) return dflt;
    int64_t x = as_int(*v);
    if (x < 0) x += n;
    if (step > 0) return std::clamp<int64_t>(x, 0, n);
    return std::clamp<int64_t>(x, -1, n - 1) + (is_stop ? 0 : 0);
  };
  const int64_t b = norm(st, step > 0 ? 0 : n - 1, false);
  const int64_t e = norm(sp, step > 0 ? n : -1, true);
  List out;
  for (int64_t k = b; step > 0 ? k < e : k > e; k += step) out.push_back(items[static_cast<size_t>(k)]);
  if (!is_str) return Value::list(std::move(out));
  std::string s;
  for (auto& x : out) s += x.s;
  return Value::str(s);
}

std::vector<std::string> py_split(const std::string& s, const Value* sep, int64_t maxsplit) {
  std::vector<std::string> out;
  if (!sep || sep->t == Value::None || sep->t == Value::Undefined) {  // runs of whitespace
    size_t p = s.find_first_not_of(kWs);
    while (p != std::string::npos) {
      if (maxsplit >= 0 && static_cast<int64_t>(out.size()) == maxsplit) {
        out.push_back(strip_chars(s.substr(p), kWs, false, true));
        break;
      }
      const size_t e = s.find_first_of(kWs, p);
      out.push_back(s.substr(p, e == std::string::npos ? std::string::npos : e - p));
      p = e == std::string::npos ? e : s.find_first_not_of(kWs, e);
    }
    return out;
  }
  if (sep->t != Value::Str || sep->s.empty()) fail("empty or non-string separator");
  size_t p = 0;
  for (;;) {
    if (maxsplit >= 0 && static_cast<int64_t>(out.size()) == maxsplit) break;
    const size_t k = s.find(sep->s, p);
    if (k == std::string::npos) break;
    out.push_back(s.substr(p, k - p));
    p = k + sep->s.size();
  }
  out.push_back(s.substr(p));
  return out;
}

Value str_list(const std::vector<std::string>& v) {
  List l;
  for (const auto& s : v) l.push_back(Value::str(s));
  return Value::list(std::move(l));
}

std::string title_case(const std::string& s) {
  std::string o = s;
  bool start = true;
  for (char& c : o) {
    const bool alpha = isalpha(static_cast<unsigned char>(c));
    if (alpha) c = static_cast<char>(start ? toupper(static_cast<unsigned char>(c)) : tolower(static_cast<unsigned char>(c)));
    start = !alpha && !isdigit(static_cast<unsigned char>(c)) && c != '\'';
  }
  return o;
}

std::string escape_html(const std::string& s) {
  std::string o;
  for (char c : s) {
    switch (c) {
      case '&': o += "&amp;"; break;
      case '<': o += "&lt;"; break;
      case '>': o += "&gt;"; break;
      case '"': o += "&#34;"; break;
      case '\'': o += "&#39;"; break;
      default: o += c;
    }
  }
  return o;
}

void arity(const Args& a, const Kwargs& kw, size_t lo, size_t hi, const std::string& name) {
  const size_t n = a.size() + kw.size();
  if (n < lo || n > hi) fail(name + "() takes " + std::to_string(lo) + "-" + std::to_string(hi) + " arguments");
}

// Bound methods of strings and dicts.
Value method(const Value& obj, const std::string& name) {
  if (obj.t == Value::Str) {
    const std::string s = obj.s;
    if (name == "strip" || name == "lstrip" || name == "rstrip") {
      const bool l = name != "rstrip", r = name != "lstrip";
      return Value::func([s, l, r, name](const Args& a, const Kwargs& kw) {
        arity(a, kw, 0, 1, name);
        return Value::str(strip_chars(s, arg_str(a, kw, 0, "chars", kWs), l, r));
      });
    }
    if (name == "split" || name == "rsplit") {
      const bool right = name == "rsplit";
      return Value::func([s, right, name](const Args& a, const Kwargs& kw) {
        arity(a, kw, 0, 2, name);
        const Value* mx = arg(a, kw, 1, "maxsplit");
        const int64_t maxsplit = mx ? as_int(*mx) : -1;
        const Value* sep = arg(a, kw, 0, "sep");
        if (!right || maxsplit < 0) return str_list(py_split(s, sep, maxsplit));
        // rsplit with a limit: split fully, then join the leading pieces back
        auto parts = py_split(s, sep, -1);
        if (static_cast<int64_t>(parts.size()) <= maxsplit + 1) return str_list(parts);
        const std::string j = sep && sep->t == Value::Str ? sep->s : " ";
        std::string head = parts[0];
        const size_t keep = parts.size() - static_cast<size_t>(maxsplit);
        for (size_t k = 1; k < keep; ++k) head += j + parts[k];
        std::vector<std::string> out = {head};
        out.insert(out.end(), parts.begin() + static_cast<long>(keep), parts.end());
        return str_list(out);
      });
    }
    if (name == "startswith" || name == "endswith") {
      const bool start = name == "startswith";
      return Value::func([s, start, name](const Args& a, const Kwargs& kw) {
        arity(a, kw, 1, 1, name);
        if (a.empty()) fail("startswith/endswith need an argument");
        List cands = a[0].t == Value::ListT ? *a[0].l : List{a[0]};
        for (const Value& c : cands) {
          if (c.t != Value::Str) fail("startswith/endswith need strings");
          if (c.s.size() <= s.size() &&
              s.compare(start ? 0 : s.size() - c.s.size(), c.s.size(), c.s) == 0)
            return Value::boolean(true);
        }
        return Value::boolean(false);
      });
    }
    if (name == "upper" || name == "lower" || name == "title" || name == "capitalize") {
      return Value::func([s, name](const Args& a, const Kwargs& kw) {
        arity(a, kw, 0, 0, name);
        if (name == "upper") return Value::str(ascii_upper(s));
        if (name == "lower") return Value::str(ascii_lower(s));
        if (name == "title") return Value::str(title_case(s));
        std::string o = ascii_lower(s);
        if (!o.empty()) o[0] = static_cast<char>(toupper(static_cast<unsigned char>(o[0])));
        return Value::str(o);
      });
    }
    if (name == "replace") {
      return Value::func([s](const Args& a, const Kwargs& kw) {
        arity(a, kw, 2, 3, "replace");
        const Value* c = arg(a, kw, 2, "count");
        return Value::str(replace_all(s, arg_str(a, kw, 0, "old", ""), arg_str(a, kw, 1, "new", ""), c ? as_int(*c) : -1));
      });
    }
    if (name == "find" || name == "count") {
      const bool find = name == "find";
      return Value::func([s, find](const Args& a, const Kwargs& kw) {
        arity(a, kw, 1, 1, find ? "find" : "count");
        const std::string sub = arg_str(a, kw, 0, "sub", "");
        if (find) {
          const size_t k = s.find(sub);
          return Value::integer(k == std::string::npos ? -1 : static_cast<int64_t>(uni::length(s.substr(0, k))));
        }
        int64_t n = 0;
        if (sub.empty()) return Value::integer(static_cast<int64_t>(uni::length(s)) + 1);
        for (size_t p = s.find(sub); p != std::string::npos; p = s.find(sub, p + sub.size())) ++n;
        return Value::integer(n);
      });
    }
    if (name == "join") {
      return Value::func([s](const Args& a, const Kwargs& kw) {
        arity(a, kw, 1, 1, "join");
        if (a.empty()) fail("join needs an iterable");
        std::string o;
        bool first = true;
        for (const Value& x : iterate(a[0])) {
          o += (first ? "" : s) + to_str(x);
          first = false;
        }
        return Value::str(o);
      });
    }
    return Value();
  }
  if (obj.t == Value::DictT) {
    const Value self = obj;
    if (name == "items" || name == "keys" || name == "values") {
      return Value::func([self, name](const Args& a, const Kwargs& kw) {
        arity(a, kw, 0, 0, name);
        List out;
        for (const auto& kv : *self.d) {
          if (name == "items") {
            Value pair = Value::list({Value::str(kv.first), kv.second});
            pair.is_tuple = true;
            out.push_back(pair);
          }
          else if (name == "keys") out.push_back(Value::str(kv.first));
          else out.push_back(kv.second);
        }
        return Value::list(std::move(out));
      });
    }
    if (name == "get") {
      return Value::func([self](const Args& a, const Kwargs& kw) {
        arity(a, kw, 1, 2, "get");
        if (a.empty()) fail("get needs a key");
        const Value* v = a[0].t == Value::Str ? self.get(a[0].s) : nullptr;
        if (v) return *v;
        const Value* d = arg(a, kw, 1, "default");
        return d ? *d : Value::none();
      });
    }
  }
  return Value();
}

Value get_attr(const Value& obj, const std::string& name) {
  if (obj.t == Value::Undefined) undefined_access("attribute '" + name + "'");
  if (obj.t == Value::DictT) {
    if (!obj.is_namespace) {
      Value m = method(obj, name);
      if (m.t != Value::Undefined) return m;
    }
    const Value* v = obj.get(name);
    return v ? *v : Value();
  }
  if (obj.t == Value::Str) return method(obj, name);
  return Value();
}

Value get_item(const Value& obj, const Value& key) {
  if (obj.t == Value::Undefined) undefined_access("item");
  if (obj.t == Value::DictT) {
    if (key.t == Value::Str) {
      const Value* v = obj.get(key.s);
      return v ? *v : Value();
    }
    return Value();
  }
  if ((obj.t == Value::ListT || obj.t == Value::Str) && (key.t == Value::Int || key.t == Value::Bool)) {
    const List items = iterate(obj);
    int64_t k = as_int(key);
    if (k < 0) k += static_cast<int64_t>(items.size());
    if (k < 0 || k >= static_cast<int64_t>(items.size())) return Value();
    return items[static_cast<size_t>(k)];
  }
  if (key.t == Value::Str) return get_attr(obj, key.s);
  return Value();
}

Value arith(const std::string& op, const Value& a, const Value& b) {
  if (op == "~") return Value::str(to_str(a) + to_str(b));
  const bool both_int = (a.t == Value::Int || a.t == Value::Bool) && (b.t == Value::Int || b.t == Value::Bool);
  if (op == "+") {
    if (a.t == Value::Str && b.t == Value::Str) {
      if (a.is_markup) return markup(a.s + (b.is_markup ? b.s : escape_html(b.s)));
      return Value::str(a.s + b.s);
    }
    if (a.t == Value::ListT && b.t == Value::ListT) {
      List l = *a.l;
      l.insert(l.end(), b.l->begin(), b.l->end());
      return Value::list(std::move(l));
    }
  }
  if (op == "*") {
    const Value* seq = a.t == Value::Str || a.t == Value::ListT ? &a : (b.t == Value::Str || b.t == Value::ListT ? &b : nullptr);
    const Value* cnt = seq == &a ? &b : &a;
    if (seq && (cnt->t == Value::Int || cnt->t == Value::Bool)) {
      const int64_t n = std::max<int64_t>(0, as_int(*cnt));
      if (seq->t == Value::Str) {
        std::string o;
        for (int64_t k = 0; k < n; ++k) o += seq->s;
        return Value::str(o);
      }
      List l;
      for (int64_t k = 0; k < n; ++k) l.insert(l.end(), seq->l->begin(), seq->l->end());
      return Value::list(std::move(l));
    }
  }
  if (!is_num(a) || !is_num(b)) fail("unsupported operand types for " + op);
  if (both_int) {
    const int64_t x = as_int(a), y = as_int(b);
    if (op == "+") return Value::integer(x + y);
    if (op == "-") return Value::integer(x - y);
    if (op == "*") return Value::integer(x * y);
    if (op == "//" || op == "%") {
      if (y == 0) fail("integer division or modulo by zero");
      int64_t q = x / y, r = x % y;
      if (r != 0 && ((r < 0) != (y < 0))) {
        --q;
        r += y;
      }
      return Value::integer(op == "//" ? q : r);
    }
    if (op == "**" && y >= 0) {
      int64_t r = 1;
      for (int64_t k = 0; k < y; ++k) r *= x;
      return Value::integer(r);
    }
  }
  const double x = num(a), y = num(b);
  if (op == "+") return Value::number(x + y);
  if (op == "-") return Value::number(x - y);
  if (op == "*") return Value::number(x * y);
  if (op == "/") {
    if (y == 0) fail("division by zero");
    return Value::number(x / y);
  }
  if (op == "//") {
    if (y == 0) fail("division by zero");
    return Value::number(std::floor(x / y));
  }
  if (op == "%") {
    if (y == 0) fail("modulo by zero");
    return Value::number(x - std::floor(x / y) * y);
  }
  if (op == "**") return Value::number(std::pow(x, y));
  fail("unknown operator " + op);
}

bool cmp_op(const std::string& op, const Value& a, const Value& b) {
  if (op == "==") return equal(a, b);
  if (op == "!=") return !equal(a, b);
  if (op == "in") return contains(b, a);
  if (op == "notin") return !contains(b, a);
  const int r = compare(a, b);
  if (op == "<") return r < 0;
  if (op == ">") return r > 0;
  if (op == "<=") return r <= 0;
  return r >= 0;
}

class Eval {
 public:
  // Positional and keyword arguments of a call, filter or test (first positional node: `from`).
  void call_values(const Expr& e, size_t from, Ctx& c, Args& args, Kwargs& kw) {
    for (size_t k = from; k < e.a.size(); ++k) {
      if (e.a[k]->k == EK::Splat) {
        for (const Value& x : iterate(eval(*e.a[k]->a[0], c))) args.push_back(x);
      } else {
        args.push_back(eval(*e.a[k], c));
      }
    }
    for (const auto& kv : e.kw) {
      if (kv.second->k == EK::KwSplat) {
        const Value d = eval(*kv.second->a[0], c);
        if (d.t != Value::DictT) fail("** needs a mapping");
        for (const auto& x : *d.d) kw.emplace_back(x.first, x.second);
      } else {
        kw.emplace_back(kv.first, eval(*kv.second, c));
      }
    }
  }

  Value eval(const Expr& e, Ctx& c) {
    c.tick();
    switch (e.k) {
      case EK::Lit: return e.lit;
      case EK::Name: return c.lookup(e.name);
      case EK::List: {
        List l;
        for (const auto& x : e.a) l.push_back(eval(*x, c));
        Value v = Value::list(std::move(l));
        v.is_tuple = e.tuple;
        return v;
      }
      case EK::Dict: {
        Value d = Value::dict();
        for (size_t k = 0; k + 1 < e.a.size(); k += 2) {
          const Value key = eval(*e.a[k], c);
          if (key.t != Value::Str) fail("dict keys must be strings");
          d.set(key.s, eval(*e.a[k + 1], c));
        }
        return d;
      }
      case EK::Attr: return get_attr(eval(*e.a[0], c), e.name);
      case EK::Item: return get_item(eval(*e.a[0], c), eval(*e.a[1], c));
      case EK::Slice: {
        const Value obj = eval(*e.a[0], c);
        Value parts[3];
        for (int k = 0; k < 3; ++k)
          if (e.a[1 + k]) parts[k] = eval(*e.a[1 + k], c);
        return slice_of(obj, e.a[1] ? &parts[0] : nullptr, e.a[2] ? &parts[1] : nullptr, e.a[3] ? &parts[2] : nullptr);
      }
      case EK::Call: {
        const Value f = eval(*e.a[0], c);
        Args args;
        Kwargs kw;
        call_values(e, 1, c, args, kw);
        if (f.t != Value::Callable) fail("value is not callable");
        if (++c.depth > 256) fail("call depth limit");
        Value r = (*f.fn)(args, kw);
        --c.depth;
        return r;
      }
      case EK::Filter: {
        const Value v = eval(*e.a[0], c);
        Args args;
        Kwargs kw;
        call_values(e, 1, c, args, kw);
        return filter(e.name, v, args, kw, c);
      }
      case EK::Test: {
        const Value v = eval(*e.a[0], c);
        Args args;
        Kwargs kw;
        call_values(e, 1, c, args, kw);
        if (!kw.empty()) fail("tests take no keyword arguments");
        return Value::boolean(test(e.name, v, args, c) != e.negate);
      }
      case EK::Neg:
      case EK::Pos: {
        const Value v = eval(*e.a[0], c);
        if (!is_num(v)) fail("bad operand for unary " + std::string(e.k == EK::Neg ? "-" : "+"));
        if (e.k == EK::Pos) return v.t == Value::Bool ? Value::integer(v.b) : v;
        return v.t == Value::Float ? Value::number(-v.f) : Value::integer(-as_int(v));
      }
      case EK::Bin: return arith(e.name, eval(*e.a[0], c), eval(*e.a[1], c));
      case EK::Cmp: {
        Value left = eval(*e.a[0], c);
        for (size_t k = 0; k < e.ops.size(); ++k) {
          Value right = eval(*e.a[k + 1], c);
          if (!cmp_op(e.ops[k], left, right)) return Value::boolean(false);
          left = std::move(right);
        }
        return Value::boolean(true);
      }
      case EK::And: {
        Value a = eval(*e.a[0], c);
        return a.truthy() ? eval(*e.a[1], c) : a;
      }
      case EK::Or: {
        Value a = eval(*e.a[0], c);
        return a.truthy() ? a : eval(*e.a[1], c);
      }
      case EK::Not: return Value::boolean(!eval(*e.a[0], c).truthy());
      case EK::Cond:
        if (eval(*e.a[1], c).truthy()) return eval(*e.a[0], c);
        return e.a[2] ? eval(*e.a[2], c) : Value();
      case EK::Splat:
      case EK::KwSplat: fail("* and ** are only allowed in calls");
    }
    fail("bad expression node");
  }

  Flow exec(const std::vector<Stmt>& body, Ctx& c, std::string& out) {
    for (const Stmt& s : body) {
      c.tick();
      if (out.size() > c.max_out) fail("template output too large");
      switch (s.k) {
        case SK::Text: out += s.text; break;
        case SK::Out: out += to_str(eval(*s.e, c)); break;
        case SK::If:
          for (const auto& br : s.branches)
            if (!br.first || eval(*br.first, c).truthy()) {
              const Flow f = exec(br.second, c, out);
              if (f != Flow::Normal) return f;
              break;
            }
          break;
        case SK::For: {
          const Flow f = run_for(s, c, out);
          (void)f;
          break;
        }
        case SK::Set: {
          Value v = eval(*s.e, c);
          assign_targets(s.targets, v, c);
          break;
        }
        case SK::SetAttr: {
          Value ns = c.lookup(s.targets[0]);
          if (ns.t != Value::DictT || !ns.is_namespace) fail("cannot assign an attribute of a non-namespace object");
          ns.set(s.targets[1], eval(*s.e, c));
          break;
        }
        case SK::SetBlock: {
          std::string captured;
          exec(s.body, c, captured);
          assign_targets(s.targets, Value::str(captured), c);
          break;
        }
        case SK::Macro: define_macro(s, c); break;
        case SK::Break: return Flow::Break;
        case SK::Continue: return Flow::Continue;
      }
    }
    return Flow::Normal;
  }

 private:
  static void assign_targets(const std::vector<std::string>& t, const Value& v, Ctx& c) {
    if (t.size() == 1) {
      c.assign(t[0], v);
      return;
    }
    const List items = iterate(v);
    if (items.size() != t.size()) fail("cannot unpack " + std::to_string(items.size()) + " values");
    for (size_t k = 0; k < t.size(); ++k) c.assign(t[k], items[k]);
  }

  Flow run_for(const Stmt& s, Ctx& c, std::string& out) {
    const Value it = eval(*s.e, c);
    if (it.t == Value::None) fail("'NoneType' object is not iterable");
    List items = iterate(it);
    if (s.filter) {
      List kept;
      c.scopes.emplace_back();
      for (const Value& x : items) {
        assign_targets(s.targets, x, c);
        if (eval(*s.filter, c).truthy()) kept.push_back(x);
      }
      c.scopes.pop_back();
      items.swap(kept);
    }
    if (items.empty()) {
      exec(s.else_body, c, out);
      return Flow::Normal;
    }
    const int64_t n = static_cast<int64_t>(items.size());
    for (int64_t k = 0; k < n; ++k) {
      c.scopes.emplace_back();  // assignments in the body do not survive the iteration
      Value loop = Value::dict();
      loop.set("index", Value::integer(k + 1));
      loop.set("index0", Value::integer(k));
      loop.set("revindex", Value::integer(n - k));
      loop.set("revindex0", Value::integer(n - k - 1));
      loop.set("first", Value::boolean(k == 0));
      loop.set("last", Value::boolean(k == n - 1));
      loop.set("length", Value::integer(n));
      loop.set("previtem", k > 0 ? items[static_cast<size_t>(k - 1)] : Value());
      loop.set("nextitem", k + 1 < n ? items[static_cast<size_t>(k + 1)] : Value());
      loop.set("cycle", Value::func([k](const Args& a, const Kwargs&) {
        if (a.empty()) fail("cycle needs arguments");
        return a[static_cast<size_t>(k) % a.size()];
      }));
      c.assign("loop", loop);
      assign_targets(s.targets, items[static_cast<size_t>(k)], c);
      const Flow f = exec(s.body, c, out);
      c.scopes.pop_back();
      if (f == Flow::Break) break;
    }
    return Flow::Normal;
  }

  // Macros see the scopes that enclosed their definition, not their caller's locals.
  void define_macro(const Stmt& s, Ctx& c) {
    const Stmt* def = &s;
    Ctx* ctx = &c;
    const size_t depth = c.scopes.size();
    c.assign(s.text, Value::func([this, def, ctx, depth](const Args& a, const Kwargs& kw) {
      if (a.size() > def->targets.size()) fail("macro '" + def->text + "' takes " + std::to_string(def->targets.size()) + " arguments");
      auto saved = ctx->scopes;
      ctx->scopes.resize(std::min(depth, ctx->scopes.size()));
      ctx->scopes.emplace_back();
      for (size_t k = 0; k < def->targets.size(); ++k) {
        const Value* v = k < a.size() ? &a[k] : kwarg(kw, def->targets[k].c_str());
        if (v) ctx->assign(def->targets[k], *v);
        else if (def->defaults[k]) ctx->assign(def->targets[k], eval(*def->defaults[k], *ctx));
        else ctx->assign(def->targets[k], Value());
      }
      std::string o;
      exec(def->body, *ctx, o);
      ctx->scopes = std::move(saved);
      return Value::str(o);  // Markup only under autoescape, which chat templates render without
    }));
  }

  bool test(const std::string& n, const Value& v, const Args& a, Ctx&) {
    static const char* const unary[] = {"defined", "undefined", "none", "string", "number", "integer", "float",
                                        "boolean", "true", "false", "mapping", "iterable", "sequence", "callable",
                                        "lower", "upper", "odd", "even"};
    bool is_unary = false;
    for (const char* u : unary) is_unary = is_unary || n == u;
    if (known_test(n) && a.size() != (is_unary ? 0u : 1u))
      fail("test '" + n + "' takes " + (is_unary ? "no argument" : "one argument"));
    if (n == "defined") return v.t != Value::Undefined;
    if (n == "undefined") return v.t == Value::Undefined;
    if (n == "none") return v.t == Value::None;
    if (n == "string") return v.t == Value::Str;
    if (n == "number") return v.t == Value::Int || v.t == Value::Float || v.t == Value::Bool;
    if (n == "integer") return v.t == Value::Int;
    if (n == "float") return v.t == Value::Float;
    if (n == "boolean") return v.t == Value::Bool;
    if (n == "true") return v.t == Value::Bool && v.b;
    if (n == "false") return v.t == Value::Bool && !v.b;
    if (n == "mapping") return v.t == Value::DictT;
    if (n == "iterable") return v.t == Value::ListT || v.t == Value::DictT || v.t == Value::Str || v.t == Value::Undefined;
    if (n == "sequence") return v.t == Value::ListT || v.t == Value::DictT || v.t == Value::Str;
    if (n == "callable") return v.t == Value::Callable;
    if (n == "lower") return v.t == Value::Str && ascii_lower(v.s) == v.s;
    if (n == "upper") return v.t == Value::Str && ascii_upper(v.s) == v.s;
    if (n == "odd" || n == "even") return (as_int(v) % 2 != 0) == (n == "odd");
    if (a.empty()) fail("unknown test '" + n + "'");
    if (n == "divisibleby") return as_int(a[0]) != 0 && as_int(v) % as_int(a[0]) == 0;
    if (n == "equalto" || n == "eq" || n == "==" || n == "sameas") return equal(v, a[0]);
    if (n == "ne" || n == "!=") return !equal(v, a[0]);
    if (n == "lt" || n == "lessthan" || n == "<") return compare(v, a[0]) < 0;
    if (n == "le" || n == "<=") return compare(v, a[0]) <= 0;
    if (n == "gt" || n == "greaterthan" || n == ">") return compare(v, a[0]) > 0;
    if (n == "ge" || n == ">=") return compare(v, a[0]) >= 0;
    if (n == "in") return contains(a[0], v);
    fail("unknown test '" + n + "'");
  }

  List select(const Value& v, const Args& a, bool by_attr, bool keep, Ctx& c) {
    List out;
    size_t k = 0;
    std::string attr;
    if (by_attr) {
      if (a.empty() || a[0].t != Value::Str) fail("selectattr needs an attribute name");
      attr = a[0].s;
      k = 1;
    }
    const std::string tname = k < a.size() ? to_str(a[k]) : "";
    const Args targs(a.begin() + static_cast<long>(std::min(a.size(), k + 1)), a.end());
    for (const Value& x : iterate(v)) {
      const Value item = by_attr ? get_attr(x, attr) : x;
      const bool ok = tname.empty() ? item.truthy() : test(tname, item, targs, c);
      if (ok == keep) out.push_back(x);
    }
    return out;
  }

  Value filter(const std::string& n, const Value& v, const Args& a, const Kwargs& kw, Ctx& c) {
    const FilterSpec* spec = find_filter(n);
    if (!spec) fail("no filter named '" + n + "'");
    if (a.size() + kw.size() < spec->min_args || (spec->max_args >= 0 && a.size() > static_cast<size_t>(spec->max_args)))
      fail("filter '" + n + "' got a wrong number of arguments");
    for (const auto& kv : kw)
      if (std::find_if(spec->kwargs.begin(), spec->kwargs.end(), [&](const char* k) { return kv.first == k; }) ==
          spec->kwargs.end())
        fail("filter '" + n + "' got an unexpected keyword argument '" + kv.first + "'");
    if (n == "trim" || n == "strip") {
      if (v.t == Value::Undefined) return Value::str("");
      return Value::str(strip_chars(to_str(v), arg_str(a, kw, 0, "chars", kWs), true, true));
    }
    if (n == "length" || n == "count") {
      if (v.t == Value::Str) return Value::integer(static_cast<int64_t>(uni::length(v.s)));
      return Value::integer(static_cast<int64_t>(iterate(v).size()));
    }
    if (n == "tojson") {
      const Value* ind = arg(a, kw, 0, "indent");
      std::string o;
      tojson(o, v, ind && ind->t != Value::None ? static_cast<int>(as_int(*ind)) : -1, 0);
      return markup(o);
    }
    if (n == "upper") return Value::str(ascii_upper(to_str(v)));
    if (n == "lower") return Value::str(ascii_lower(to_str(v)));
    if (n == "title") return Value::str(title_case(to_str(v)));
    if (n == "capitalize") {
      std::string o = ascii_lower(to_str(v));
      if (!o.empty()) o[0] = static_cast<char>(toupper(static_cast<unsigned char>(o[0])));
      return Value::str(o);
    }
    if (n == "first" || n == "last") {
      const List items = iterate(v);
      if (items.empty()) return Value();
      return n == "first" ? items.front() : items.back();
    }
    if (n == "join") {
      const std::string sep = arg_str(a, kw, 0, "d", "");
      const Value* at = arg(a, kw, 1, "attribute");
      std::string o;
      bool first = true;
      for (const Value& x : iterate(v)) {
        o += (first ? "" : sep) + to_str(at ? get_attr(x, to_str(*at)) : x);
        first = false;
      }
      return Value::str(o);
    }
    if (n == "default" || n == "d") {
      const Value* dv = arg(a, kw, 0, "default_value");
      const Value* bo = arg(a, kw, 1, "boolean");
      const bool use = v.t == Value::Undefined || (bo && bo->truthy() && !v.truthy());
      return use ? (dv ? *dv : Value::str("")) : v;
    }
    if (n == "list") return Value::list(iterate(v));
    if (n == "int") {
      if (v.t == Value::Str) {
        char* end = nullptr;
        const long long x = strtoll(v.s.c_str(), &end, 10);
        if (end && *end == '\0' && !v.s.empty()) return Value::integer(x);
        const Value* dv = arg(a, kw, 0, "default");
        return dv ? *dv : Value::integer(0);
      }
      if (is_num(v)) return Value::integer(as_int(v));
      const Value* dv = arg(a, kw, 0, "default");
      return dv ? *dv : Value::integer(0);
    }
    if (n == "float") {
      if (is_num(v)) return Value::number(num(v));
      if (v.t == Value::Str) return Value::number(strtod(v.s.c_str(), nullptr));
      return Value::number(0);
    }
    if (n == "string") return Value::str(to_str(v));
    if (n == "items") {
      if (v.t == Value::Undefined) return Value::list();
      return (*get_attr(v, "items").fn)({}, {});
    }
    if (n == "reverse") {
      if (v.t == Value::Str) {
        auto cs = chars(v.s);
        std::string o;
        for (size_t k = cs.size(); k-- > 0;) o += cs[k];
        return Value::str(o);
      }
      List l = iterate(v);
      std::reverse(l.begin(), l.end());
      return Value::list(std::move(l));
    }
    if (n == "replace") {
      const Value* cnt = arg(a, kw, 2, "count");
      return Value::str(replace_all(to_str(v), arg_str(a, kw, 0, "old", ""), arg_str(a, kw, 1, "new", ""),
                                    cnt && cnt->t != Value::None ? as_int(*cnt) : -1));
    }
    if (n == "safe") return v.is_markup ? v : markup(to_str(v));
    if (n == "e" || n == "escape") return v.is_markup ? v : markup(escape_html(to_str(v)));
    if (n == "abs") {
      if (v.t == Value::Float) return Value::number(std::fabs(v.f));
      return Value::integer(std::llabs(as_int(v)));
    }
    if (n == "map") {
      List out;
      const Value* at = kwarg(kw, "attribute");
      for (const Value& x : iterate(v)) {
        if (at) {
          Value r = get_attr(x, to_str(*at));
          const Value* dflt = kwarg(kw, "default");
          out.push_back(r.t == Value::Undefined && dflt ? *dflt : r);
        } else {
          if (a.empty()) fail("map needs a filter name or attribute=");
          const Args rest(a.begin() + 1, a.end());
          out.push_back(filter(to_str(a[0]), x, rest, {}, c));
        }
      }
      return Value::list(std::move(out));
    }
    if (n == "selectattr" || n == "rejectattr") return Value::list(select(v, a, true, n == "selectattr", c));
    if (n == "select" || n == "reject") return Value::list(select(v, a, false, n == "select", c));
    if (n == "indent") {
      const Value* w = arg(a, kw, 0, "width");
      const Value* first = arg(a, kw, 1, "first");
      const Value* blank = arg(a, kw, 2, "blank");
      const std::string pad = w && w->t == Value::Str ? w->s : std::string(static_cast<size_t>(w ? as_int(*w) : 4), ' ');
      const std::string s = to_str(v);
      std::string o;
      size_t p = 0;
      bool line0 = true;
      while (p <= s.size()) {
        const size_t e = s.find('\n', p);
        const std::string ln = s.substr(p, e == std::string::npos ? std::string::npos : e - p);
        const bool add = line0 ? (first && first->truthy()) : (!ln.empty() || (blank && blank->truthy()));
        o += (add ? pad : "") + ln;
        if (e == std::string::npos) break;
        o += '\n';
        p = e + 1;
        line0 = false;
      }
      return Value::str(o);
    }
    if (n == "unique") {
      List out;
      for (const Value& x : iterate(v)) {
        bool seen = false;
        for (const Value& y : out) seen = seen || equal(x, y);
        if (!seen) out.push_back(x);
      }
      return Value::list(std::move(out));
    }
    fail("unknown filter '" + n + "'");
  }
};

Value make_namespace(const Args& a, const Kwargs& kw) {
  Value ns = Value::dict();
  ns.is_namespace = true;
  if (a.size() > 1) fail("namespace / dict take at most one positional argument");
  for (const Value& x : a) {
    if (x.t == Value::DictT) {
      for (const auto& kv : *x.d) ns.set(kv.first, kv.second);
    } else if (x.t == Value::ListT) {  // (key, value) pairs
      for (const Value& p : *x.l) {
        if (p.t != Value::ListT || p.l->size() != 2 || (*p.l)[0].t != Value::Str) fail("dict needs (key, value) pairs");
        ns.set((*p.l)[0].s, (*p.l)[1]);
      }
    } else {
      fail("namespace / dict need a mapping");
    }
  }
  for (const auto& kv : kw) ns.set(kv.first, kv.second);
  return ns;
}

}  // namespace

std::string to_str(const Value& v) {
  switch (v.t) {
    case Value::Undefined: return "";
    case Value::None: return "None";
    case Value::Bool: return v.b ? "True" : "False";
    case Value::Int: return std::to_string(v.i);
    case Value::Float: return float_repr(v.f);
    case Value::Str: return v.s;
    case Value::ListT:
    case Value::DictT: return repr(v);
    case Value::Callable: return "<function>";
  }
  return "";
}

Value from_json(const json::Value& v) {
  switch (v.type()) {
    case json::Value::Type::Null: return Value::none();
    case json::Value::Type::Bool: return Value::boolean(v.as_bool());
    case json::Value::Type::Int: return Value::integer(v.as_int());
    case json::Value::Type::Double: return Value::number(v.as_double());
    case json::Value::Type::String: return Value::str(v.as_string());
    case json::Value::Type::Array: {
      List l;
      for (const auto& x : v.as_array()) l.push_back(from_json(x));
      return Value::list(std::move(l));
    }
    case json::Value::Type::Object: {
      Value d = Value::dict();
      for (const auto& kv : v.as_object()) d.set(kv.first, from_json(kv.second));
      return d;
    }
  }
  return Value();
}

struct Template::Impl {
  std::vector<Stmt> body;
};

Template::Template(const std::string& source) : impl_(std::make_unique<Impl>()) {
  impl_->body = Builder(chunk_source(source)).build();
}
Template::~Template() = default;
Template::Template(Template&&) noexcept = default;
Template& Template::operator=(Template&&) noexcept = default;

std::string Template::render(const Value& globals) const {
  Ctx c;
  c.scopes.emplace_back();
  c.assign("range", Value::func([](const Args& a, const Kwargs&) {
    int64_t b = 0, e = 0, st = 1;
    if (a.size() == 1) e = as_int(a[0]);
    else if (a.size() >= 2) {
      b = as_int(a[0]);
      e = as_int(a[1]);
      if (a.size() > 2) st = as_int(a[2]);
    } else {
      fail("range needs arguments");
    }
    if (st == 0) fail("range step cannot be zero");
    List l;
    for (int64_t k = b; st > 0 ? k < e : k > e; k += st) {
      l.push_back(Value::integer(k));
      if (l.size() > 1000000) fail("range too large");
    }
    return Value::list(std::move(l));
  }));
  c.assign("namespace", Value::func(make_namespace));
  c.assign("dict", Value::func([](const Args& a, const Kwargs& kw) {
    Value d = make_namespace(a, kw);
    d.is_namespace = false;
    return d;
  }));
  c.assign("raise_exception", Value::func([](const Args& a, const Kwargs&) -> Value {
    fail("raise_exception: " + (a.empty() ? std::string() : to_str(a[0])));
  }));
  if (globals.t == Value::DictT)
    for (const auto& kv : *globals.d) c.assign(kv.first, kv.second);
  c.scopes.emplace_back();  // the template's own assignments
  std::string out;
  Eval ev;
  ev.exec(impl_->body, c, out);
  return out;
}

}  // namespace vmc::jinja
