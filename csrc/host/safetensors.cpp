// safetensors reader (see safetensors.hpp).
#include "safetensors.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace vmc {
namespace {

constexpr uint64_t kMaxHeader = 100ull << 20;

// Minimal JSON reader for the header: objects, arrays, strings (with escapes), integers, and
// skipping of other scalars (floats, true / false / null) wherever they appear.
class Json {
 public:
  Json(const char* p, const char* e, const std::string& path) : p_(p), e_(e), path_(path) {}

  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool peek(char c) {
    ws();
    return p_ < e_ && *p_ == c;
  }
  void expect(char c) {
    ws();
    if (p_ >= e_ || *p_ != c) fail(std::string("expected '") + c + "'");
    ++p_;
  }
  [[noreturn]] void fail(const std::string& what) const {
    throw std::runtime_error("safetensors: bad header in " + path_ + ": " + what);
  }

  std::string str() {
    expect('"');
    std::string out;
    while (true) {
      if (p_ >= e_) fail("unterminated string");
      char c = *p_++;
      if (c == '"') return out;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (p_ >= e_) fail("bad escape");
      char x = *p_++;
      switch (x) {
        case '"': out.push_back('"'); break;
        case '\\': out.push_back('\\'); break;
        case '/': out.push_back('/'); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': append_utf8(out, code_unit()); break;
        default: fail("bad escape");
      }
    }
  }

  int64_t integer() {
    ws();
    bool neg = false;
    if (p_ < e_ && *p_ == '-') {
      neg = true;
      ++p_;
    }
    if (p_ >= e_ || *p_ < '0' || *p_ > '9') fail("expected an integer");
    int64_t v = 0;
    while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
      if (v > (INT64_MAX - 9) / 10) fail("integer overflow");
      v = v * 10 + (*p_++ - '0');
    }
    if (p_ < e_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) fail("expected an integer");
    return neg ? -v : v;
  }

  std::vector<int64_t> int_array() {
    std::vector<int64_t> v;
    expect('[');
    if (peek(']')) {
      ++p_;
      return v;
    }
    while (true) {
      v.push_back(integer());
      if (peek(',')) {
        ++p_;
        continue;
      }
      expect(']');
      return v;
    }
  }

  // Skip any JSON value.
  void skip() {
    ws();
    if (p_ >= e_) fail("unexpected end");
    char c = *p_;
    if (c == '"') {
      str();
    } else if (c == '{' || c == '[') {
      const char close = c == '{' ? '}' : ']';
      ++p_;
      if (peek(close)) {
        ++p_;
        return;
      }
      while (true) {
        if (c == '{') {
          str();
          expect(':');
        }
        skip();
        if (peek(',')) {
          ++p_;
          continue;
        }
        expect(close);
        return;
      }
    } else {
      while (p_ < e_ && *p_ != ',' && *p_ != '}' && *p_ != ']' && *p_ != ' ' && *p_ != '\n') ++p_;
    }
  }

  bool at_end() {
    ws();
    return p_ >= e_;
  }

 private:
  uint32_t hex4() {
    if (e_ - p_ < 4) fail("bad \\u escape");
    uint32_t v = 0;
    for (int i = 0; i < 4; ++i) {
      char h = *p_++;
      v <<= 4;
      if (h >= '0' && h <= '9') v |= h - '0';
      else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
      else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
      else fail("bad \\u escape");
    }
    return v;
  }
  uint32_t code_unit() {
    uint32_t u = hex4();
    if (u >= 0xD800 && u < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
      p_ += 2;
      uint32_t lo = hex4();
      if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
      u = 0x10000 + ((u - 0xD800) << 10) + (lo - 0xDC00);
    }
    return u;
  }
  static void append_utf8(std::string& s, uint32_t u) {
    if (u < 0x80) {
      s.push_back(static_cast<char>(u));
    } else if (u < 0x800) {
      s.push_back(static_cast<char>(0xC0 | (u >> 6)));
      s.push_back(static_cast<char>(0x80 | (u & 0x3F)));
    } else if (u < 0x10000) {
      s.push_back(static_cast<char>(0xE0 | (u >> 12)));
      s.push_back(static_cast<char>(0x80 | ((u >> 6) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | (u & 0x3F)));
    } else {
      s.push_back(static_cast<char>(0xF0 | (u >> 18)));
      s.push_back(static_cast<char>(0x80 | ((u >> 12) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | ((u >> 6) & 0x3F)));
      s.push_back(static_cast<char>(0x80 | (u & 0x3F)));
    }
  }

  const char* p_;
  const char* e_;
  const std::string& path_;
};

}  // namespace

int st_dtype_size(const std::string& d) {
  if (d == "F64" || d == "I64" || d == "U64") return 8;
  if (d == "F32" || d == "I32" || d == "U32") return 4;
  if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
  if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
  return 0;
}

std::shared_ptr<SafetensorsFile> SafetensorsFile::open(const std::string& path) {
  std::shared_ptr<SafetensorsFile> f(new SafetensorsFile());
  f->path_ = path;
  f->fd_ = ::open(path.c_str(), O_RDONLY);
  if (f->fd_ < 0) throw std::runtime_error("safetensors: cannot open " + path);
  struct stat st;
  if (fstat(f->fd_, &st) != 0) throw std::runtime_error("safetensors: stat failed for " + path);
  f->size_ = static_cast<uint64_t>(st.st_size);
  if (f->size_ < 8) throw std::runtime_error("safetensors: " + path + " is shorter than 8 bytes");
  void* m = mmap(nullptr, f->size_, PROT_READ, MAP_SHARED, f->fd_, 0);
  if (m == MAP_FAILED) throw std::runtime_error("safetensors: mmap failed for " + path);
  f->base_ = static_cast<const uint8_t*>(m);
  f->parse();
  return f;
}

SafetensorsFile::~SafetensorsFile() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
  if (fd_ >= 0) ::close(fd_);
}

const StTensorInfo* SafetensorsFile::find(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

void SafetensorsFile::parse() {
  uint64_t n = 0;
  std::memcpy(&n, base_, 8);  // little-endian host
  if (n > kMaxHeader || 8 + n > size_) throw std::runtime_error("safetensors: bad header length in " + path_);
  const uint64_t data0 = 8 + n;
  const char* h = reinterpret_cast<const char*>(base_ + 8);
  Json j(h, h + n, path_);
  j.expect('{');
  if (j.peek('}')) return;
  while (true) {
    std::string name = j.str();
    j.expect(':');
    if (name == "__metadata__") {
      j.expect('{');
      if (!j.peek('}')) {
        while (true) {
          std::string k = j.str();
          j.expect(':');
          metadata_[k] = j.str();
          if (j.peek(',')) {
            j.expect(',');
            continue;
          }
          break;
        }
      }
      j.expect('}');
    } else {
      StTensorInfo t;
      t.name = name;
      std::vector<int64_t> offs;
      bool has_dtype = false, has_shape = false;
      j.expect('{');
      while (!j.peek('}')) {
        std::string k = j.str();
        j.expect(':');
        if (k == "dtype") {
          t.dtype = j.str();
          has_dtype = true;
        } else if (k == "shape") {
          t.shape = j.int_array();
          has_shape = true;
        } else if (k == "data_offsets") {
          offs = j.int_array();
        } else {
          j.skip();
        }
        if (j.peek(',')) j.expect(',');
      }
      j.expect('}');
      const int es = st_dtype_size(t.dtype);
      if (!has_dtype || !has_shape || offs.size() != 2 || es == 0)
        throw std::runtime_error("safetensors: tensor " + name + " in " + path_ + " has a bad entry");
      uint64_t numel = 1, nbytes = 0;
      for (int64_t d : t.shape) {
        if (d < 0) throw std::runtime_error("safetensors: negative dimension in " + name);
        if (__builtin_mul_overflow(numel, static_cast<uint64_t>(d), &numel))
          throw std::runtime_error("safetensors: size of " + name + " overflows");
      }
      if (__builtin_mul_overflow(numel, static_cast<uint64_t>(es), &nbytes))
        throw std::runtime_error("safetensors: size of " + name + " overflows");
      if (offs[0] < 0 || offs[1] < offs[0] || static_cast<uint64_t>(offs[1] - offs[0]) != nbytes ||
          static_cast<uint64_t>(offs[1]) > size_ - data0)
        throw std::runtime_error("safetensors: tensor " + name + " byte range does not match its shape in " + path_);
      t.begin = data0 + static_cast<uint64_t>(offs[0]);
      t.end = data0 + static_cast<uint64_t>(offs[1]);
      if (index_.count(name)) throw std::runtime_error("safetensors: duplicate tensor " + name);
      index_[name] = tensors_.size();
      tensors_.push_back(std::move(t));
    }
    if (j.peek(',')) {
      j.expect(',');
      continue;
    }
    j.expect('}');
    break;
  }
  if (!j.at_end()) throw std::runtime_error("safetensors: trailing bytes after the header JSON in " + path_);
}

}  // namespace vmc
