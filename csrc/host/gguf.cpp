#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace vmc {

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  template <class T>
  T read() {
    if (p + sizeof(T) > end) throw std::runtime_error("gguf: truncated file");
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string read_str() {
    uint64_t n = read<uint64_t>();
    if (n > static_cast<uint64_t>(end - p)) throw std::runtime_error("gguf: bad string length");
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

void read_scalar_into(Cursor& c, GValueType t, GValue& v, bool array_elem) {
  auto push_i = [&](int64_t x) { if (array_elem) v.ai.push_back(x); else v.i = x; };
  auto push_u = [&](uint64_t x) { if (array_elem) v.au.push_back(x); else v.u = x; };
  auto push_f = [&](double x) { if (array_elem) v.af.push_back(x); else v.f = x; };
  switch (t) {
    case GValueType::UINT8: push_u(c.read<uint8_t>()); break;
    case GValueType::INT8: push_i(c.read<int8_t>()); break;
    case GValueType::UINT16: push_u(c.read<uint16_t>()); break;
    case GValueType::INT16: push_i(c.read<int16_t>()); break;
    case GValueType::UINT32: push_u(c.read<uint32_t>()); break;
    case GValueType::INT32: push_i(c.read<int32_t>()); break;
    case GValueType::UINT64: push_u(c.read<uint64_t>()); break;
    case GValueType::INT64: push_i(c.read<int64_t>()); break;
    case GValueType::FLOAT32: push_f(c.read<float>()); break;
    case GValueType::FLOAT64: push_f(c.read<double>()); break;
    case GValueType::BOOL: {
      uint8_t b = c.read<uint8_t>();
      if (array_elem) v.ab.push_back(b); else v.b = b != 0;
      break;
    }
    case GValueType::STRING: {
      std::string s = c.read_str();
      if (array_elem) v.as.push_back(std::move(s)); else v.s = std::move(s);
      break;
    }
    default:
      throw std::runtime_error("gguf: bad value type " + std::to_string(static_cast<uint32_t>(t)));
  }
}

GValue read_value(Cursor& c, GValueType t) {
  GValue v;
  v.type = t;
  if (t == GValueType::ARRAY) {
    auto et = static_cast<GValueType>(c.read<uint32_t>());
    uint64_t n = c.read<uint64_t>();
    v.elem_type = et;
    if (et == GValueType::ARRAY) throw std::runtime_error("gguf: nested arrays unsupported");
    for (uint64_t k = 0; k < n; ++k) read_scalar_into(c, et, v, true);
  } else {
    read_scalar_into(c, t, v, false);
  }
  return v;
}

}  // namespace

std::shared_ptr<GgufFile> GgufFile::open(const std::string& path) {
  std::shared_ptr<GgufFile> f(new GgufFile());
  f->path_ = path;
  f->fd_ = ::open(path.c_str(), O_RDONLY);
  if (f->fd_ < 0) throw std::runtime_error("gguf: cannot open " + path);
  struct stat st;
  if (fstat(f->fd_, &st) != 0) throw std::runtime_error("gguf: stat failed for " + path);
  f->size_ = static_cast<uint64_t>(st.st_size);
  void* m = mmap(nullptr, f->size_, PROT_READ, MAP_SHARED, f->fd_, 0);
  if (m == MAP_FAILED) throw std::runtime_error("gguf: mmap failed for " + path);
  f->base_ = static_cast<const uint8_t*>(m);
  f->parse();
  return f;
}

GgufFile::~GgufFile() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
  if (fd_ >= 0) ::close(fd_);
}

void GgufFile::parse() {
  Cursor c{base_, base_ + size_};
  if (c.read<uint32_t>() != kMagic) throw std::runtime_error("gguf: bad magic in " + path_);
  version_ = c.read<uint32_t>();
  if (version_ < 2 || version_ > 3) throw std::runtime_error("gguf: unsupported version " + std::to_string(version_));
  uint64_t n_tensors = c.read<uint64_t>();
  uint64_t n_kv = c.read<uint64_t>();
  for (uint64_t k = 0; k < n_kv; ++k) {
    std::string key = c.read_str();
    auto t = static_cast<GValueType>(c.read<uint32_t>());
    GValue v = read_value(c, t);
    if (kv_.count(key) == 0) key_order_.push_back(key);
    kv_[key] = std::move(v);
  }
  if (has("general.alignment")) {
    const auto& a = get("general.alignment");
    alignment_ = a.u ? a.u : static_cast<uint64_t>(a.i);
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1))) throw std::runtime_error("gguf: bad alignment");
  }
  for (uint64_t k = 0; k < n_tensors; ++k) {
    GTensorInfo ti;
    ti.name = c.read_str();
    uint32_t nd = c.read<uint32_t>();
    if (nd > 4) throw std::runtime_error("gguf: tensor rank > 4: " + ti.name);
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t n = c.read<uint64_t>();
      if (n > (1ull << 40)) throw std::runtime_error("gguf: implausible dimension of tensor " + ti.name);
      ti.ne.push_back(static_cast<int64_t>(n));
    }
    uint32_t ty = c.read<uint32_t>();
    if (!gtype_known(ty)) throw std::runtime_error("gguf: unsupported tensor type " + std::to_string(ty) + " for " + ti.name);
    ti.type = static_cast<GType>(ty);
    ti.offset = c.read<uint64_t>();
    ti.nbytes = gtype_row_bytes(ti.type, ti.ne.empty() ? 1 : ti.ne[0]);
    for (size_t d = 1; d < ti.ne.size(); ++d)  // a size that does not fit in 64 bits cannot be in the file
      if (__builtin_mul_overflow(ti.nbytes, static_cast<uint64_t>(ti.ne[d]), &ti.nbytes))
        throw std::runtime_error("gguf: size of tensor " + ti.name + " overflows");
    tensor_index_[ti.name] = tensors_.size();
    tensors_.push_back(std::move(ti));
  }
  uint64_t pos = static_cast<uint64_t>(c.p - base_);
  data_offset_ = (pos + alignment_ - 1) / alignment_ * alignment_;
  for (auto& t : tensors_) {  // compared without sums that could wrap around
    if (data_offset_ > size_ || t.offset > size_ - data_offset_ || t.nbytes > size_ - data_offset_ - t.offset)
      throw std::runtime_error("gguf: tensor " + t.name + " extends past end of file");
  }
}

const GValue& GgufFile::get(const std::string& key) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) throw std::runtime_error("gguf: missing key " + key);
  return it->second;
}

const GTensorInfo* GgufFile::find_tensor(const std::string& name) const {
  auto it = tensor_index_.find(name);
  return it == tensor_index_.end() ? nullptr : &tensors_[it->second];
}

int64_t GgufFile::get_int(const std::string& key, int64_t def) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return def;
  const auto& v = it->second;
  switch (v.type) {
    case GValueType::UINT8: case GValueType::UINT16: case GValueType::UINT32: case GValueType::UINT64:
      return static_cast<int64_t>(v.u);
    case GValueType::INT8: case GValueType::INT16: case GValueType::INT32: case GValueType::INT64:
      return v.i;
    case GValueType::BOOL: return v.b ? 1 : 0;
    case GValueType::FLOAT32: case GValueType::FLOAT64: return static_cast<int64_t>(v.f);
    default: return def;
  }
}

double GgufFile::get_float(const std::string& key, double def) const {
  auto it = kv_.find(key);
  if (it == kv_.end()) return def;
  const auto& v = it->second;
  if (v.type == GValueType::FLOAT32 || v.type == GValueType::FLOAT64) return v.f;
  return static_cast<double>(get_int(key, static_cast<int64_t>(def)));
}

std::string GgufFile::get_str(const std::string& key, const std::string& def) const {
  auto it = kv_.find(key);
  if (it == kv_.end() || it->second.type != GValueType::STRING) return def;
  return it->second.s;
}

// ----------------------------------------------------------------------------------------------
// Writer

namespace {
template <class T>
void put(FILE* fp, T v) { fwrite(&v, sizeof(T), 1, fp); }
void put_str(FILE* fp, const std::string& s) {
  put<uint64_t>(fp, s.size());
  fwrite(s.data(), 1, s.size(), fp);
}
void write_scalar(FILE* fp, GValueType t, const GValue& v, size_t idx, bool arr) {
  auto gi = [&]() { return arr ? v.ai.at(idx) : v.i; };
  auto gu = [&]() { return arr ? v.au.at(idx) : v.u; };
  auto gf = [&]() { return arr ? v.af.at(idx) : v.f; };
  switch (t) {
    case GValueType::UINT8: put<uint8_t>(fp, static_cast<uint8_t>(gu())); break;
    case GValueType::INT8: put<int8_t>(fp, static_cast<int8_t>(gi())); break;
    case GValueType::UINT16: put<uint16_t>(fp, static_cast<uint16_t>(gu())); break;
    case GValueType::INT16: put<int16_t>(fp, static_cast<int16_t>(gi())); break;
    case GValueType::UINT32: put<uint32_t>(fp, static_cast<uint32_t>(gu())); break;
    case GValueType::INT32: put<int32_t>(fp, static_cast<int32_t>(gi())); break;
    case GValueType::UINT64: put<uint64_t>(fp, gu()); break;
    case GValueType::INT64: put<int64_t>(fp, gi()); break;
    case GValueType::FLOAT32: put<float>(fp, static_cast<float>(gf())); break;
    case GValueType::FLOAT64: put<double>(fp, gf()); break;
    case GValueType::BOOL: put<uint8_t>(fp, arr ? v.ab.at(idx) : (v.b ? 1 : 0)); break;
    case GValueType::STRING: put_str(fp, arr ? v.as.at(idx) : v.s); break;
    default: throw std::runtime_error("gguf writer: bad scalar type");
  }
}
size_t array_len(const GValue& v) {
  switch (v.elem_type) {
    case GValueType::STRING: return v.as.size();
    case GValueType::BOOL: return v.ab.size();
    case GValueType::FLOAT32: case GValueType::FLOAT64: return v.af.size();
    case GValueType::UINT8: case GValueType::UINT16: case GValueType::UINT32: case GValueType::UINT64:
      return v.au.size();
    default: return v.ai.size();
  }
}
}  // namespace

void gguf_write_value(FILE* fp, const GValue& v) {
  put<uint32_t>(fp, static_cast<uint32_t>(v.type));
  if (v.type == GValueType::ARRAY) {
    put<uint32_t>(fp, static_cast<uint32_t>(v.elem_type));
    size_t n = array_len(v);
    put<uint64_t>(fp, n);
    for (size_t k = 0; k < n; ++k) write_scalar(fp, v.elem_type, v, k, true);
  } else {
    write_scalar(fp, v.type, v, 0, false);
  }
}

void GgufWriter::set(const std::string& key, const GValue& v) {
  for (auto& kv : kv_) {
    if (kv.first == key) { kv.second = v; return; }
  }
  kv_.emplace_back(key, v);
}

void GgufWriter::add_tensor(const std::string& name, const std::vector<int64_t>& ne, GType type) {
  GTensorInfo ti;
  ti.name = name;
  ti.ne = ne;
  ti.type = type;
  ti.nbytes = gtype_row_bytes(type, ne.empty() ? 1 : ne[0]);
  for (size_t d = 1; d < ne.size(); ++d) ti.nbytes *= static_cast<uint64_t>(ne[d]);
  ti.offset = (data_size_ + alignment_ - 1) / alignment_ * alignment_;
  data_size_ = ti.offset + ti.nbytes;
  tensors_.push_back(std::move(ti));
}

void GgufWriter::write_header(FILE* fp) {
  put<uint32_t>(fp, kMagic);
  put<uint32_t>(fp, 3);
  put<uint64_t>(fp, tensors_.size());
  bool has_align = false;
  for (auto& kv : kv_) has_align |= kv.first == "general.alignment";
  put<uint64_t>(fp, kv_.size() + (has_align || alignment_ == 32 ? 0 : 1));
  for (auto& kv : kv_) {
    put_str(fp, kv.first);
    gguf_write_value(fp, kv.second);
  }
  if (!has_align && alignment_ != 32) {
    put_str(fp, "general.alignment");
    GValue a;
    a.type = GValueType::UINT32;
    a.u = alignment_;
    gguf_write_value(fp, a);
  }
  for (auto& t : tensors_) {
    put_str(fp, t.name);
    put<uint32_t>(fp, static_cast<uint32_t>(t.ne.size()));
    for (auto d : t.ne) put<uint64_t>(fp, static_cast<uint64_t>(d));
    put<uint32_t>(fp, static_cast<uint32_t>(t.type));
    put<uint64_t>(fp, t.offset);
  }
}

}  // namespace vmc
