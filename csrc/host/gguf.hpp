// GGUF v2/v3 container: memory-mapped reader and streaming writer.
//
// Reader capability matches the reference's GgufReader (src/core/gguf_reader.cpp:61 load,
// :98 read_header, :279 read_kv, :318 read_tensor_info): header, typed KV metadata including
// arrays, tensor infos, aligned data section. The writer has no counterpart in the reference's
// runtime; it produces the seeded random-init checkpoints used by tests and benchmarks.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <variant>
#include <vector>

#include "ggml_types.hpp"

namespace vmc {

enum class GValueType : uint32_t {
  UINT8 = 0, INT8 = 1, UINT16 = 2, INT16 = 3, UINT32 = 4, INT32 = 5, FLOAT32 = 6,
  BOOL = 7, STRING = 8, ARRAY = 9, UINT64 = 10, INT64 = 11, FLOAT64 = 12,
};

// A metadata value. Scalars are widened (integers to int64/uint64, floats to double);
// the original type is kept so that a round trip writes the same bytes.
struct GValue {
  GValueType type = GValueType::UINT32;
  GValueType elem_type = GValueType::UINT32;  // for ARRAY
  int64_t i = 0;
  uint64_t u = 0;
  double f = 0.0;
  bool b = false;
  std::string s;
  std::vector<int64_t> ai;
  std::vector<uint64_t> au;
  std::vector<double> af;
  std::vector<std::string> as;
  std::vector<uint8_t> ab;  // BOOL arrays
};

struct GTensorInfo {
  std::string name;
  std::vector<int64_t> ne;  // ne[0] is the innermost (row) dimension
  GType type = GType::F32;
  uint64_t offset = 0;      // relative to the data section
  uint64_t nbytes = 0;
  int64_t n_elements() const {
    int64_t n = 1;
    for (auto d : ne) n *= d;
    return n;
  }
};

class GgufFile {
 public:
  static std::shared_ptr<GgufFile> open(const std::string& path);
  ~GgufFile();

  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  const std::vector<std::string>& keys() const { return key_order_; }
  bool has(const std::string& key) const { return kv_.count(key) != 0; }
  const GValue& get(const std::string& key) const;
  const std::vector<GTensorInfo>& tensors() const { return tensors_; }
  const GTensorInfo* find_tensor(const std::string& name) const;
  const uint8_t* tensor_data(const GTensorInfo& t) const { return base_ + data_offset_ + t.offset; }
  uint64_t data_offset() const { return data_offset_; }
  uint64_t file_size() const { return size_; }
  const std::string& path() const { return path_; }

  // Typed getters with defaults (mirror the reference's get_u32/get_f32/get_str helpers).
  int64_t get_int(const std::string& key, int64_t def) const;
  double get_float(const std::string& key, double def) const;
  std::string get_str(const std::string& key, const std::string& def) const;

 private:
  GgufFile() = default;
  void parse();
  std::string path_;
  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  uint64_t size_ = 0;
  uint32_t version_ = 0;
  uint64_t alignment_ = 32;
  uint64_t data_offset_ = 0;
  std::map<std::string, GValue> kv_;
  std::vector<std::string> key_order_;
  std::vector<GTensorInfo> tensors_;
  std::map<std::string, size_t> tensor_index_;
};

// Streaming writer. Metadata and tensor infos are collected first; write() emits the header,
// then each tensor's bytes through a caller-supplied producer so that multi-GB checkpoints are
// never held in memory at once.
class GgufWriter {
 public:
  explicit GgufWriter(uint64_t alignment = 32) : alignment_(alignment) {}
  void set(const std::string& key, const GValue& v);
  void add_tensor(const std::string& name, const std::vector<int64_t>& ne, GType type);
  // producer(index, dst, nbytes) fills one tensor's bytes.
  template <class F>
  void write(const std::string& path, F&& producer);
  const std::vector<GTensorInfo>& tensors() const { return tensors_; }

 private:
  void write_header(FILE* fp);
  uint64_t alignment_;
  std::vector<std::pair<std::string, GValue>> kv_;
  std::vector<GTensorInfo> tensors_;
  uint64_t data_size_ = 0;
};

void gguf_write_value(FILE* fp, const GValue& v);

template <class F>
void GgufWriter::write(const std::string& path, F&& producer) {
  FILE* fp = fopen(path.c_str(), "wb");
  if (!fp) throw std::runtime_error("cannot open " + path + " for writing");
  write_header(fp);
  long pos = ftell(fp);
  uint64_t pad = (alignment_ - (static_cast<uint64_t>(pos) % alignment_)) % alignment_;
  std::vector<uint8_t> zeros(alignment_, 0);
  fwrite(zeros.data(), 1, pad, fp);
  std::vector<uint8_t> buf;
  uint64_t written = 0;
  for (size_t i = 0; i < tensors_.size(); ++i) {
    auto& t = tensors_[i];
    if (written < t.offset) {
      fwrite(zeros.data(), 1, t.offset - written, fp);
      written = t.offset;
    }
    buf.resize(t.nbytes);
    producer(i, buf.data(), t.nbytes);
    fwrite(buf.data(), 1, t.nbytes, fp);
    written += t.nbytes;
  }
  if (fclose(fp) != 0) throw std::runtime_error("write failed for " + path);
}

}  // namespace vmc
