// safetensors container (HuggingFace checkpoints): memory-mapped reader.
//
// Counterpart of the reference's SafeTensorsLoader (src/model/model_loader.cpp:78-296). The layout
// is the format's public specification: an 8-byte little-endian header length N, N bytes of JSON
// ({name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {string: string}};
// offsets relative to the first byte after the header), then the row-major tensor bytes. The
// header is parsed by a small JSON reader of our own; every byte range is checked against the
// tensor's shape and the file size before a view of it is handed out.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace vmc {

struct StTensorInfo {
  std::string name;
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0;  // absolute file offsets
  uint64_t end = 0;
};

// Bytes per element of a safetensors dtype name (0 if unknown).
int st_dtype_size(const std::string& dtype);

class SafetensorsFile {
 public:
  static std::shared_ptr<SafetensorsFile> open(const std::string& path);
  ~SafetensorsFile();

  const std::vector<StTensorInfo>& tensors() const { return tensors_; }
  const std::map<std::string, std::string>& metadata() const { return metadata_; }
  const StTensorInfo* find(const std::string& name) const;
  const uint8_t* data(const StTensorInfo& t) const { return base_ + t.begin; }
  uint64_t file_size() const { return size_; }
  const std::string& path() const { return path_; }

 private:
  SafetensorsFile() = default;
  void parse();
  std::string path_;
  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  uint64_t size_ = 0;
  std::vector<StTensorInfo> tensors_;
  std::map<std::string, size_t> index_;
  std::map<std::string, std::string> metadata_;
};

}  // namespace vmc
