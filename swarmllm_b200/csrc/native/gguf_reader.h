// Memory-mapped GGUF reader (format version 2/3).
//
// Parses the header, the typed metadata key/values and the tensor table, and
// hands out zero-copy views of tensor bytes.  The reference reads GGUF through
// candle's gguf_file plus its own shard layer (src/inference/split/gguf_meta.rs,
// src/inference/split/shard_reader.rs:36,56); this reader is written from the
// GGUF specification (ggml docs/gguf.md): little-endian, strings are
// (u64 length, bytes), tensor data aligned to general.alignment (default 32).
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <variant>
#include <vector>

namespace pybind11 {
class module_;
}

namespace swarm_native {

struct GgufValue;
using GgufArray = std::vector<GgufValue>;
struct GgufValue {
  // type ids follow the GGUF spec: 0 u8,1 i8,2 u16,3 i16,4 u32,5 i32,6 f32,7 bool,
  // 8 string,9 array,10 u64,11 i64,12 f64
  uint32_t type = 0;
  std::variant<uint64_t, int64_t, double, bool, std::string, GgufArray> v;
};

struct GgufTensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // ne[0] innermost
  uint32_t type = 0;
  uint64_t offset = 0;         // relative to the data section
  uint64_t nbytes = 0;
};

class GgufFile {
 public:
  explicit GgufFile(const std::string& path);
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  uint64_t data_offset() const { return data_offset_; }
  const std::vector<std::pair<std::string, GgufValue>>& metadata() const { return kv_; }
  const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
  const uint8_t* base() const { return base_; }
  uint64_t size() const { return size_; }

  static uint64_t tensor_nbytes(uint32_t type, const std::vector<uint64_t>& dims);

 private:
  const uint8_t* base_ = nullptr;
  uint64_t size_ = 0;
  int fd_ = -1;
  uint32_t version_ = 0;
  uint64_t alignment_ = 32;
  uint64_t data_offset_ = 0;
  std::vector<std::pair<std::string, GgufValue>> kv_;
  std::vector<GgufTensorInfo> tensors_;
};

void bind_gguf(pybind11::module_& m);

}  // namespace swarm_native
