#include "gguf_reader.h"

#include <fcntl.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <memory>
#include <stdexcept>

namespace py = pybind11;

namespace swarm_native {

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  template <typename T>
  T get() {
    if (p + sizeof(T) > end) throw std::runtime_error("gguf: truncated file");
    T v;
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (p + n > end) throw std::runtime_error("gguf: truncated string");
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

GgufValue read_value(Cursor& c, uint32_t type, int depth = 0) {
  if (depth > 4) throw std::runtime_error("gguf: nested arrays too deep");
  GgufValue v;
  v.type = type;
  switch (type) {
    case 0: v.v = (uint64_t)c.get<uint8_t>(); break;
    case 1: v.v = (int64_t)c.get<int8_t>(); break;
    case 2: v.v = (uint64_t)c.get<uint16_t>(); break;
    case 3: v.v = (int64_t)c.get<int16_t>(); break;
    case 4: v.v = (uint64_t)c.get<uint32_t>(); break;
    case 5: v.v = (int64_t)c.get<int32_t>(); break;
    case 6: v.v = (double)c.get<float>(); break;
    case 7: v.v = (bool)(c.get<uint8_t>() != 0); break;
    case 8: v.v = c.str(); break;
    case 9: {
      const uint32_t et = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      GgufArray arr;
      arr.reserve(n);
      for (uint64_t i = 0; i < n; ++i) arr.push_back(read_value(c, et, depth + 1));
      v.v = std::move(arr);
      break;
    }
    case 10: v.v = c.get<uint64_t>(); break;
    case 11: v.v = c.get<int64_t>(); break;
    case 12: v.v = c.get<double>(); break;
    default: throw std::runtime_error("gguf: unknown metadata type " + std::to_string(type));
  }
  return v;
}

// (values per block, bytes per block) for the GGML types this engine knows.
std::pair<uint64_t, uint64_t> block_shape(uint32_t t) {
  switch (t) {
    case 0: return {1, 4};     // F32
    case 1: return {1, 2};     // F16
    case 2: return {32, 18};   // Q4_0
    case 3: return {32, 20};   // Q4_1
    case 6: return {32, 22};   // Q5_0
    case 7: return {32, 24};   // Q5_1
    case 8: return {32, 34};   // Q8_0
    case 10: return {256, 84};  // Q2_K
    case 11: return {256, 110}; // Q3_K
    case 12: return {256, 144}; // Q4_K
    case 13: return {256, 176}; // Q5_K
    case 14: return {256, 210}; // Q6_K
    case 20: return {32, 18};   // IQ4_NL
    case 23: return {256, 136}; // IQ4_XS
    case 24: return {1, 1};     // I8
    case 25: return {1, 2};     // I16
    case 26: return {1, 4};     // I32
    case 27: return {1, 8};     // I64
    case 28: return {1, 8};     // F64
    case 30: return {1, 2};     // BF16
    case 39: return {32, 17};   // MXFP4
    default: return {0, 0};
  }
}

}  // namespace

uint64_t GgufFile::tensor_nbytes(uint32_t type, const std::vector<uint64_t>& dims) {
  auto [bv, bb] = block_shape(type);
  if (bv == 0) throw std::runtime_error("gguf: unsupported tensor type " + std::to_string(type));
  uint64_t n = 1;
  for (auto d : dims) n *= d;
  if (dims.empty() || dims[0] % bv != 0) throw std::runtime_error("gguf: row not a whole number of blocks");
  return n / bv * bb;
}

GgufFile::GgufFile(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("gguf: cannot open " + path);
  struct stat st;
  if (fstat(fd_, &st) != 0) throw std::runtime_error("gguf: stat failed");
  size_ = (uint64_t)st.st_size;
  void* m = mmap(nullptr, size_, PROT_READ, MAP_SHARED, fd_, 0);
  if (m == MAP_FAILED) {
    ::close(fd_);
    throw std::runtime_error("gguf: mmap failed");
  }
  base_ = static_cast<const uint8_t*>(m);
  Cursor c{base_, base_ + size_};
  if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("gguf: bad magic");
  version_ = c.get<uint32_t>();
  if (version_ < 2 || version_ > 3) throw std::runtime_error("gguf: unsupported version");
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    const uint32_t t = c.get<uint32_t>();
    GgufValue v = read_value(c, t);
    if (key == "general.alignment" && (t == 4 || t == 5 || t == 10))
      alignment_ = std::holds_alternative<uint64_t>(v.v) ? std::get<uint64_t>(v.v)
                                                         : (uint64_t)std::get<int64_t>(v.v);
    kv_.emplace_back(std::move(key), std::move(v));
  }
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensorInfo ti;
    ti.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (nd > 4) throw std::runtime_error("gguf: too many dims");
    for (uint32_t d = 0; d < nd; ++d) ti.dims.push_back(c.get<uint64_t>());
    ti.type = c.get<uint32_t>();
    ti.offset = c.get<uint64_t>();
    ti.nbytes = tensor_nbytes(ti.type, ti.dims);
    tensors_.push_back(std::move(ti));
  }
  const uint64_t pos = (uint64_t)(c.p - base_);
  data_offset_ = (pos + alignment_ - 1) / alignment_ * alignment_;
  for (auto& t : tensors_)
    if (data_offset_ + t.offset + t.nbytes > size_) throw std::runtime_error("gguf: tensor out of file: " + t.name);
}

GgufFile::~GgufFile() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
  if (fd_ >= 0) ::close(fd_);
}

static py::object value_to_py(const GgufValue& v) {
  return std::visit(
      [&](auto&& x) -> py::object {
        using T = std::decay_t<decltype(x)>;
        if constexpr (std::is_same_v<T, GgufArray>) {
          py::list l;
          for (auto& e : x) l.append(value_to_py(e));
          return l;
        } else if constexpr (std::is_same_v<T, std::string>) {
          return py::bytes(x).attr("decode")("utf-8", "replace");
        } else {
          return py::cast(x);
        }
      },
      v.v);
}

void bind_gguf(py::module_& m) {
  py::class_<GgufFile, std::shared_ptr<GgufFile>>(m, "GgufFile")
      .def(py::init<const std::string&>())
      .def_property_readonly("version", &GgufFile::version)
      .def_property_readonly("alignment", &GgufFile::alignment)
      .def_property_readonly("data_offset", &GgufFile::data_offset)
      .def("metadata",
           [](const GgufFile& f) {
             py::dict d;
             for (auto& [k, v] : f.metadata()) d[py::str(k)] = value_to_py(v);
             return d;
           })
      .def("metadata_types",
           [](const GgufFile& f) {
             py::dict d;
             for (auto& [k, v] : f.metadata()) {
               uint32_t et = 0;
               if (v.type == 9) {
                 auto& arr = std::get<GgufArray>(v.v);
                 et = arr.empty() ? 0 : arr[0].type;
               }
               d[py::str(k)] = py::make_tuple(v.type, et);
             }
             return d;
           })
      .def("tensors",
           [](const GgufFile& f) {
             py::list l;
             for (auto& t : f.tensors())
               l.append(py::make_tuple(t.name, t.dims, t.type, t.offset, t.nbytes));
             return l;
           })
      .def("tensor_bytes",
           [](std::shared_ptr<GgufFile> f, const std::string& name) {
             for (auto& t : f->tensors()) {
               if (t.name != name) continue;
               const uint8_t* p = f->base() + f->data_offset() + t.offset;
               py::capsule owner(new std::shared_ptr<GgufFile>(f), [](void* q) {
                 delete static_cast<std::shared_ptr<GgufFile>*>(q);
               });
               py::array_t<uint8_t> a({(py::ssize_t)t.nbytes}, {1}, p, owner);
               a.attr("setflags")(py::arg("write") = false);  // the mapping is read-only
               return a;
             }
             throw py::key_error(name);
           })
      .def_static("tensor_nbytes", &GgufFile::tensor_nbytes);
}

}  // namespace swarm_native
