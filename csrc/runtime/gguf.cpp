// GGUF (v2/v3) container reader: header, metadata key/values, tensor table.
//
// Format (little endian): "GGUF" magic, u32 version, u64 tensor_count,
// u64 kv_count, kv pairs (gguf string key, u32 value type, value), tensor
// infos (name, u32 n_dims, u64 dims[n_dims] innermost first, u32 ggml type,
// u64 offset relative to the data section), padding to general.alignment
// (default 32), then the data section.  Tensor bytes are not read here: the
// Python side maps them with numpy.memmap at data_offset + offset.
//
// Reference behaviour: candle's gguf_file reader as used by
// crates/engine/src/executor/candle.rs:682-841 (config synthesis from
// {arch}.* keys) and crates/engine/src/bin/inspect_gguf.rs:1-118.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace {

enum GGUFType : uint32_t {
  T_UINT8 = 0, T_INT8 = 1, T_UINT16 = 2, T_INT16 = 3, T_UINT32 = 4, T_INT32 = 5, T_FLOAT32 = 6,
  T_BOOL = 7, T_STRING = 8, T_ARRAY = 9, T_UINT64 = 10, T_INT64 = 11, T_FLOAT64 = 12,
};

// ggml tensor types: (block elements, block bytes)
struct TypeInfo {
  const char* name;
  int block;
  int bytes;
};
TypeInfo ggml_type_info(uint32_t t) {
  switch (t) {
    case 0: return {"F32", 1, 4};
    case 1: return {"F16", 1, 2};
    case 2: return {"Q4_0", 32, 18};
    case 3: return {"Q4_1", 32, 20};
    case 6: return {"Q5_0", 32, 22};
    case 7: return {"Q5_1", 32, 24};
    case 8: return {"Q8_0", 32, 34};
    case 9: return {"Q8_1", 32, 36};
    case 10: return {"Q2_K", 256, 84};
    case 11: return {"Q3_K", 256, 110};
    case 12: return {"Q4_K", 256, 144};
    case 13: return {"Q5_K", 256, 176};
    case 14: return {"Q6_K", 256, 210};
    case 15: return {"Q8_K", 256, 292};
    case 24: return {"I8", 1, 1};
    case 25: return {"I16", 1, 2};
    case 26: return {"I32", 1, 4};
    case 27: return {"I64", 1, 8};
    case 28: return {"F64", 1, 8};
    case 30: return {"BF16", 1, 2};
    default: return {"UNKNOWN", 0, 0};
  }
}

class Reader {
 public:
  explicit Reader(const std::string& path) {
    f_ = std::fopen(path.c_str(), "rb");
    if (!f_) throw std::runtime_error("gguf: cannot open " + path);
  }
  ~Reader() {
    if (f_) std::fclose(f_);
  }
  void read(void* dst, size_t n) {
    if (std::fread(dst, 1, n, f_) != n) throw std::runtime_error("gguf: truncated file");
    pos_ += n;
  }
  template <typename T>
  T get() {
    T v;
    read(&v, sizeof(T));
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (n > (1ull << 32)) throw std::runtime_error("gguf: string too long");
    std::string s(n, '\0');
    if (n) read(&s[0], n);
    return s;
  }
  uint64_t pos() const { return pos_; }

 private:
  std::FILE* f_ = nullptr;
  uint64_t pos_ = 0;
};

py::object read_scalar(Reader& r, uint32_t t) {
  switch (t) {
    case T_UINT8: return py::int_(r.get<uint8_t>());
    case T_INT8: return py::int_(r.get<int8_t>());
    case T_UINT16: return py::int_(r.get<uint16_t>());
    case T_INT16: return py::int_(r.get<int16_t>());
    case T_UINT32: return py::int_(r.get<uint32_t>());
    case T_INT32: return py::int_(r.get<int32_t>());
    case T_FLOAT32: return py::float_(r.get<float>());
    case T_BOOL: return py::bool_(r.get<uint8_t>() != 0);
    case T_STRING: {
      std::string s = r.str();
      return py::str(PyUnicode_DecodeUTF8(s.data(), s.size(), "replace"), false);
    }
    case T_UINT64: return py::int_(r.get<uint64_t>());
    case T_INT64: return py::int_(r.get<int64_t>());
    case T_FLOAT64: return py::float_(r.get<double>());
    default: throw std::runtime_error("gguf: unknown value type " + std::to_string(t));
  }
}

py::object read_value(Reader& r, uint32_t t) {
  if (t != T_ARRAY) return read_scalar(r, t);
  const uint32_t et = r.get<uint32_t>();
  const uint64_t n = r.get<uint64_t>();
  py::list out;
  for (uint64_t i = 0; i < n; ++i) out.append(read_value(r, et));
  return out;
}

py::dict read_gguf(const std::string& path) {
  Reader r(path);
  char magic[4];
  r.read(magic, 4);
  if (std::memcmp(magic, "GGUF", 4) != 0) throw std::runtime_error("gguf: bad magic (not a GGUF file)");
  const uint32_t version = r.get<uint32_t>();
  if (version < 2 || version > 3) throw std::runtime_error("gguf: unsupported version " + std::to_string(version));
  const uint64_t n_tensors = r.get<uint64_t>();
  const uint64_t n_kv = r.get<uint64_t>();
  py::dict meta;
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = r.str();
    const uint32_t t = r.get<uint32_t>();
    meta[py::str(key)] = read_value(r, t);
  }
  uint64_t alignment = 32;
  if (meta.contains("general.alignment")) alignment = meta["general.alignment"].cast<uint64_t>();
  if (alignment == 0 || (alignment & (alignment - 1))) throw std::runtime_error("gguf: bad alignment");
  py::list tensors;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    std::string name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (nd > 8) throw std::runtime_error("gguf: too many dims");
    std::vector<uint64_t> ne(nd);
    uint64_t nel = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      ne[d] = r.get<uint64_t>();
      nel *= ne[d];
    }
    const uint32_t type = r.get<uint32_t>();
    const uint64_t offset = r.get<uint64_t>();
    const TypeInfo ti = ggml_type_info(type);
    py::dict t;
    t["name"] = name;
    t["ne"] = ne;  // ggml order (innermost first)
    std::vector<uint64_t> shape(ne.rbegin(), ne.rend());
    t["shape"] = shape;  // row-major (numpy / torch) order
    t["type"] = type;
    t["type_name"] = ti.name;
    t["offset"] = offset;
    t["n_elements"] = nel;
    t["n_bytes"] = ti.block ? (nel / ti.block) * ti.bytes : 0;
    tensors.append(t);
  }
  const uint64_t data_offset = (r.pos() + alignment - 1) / alignment * alignment;
  py::dict out;
  out["version"] = version;
  out["metadata"] = meta;
  out["tensors"] = tensors;
  out["alignment"] = alignment;
  out["data_offset"] = data_offset;
  return out;
}

}  // namespace

void register_gguf(py::module_& m) {
  m.def("read_gguf", &read_gguf, "Parse a GGUF file's header, metadata and tensor table");
  m.def("ggml_type_name", [](uint32_t t) { return std::string(ggml_type_info(t).name); });
  m.def("ggml_type_block", [](uint32_t t) {
    const TypeInfo ti = ggml_type_info(t);
    return py::make_tuple(ti.block, ti.bytes);
  });
}
