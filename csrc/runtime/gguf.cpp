// GGUF index parser: header, metadata key/values and tensor directory.
// Tensor data is not touched here; Python memory-maps it from `data_offset`.
//
// Format (GGUF v2/v3, as read by openmini-server/src/model/inference/gguf.rs:1357-1372,1658-2030):
//   u32 magic "GGUF" | u32 version | u64 n_tensors | u64 n_kv
//   kv:     string key | u32 type | value        (types 0..12; 8 = string, 9 = array)
//   tensor: string name | u32 n_dims | u64 dims[n_dims] | u32 ggml type | u64 offset
//   data starts at the next multiple of general.alignment (default 32).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;

namespace om_rt {

class Reader {
 public:
  explicit Reader(const std::string& path) {
    f_ = std::fopen(path.c_str(), "rb");
    if (!f_) throw std::runtime_error("cannot open " + path);
  }
  ~Reader() {
    if (f_) std::fclose(f_);
  }
  void read(void* dst, size_t n) {
    if (std::fread(dst, 1, n, f_) != n) throw std::runtime_error("GGUF: unexpected end of file");
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
    if (n > (1ull << 30)) throw std::runtime_error("GGUF: string too long");
    std::string s(n, '\0');
    if (n) read(&s[0], n);
    return s;
  }
  uint64_t pos() const { return pos_; }

 private:
  FILE* f_ = nullptr;
  uint64_t pos_ = 0;
};

static py::object read_value(Reader& r, uint32_t type) {
  switch (type) {
    case 0: return py::int_(r.get<uint8_t>());
    case 1: return py::int_(r.get<int8_t>());
    case 2: return py::int_(r.get<uint16_t>());
    case 3: return py::int_(r.get<int16_t>());
    case 4: return py::int_(r.get<uint32_t>());
    case 5: return py::int_(r.get<int32_t>());
    case 6: return py::float_(r.get<float>());
    case 7: return py::bool_(r.get<uint8_t>() != 0);
    case 8: return py::str(r.str());
    case 9: {
      const uint32_t et = r.get<uint32_t>();
      const uint64_t n = r.get<uint64_t>();
      py::list l;
      for (uint64_t i = 0; i < n; ++i) l.append(read_value(r, et));
      return std::move(l);
    }
    case 10: return py::int_(r.get<uint64_t>());
    case 11: return py::int_(r.get<int64_t>());
    case 12: return py::float_(r.get<double>());
    default: throw std::runtime_error("GGUF: unknown metadata type " + std::to_string(type));
  }
}

// Returns {"version", "metadata": {k: v}, "tensors": [(name, dims, type, offset)], "data_offset", "alignment"}
py::dict parse_gguf(const std::string& path) {
  Reader r(path);
  const uint32_t magic = r.get<uint32_t>();
  if (magic != 0x46554747u) throw std::runtime_error("not a GGUF file (bad magic)");
  const uint32_t version = r.get<uint32_t>();
  if (version < 2 || version > 3) throw std::runtime_error("unsupported GGUF version " + std::to_string(version));
  const uint64_t nt = r.get<uint64_t>();
  const uint64_t nkv = r.get<uint64_t>();
  py::dict meta;
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nkv; ++i) {
    std::string key = r.str();
    const uint32_t t = r.get<uint32_t>();
    py::object v = read_value(r, t);
    if (key == "general.alignment") alignment = v.cast<uint64_t>();
    meta[py::str(key)] = v;
  }
  py::list tensors;
  for (uint64_t i = 0; i < nt; ++i) {
    std::string name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    if (nd > 8) throw std::runtime_error("GGUF: too many dims");
    py::list dims;
    for (uint32_t d = 0; d < nd; ++d) dims.append(r.get<uint64_t>());
    const uint32_t type = r.get<uint32_t>();
    const uint64_t off = r.get<uint64_t>();
    tensors.append(py::make_tuple(name, dims, type, off));
  }
  const uint64_t data_off = (r.pos() + alignment - 1) / alignment * alignment;
  py::dict out;
  out["version"] = version;
  out["metadata"] = meta;
  out["tensors"] = tensors;
  out["data_offset"] = data_off;
  out["alignment"] = alignment;
  return out;
}

}  // namespace om_rt

void bind_gguf(py::module_& m) { m.def("parse_gguf", &om_rt::parse_gguf); }
