// Native GGUF header parser over a read-only memory map.
//
// Parity: the reference's GgufReader (barq_core/src/gguf.rs:250-372): magic, version <= 3,
// tensor and key/value counts, the 13 metadata value types with nested arrays, tensor infos and
// the aligned start of the data section.  The reference reads the whole file into memory and
// dequantizes every tensor to f32 at load; here the file is mapped once and the whole mapping is
// returned as a zero-copy uint8 torch tensor whose storage owns the map (munmap runs when the last
// view of any tensor in the file is gone), so tensors are slices of the page cache.
//
// parse(path) -> (version, metadata: dict, metadata_types: dict, tensors: list of
//                 (name, shape tuple, ggml type, offset), alignment, data_offset, file: uint8 tensor)
// Malformed input raises ValueError with the byte position; every read is bounds-checked.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <torch/extension.h>

namespace py = pybind11;

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint64_t kMaxCount = 10000000ull;
constexpr uint64_t kMaxString = 1ull << 32;
constexpr int kMaxDepth = 8;

enum VT : uint32_t {
  U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7,
  STR = 8, ARR = 9, U64 = 10, I64 = 11, F64 = 12
};

struct Mapping {
  void* base = nullptr;
  size_t size = 0;
  ~Mapping() {
    if (base != nullptr && base != MAP_FAILED) munmap(base, size);
  }
};

struct Cursor {
  const uint8_t* p;
  size_t n;
  size_t pos = 0;

  [[noreturn]] void fail(const std::string& what) const {
    throw py::value_error(what + " (at byte " + std::to_string(pos) + ")");
  }
  void need(uint64_t k) const {
    if (k > n || pos > n - k) fail("truncated GGUF: need " + std::to_string(k) + " more bytes");
  }
  template <class T>
  T get() {
    need(sizeof(T));
    T v;
    std::memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::pair<const char*, size_t> str() {
    uint64_t len = get<uint64_t>();
    if (len > kMaxString) fail("implausible string length " + std::to_string(len));
    need(len);
    const char* s = reinterpret_cast<const char*>(p + pos);
    pos += len;
    return {s, static_cast<size_t>(len)};
  }
};

py::object utf8(const char* s, size_t n) {
  PyObject* o = PyUnicode_DecodeUTF8(s, static_cast<Py_ssize_t>(n), "replace");
  if (o == nullptr) throw py::error_already_set();
  return py::reinterpret_steal<py::object>(o);
}

size_t scalar_size(uint32_t t) {
  switch (t) {
    case U8: case I8: case BOOL: return 1;
    case U16: case I16: return 2;
    case U32: case I32: case F32: return 4;
    case U64: case I64: case F64: return 8;
    default: return 0;
  }
}

py::object scalar(Cursor& c, uint32_t t) {
  switch (t) {
    case U8: return py::int_(c.get<uint8_t>());
    case I8: return py::int_(c.get<int8_t>());
    case U16: return py::int_(c.get<uint16_t>());
    case I16: return py::int_(c.get<int16_t>());
    case U32: return py::int_(c.get<uint32_t>());
    case I32: return py::int_(c.get<int32_t>());
    case F32: return py::float_(c.get<float>());
    case BOOL: return py::bool_(c.get<uint8_t>() != 0);
    case U64: return py::int_(c.get<uint64_t>());
    case I64: return py::int_(c.get<int64_t>());
    case F64: return py::float_(c.get<double>());
    default: c.fail("unknown GGUF value type " + std::to_string(t));
  }
}

template <class T>
py::object numeric_array(Cursor& c, uint64_t count) {
  py::array_t<T> a(static_cast<py::ssize_t>(count));
  std::memcpy(a.mutable_data(), c.p + c.pos, count * sizeof(T));
  c.pos += count * sizeof(T);
  return std::move(a);
}

py::object value(Cursor& c, uint32_t t, int depth) {
  if (t == STR) {
    auto s = c.str();
    return utf8(s.first, s.second);
  }
  if (t != ARR) return scalar(c, t);
  if (depth > kMaxDepth) c.fail("array nesting too deep");
  uint32_t et = c.get<uint32_t>();
  uint64_t count = c.get<uint64_t>();
  size_t es = scalar_size(et);
  if (es > 0) {
    if (count > (c.n - c.pos) / es) c.fail("truncated GGUF array");
    if (count <= 64) {  // short arrays come back as lists, long numeric ones as numpy arrays
      py::list l;
      for (uint64_t i = 0; i < count; ++i) l.append(scalar(c, et));
      return std::move(l);
    }
    switch (et) {
      case U8: return numeric_array<uint8_t>(c, count);
      case I8: return numeric_array<int8_t>(c, count);
      case U16: return numeric_array<uint16_t>(c, count);
      case I16: return numeric_array<int16_t>(c, count);
      case U32: return numeric_array<uint32_t>(c, count);
      case I32: return numeric_array<int32_t>(c, count);
      case F32: return numeric_array<float>(c, count);
      case BOOL: return numeric_array<bool>(c, count);
      case U64: return numeric_array<uint64_t>(c, count);
      case I64: return numeric_array<int64_t>(c, count);
      case F64: return numeric_array<double>(c, count);
    }
  }
  if (et != STR && et != ARR) c.fail("unknown GGUF array element type " + std::to_string(et));
  // every element takes at least 8 bytes (a length or a header), which bounds the loop
  if (count > (c.n - c.pos) / 8) c.fail("truncated GGUF array");
  py::list l;
  for (uint64_t i = 0; i < count; ++i) l.append(value(c, et, depth + 1));
  return std::move(l);
}

py::tuple parse_buffer(const uint8_t* data, size_t size) {
  Cursor c{data, size};
  uint32_t magic = c.get<uint32_t>();
  if (magic != kMagic) {
    char buf[16];
    std::snprintf(buf, sizeof(buf), "0x%08x", magic);
    c.fail(std::string("bad magic ") + buf);
  }
  uint32_t version = c.get<uint32_t>();
  if (version < 1 || version > 3) c.fail("unsupported GGUF version " + std::to_string(version));
  if (version == 1) c.fail("GGUF v1 (32-bit counts) is not supported");
  uint64_t n_tensors = c.get<uint64_t>();
  uint64_t n_kv = c.get<uint64_t>();
  if (n_tensors > kMaxCount || n_kv > kMaxCount) c.fail("implausible tensor/kv count");
  py::dict md, mdt;
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < n_kv; ++i) {
    auto k = c.str();
    py::object key = utf8(k.first, k.second);
    uint32_t t = c.get<uint32_t>();
    if (t > F64) c.fail("unknown GGUF value type " + std::to_string(t));
    py::object v = value(c, t, 0);
    if (k.second == 17 && std::memcmp(k.first, "general.alignment", 17) == 0 && t != STR && t != ARR)
      alignment = py::cast<uint64_t>(v);
    md[key] = v;
    mdt[key] = py::int_(t);
  }
  if (alignment == 0 || (alignment & (alignment - 1)) != 0) c.fail("alignment must be a power of two");
  py::list tensors;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    auto nm = c.str();
    uint32_t nd = c.get<uint32_t>();
    if (nd > 8) c.fail("tensor with " + std::to_string(nd) + " dims");
    py::tuple shape(nd);
    for (uint32_t d = 0; d < nd; ++d) shape[d] = py::int_(c.get<uint64_t>());
    uint32_t type = c.get<uint32_t>();
    uint64_t off = c.get<uint64_t>();
    tensors.append(py::make_tuple(utf8(nm.first, nm.second), shape, type, off));
  }
  uint64_t data_offset = (c.pos + alignment - 1) / alignment * alignment;
  return py::make_tuple(version, md, mdt, tensors, alignment, data_offset);
}

py::tuple parse(const std::string& path) {
  int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) throw py::value_error(path + ": cannot open (" + std::strerror(errno) + ")");
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw py::value_error(path + ": cannot stat");
  }
  auto map = std::make_shared<Mapping>();
  map->size = static_cast<size_t>(st.st_size);
  if (map->size < 24) {
    close(fd);
    throw py::value_error(path + ": too small for a GGUF header");
  }
  map->base = mmap(nullptr, map->size, PROT_READ, MAP_SHARED, fd, 0);
  close(fd);
  if (map->base == MAP_FAILED) throw py::value_error(path + ": mmap failed");
  py::tuple head = parse_buffer(static_cast<const uint8_t*>(map->base), map->size);
  // the storage's deleter holds the mapping; torch never writes through this (read-only) view
  torch::Tensor file = torch::from_blob(map->base, {static_cast<int64_t>(map->size)},
                                        [map](void*) mutable { map.reset(); },
                                        torch::TensorOptions().dtype(torch::kUInt8));
  py::list out;
  for (auto h : head) out.append(h);
  out.append(file);
  return py::tuple(out);
}

py::tuple parse_bytes(py::bytes b) {
  std::string s = b;
  return parse_buffer(reinterpret_cast<const uint8_t*>(s.data()), s.size());
}

}  // namespace

void register_tokenizer(py::module_& m);  // tokenizer_native.cpp
void register_grammar(py::module_& m);    // grammar_native.cpp
void register_kvcache(py::module_& m);    // kvcache_native.cpp
void register_scheduler(py::module_& m);  // scheduler_native.cpp
void register_sampler(py::module_& m);    // sampler_native.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "barq native runtime pieces (GGUF parser, tokenizer merge loops, grammar recognizer, KV block pool, "
            "radix prefix cache, continuous-batching scheduler core, host sampler chain)";
  register_tokenizer(m);
  register_grammar(m);
  register_kvcache(m);
  register_scheduler(m);
  register_sampler(m);
  m.def("gguf_parse", &parse, "memory-map and parse a GGUF file");
  m.def("gguf_parse_bytes", &parse_bytes, "parse a GGUF header held in memory (no tensor data view)");
}
