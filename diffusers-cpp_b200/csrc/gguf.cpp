// GGUF reader (see gguf.hpp).  The parser is bounds-checked at every read:
// a truncated or corrupt file fails with DCPP_ERR_INVALID_ARG naming what
// was being read, never with an out-of-range access.
#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <filesystem>

#include "runtime.hpp"

namespace dcpp {

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr int kMaxDims = 4;               // ggml tensors have at most four dimensions

enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

// Little-endian cursor over the mapping; every read checks the bounds.
struct Cursor {
  const uint8_t* p;
  uint64_t size, pos = 0;
  const std::string& path;

  [[noreturn]] void truncated(const char* what) const {
    fail(DCPP_ERR_INVALID_ARG, "Failed to initialize GGUF file: " + path + ": truncated while reading " + what +
                                   " at byte " + std::to_string(pos));
  }
  void need(uint64_t n, const char* what) const {
    if (n > size - pos) truncated(what);
  }
  template <class T>
  T get(const char* what) {
    need(sizeof(T), what);
    T v;
    memcpy(&v, p + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str(const char* what) {
    const uint64_t n = get<uint64_t>(what);
    need(n, what);
    std::string s(reinterpret_cast<const char*>(p + pos), n);
    pos += n;
    return s;
  }
};

uint64_t scalar_bytes(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
  }
}

bool is_float(uint32_t t) { return t == kF32 || t == kF64; }

// One scalar of type t as int64 / double.
void read_scalar(Cursor& c, uint32_t t, int64_t& i, double& f) {
  switch (t) {
    case kU8: i = c.get<uint8_t>("a u8 value"); break;
    case kI8: i = c.get<int8_t>("an i8 value"); break;
    case kBool: i = c.get<uint8_t>("a bool value") != 0; break;
    case kU16: i = c.get<uint16_t>("a u16 value"); break;
    case kI16: i = c.get<int16_t>("an i16 value"); break;
    case kU32: i = c.get<uint32_t>("a u32 value"); break;
    case kI32: i = c.get<int32_t>("an i32 value"); break;
    case kU64: i = static_cast<int64_t>(c.get<uint64_t>("a u64 value")); break;
    case kI64: i = c.get<int64_t>("an i64 value"); break;
    case kF32: f = c.get<float>("an f32 value"); break;
    case kF64: f = c.get<double>("an f64 value"); break;
    default: break;
  }
  if (is_float(t)) i = static_cast<int64_t>(f);
  else f = static_cast<double>(i);
}

void read_value(Cursor& c, uint32_t type, GGUFValue& v, const std::string& key) {
  v.type = type;
  if (type == kString) {
    v.s = c.str("a string value");
    return;
  }
  if (type == kArray) {
    v.elem_type = c.get<uint32_t>("an array element type");
    if (v.elem_type == kArray)
      fail(DCPP_ERR_UNSUPPORTED, "Failed to initialize GGUF file: " + c.path + ": nested array in '" + key + "'");
    v.count = c.get<uint64_t>("an array length");
    if (v.elem_type == kString) {
      // Each string takes at least its 8-byte length.
      if (v.count > (c.size - c.pos) / 8) c.truncated("a string array");
      v.as.reserve(v.count);
      for (uint64_t k = 0; k < v.count; ++k) v.as.push_back(c.str("a string array element"));
      return;
    }
    const uint64_t eb = scalar_bytes(v.elem_type);
    if (eb == 0)
      fail(DCPP_ERR_INVALID_ARG, "Failed to initialize GGUF file: " + c.path + ": array of unknown type " +
                                     std::to_string(v.elem_type) + " in '" + key + "'");
    if (v.count > (c.size - c.pos) / eb) c.truncated("an array");
    if (is_float(v.elem_type)) v.af.resize(v.count);
    else v.ai.resize(v.count);
    for (uint64_t k = 0; k < v.count; ++k) {
      int64_t i = 0;
      double f = 0;
      read_scalar(c, v.elem_type, i, f);
      if (is_float(v.elem_type)) v.af[k] = f;
      else v.ai[k] = i;
    }
    return;
  }
  if (scalar_bytes(type) == 0)
    fail(DCPP_ERR_INVALID_ARG, "Failed to initialize GGUF file: " + c.path + ": value of unknown type " +
                                   std::to_string(type) + " in '" + key + "'");
  read_scalar(c, type, v.i, v.f);
}

std::string resolve_path(const std::string& path) {
  namespace fs = std::filesystem;
  std::error_code ec;
  if (!fs::exists(path, ec)) fail(DCPP_ERR_NOT_FOUND, "No such GGUF file in path: " + path);
  if (!fs::is_directory(path, ec)) return path;
  std::vector<std::string> found;
  for (const auto& e : fs::directory_iterator(path, ec))
    if (e.is_regular_file(ec) && e.path().extension() == ".gguf") found.push_back(e.path().string());
  if (found.empty()) fail(DCPP_ERR_NOT_FOUND, "No such GGUF file in path: " + path);
  std::sort(found.begin(), found.end());
  return found.front();
}

}  // namespace

GGUFTypeSize gguf_type_size(int type) {
  // ggml's type traits for the types a GGUF checkpoint of this pipeline can
  // hold (block elements, block bytes).
  switch (type) {
    case 0: return {1, 4};      // F32
    case 1: return {1, 2};      // F16
    case 2: return {32, 18};    // Q4_0
    case 3: return {32, 20};    // Q4_1
    case 6: return {32, 22};    // Q5_0
    case 7: return {32, 24};    // Q5_1
    case 8: return {32, 34};    // Q8_0
    case 9: return {32, 40};    // Q8_1
    case 10: return {256, 84};  // Q2_K
    case 11: return {256, 110}; // Q3_K
    case 12: return {256, 144}; // Q4_K
    case 13: return {256, 176}; // Q5_K
    case 14: return {256, 210}; // Q6_K
    case 15: return {256, 292}; // Q8_K
    case 24: return {1, 1};     // I8
    case 25: return {1, 2};     // I16
    case 26: return {1, 4};     // I32
    case 27: return {1, 8};     // I64
    case 28: return {1, 8};     // F64
    case 30: return {1, 2};     // BF16
    default: return {0, 0};
  }
}

std::vector<int64_t> GGUFTensorInfo::shape() const {
  int n = 0;
  for (int i = 0; i < static_cast<int>(ne.size()); ++i)
    if (ne[i] > 1 || (i == 0 && ne[0] == 1)) n = i + 1;
  if (n == 0) fail(DCPP_ERR_INVALID_ARG, "GGUF tensor '" + name + "' has invalid dimensions");
  std::vector<int64_t> s(n);
  for (int r = 0; r < n; ++r) s[r] = ne[n - 1 - r];
  return s;
}

GGUFFile::GGUFFile(const std::string& path) {
  path_ = resolve_path(path);
  const int fd = ::open(path_.c_str(), O_RDONLY);
  if (fd < 0) fail(DCPP_ERR_NOT_FOUND, "Failed to open GGUF file: " + path_ + ": " + strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    ::close(fd);
    fail(DCPP_ERR_INVALID_ARG, "Failed to initialize GGUF file: " + path_ + ": empty or unreadable");
  }
  size_ = static_cast<uint64_t>(st.st_size);
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) fail(DCPP_ERR_INVALID_ARG, "Failed to open GGUF file: " + path_ + ": mmap failed");
  base_ = static_cast<const uint8_t*>(m);
  try {
    Cursor c{base_, size_, 0, path_};
    const std::string bad = "Failed to initialize GGUF file: " + path_ + ": ";
    if (c.get<uint32_t>("the magic") != kMagic) fail(DCPP_ERR_INVALID_ARG, bad + "not a GGUF file (bad magic)");
    version_ = c.get<uint32_t>("the version");
    if (version_ == 1) fail(DCPP_ERR_UNSUPPORTED, bad + "GGUF version 1 is not supported");
    if ((version_ & 0xFFFFu) == 0 && version_ != 0)
      fail(DCPP_ERR_UNSUPPORTED, bad + "big-endian GGUF is not supported");
    if (version_ < 2 || version_ > 3) fail(DCPP_ERR_UNSUPPORTED, bad + "unknown GGUF version " + std::to_string(version_));
    const uint64_t n_tensors = c.get<uint64_t>("the tensor count");
    const uint64_t n_kv = c.get<uint64_t>("the metadata count");
    // Lower bounds on an entry's size keep corrupt counts from allocating.
    if (n_kv > (size_ - c.pos) / 12) c.truncated("the metadata");
    kv_.reserve(n_kv);
    for (uint64_t k = 0; k < n_kv; ++k) {
      std::string key = c.str("a metadata key");
      const uint32_t type = c.get<uint32_t>("a metadata type");
      GGUFValue v;
      read_value(c, type, v, key);
      if (key == "general.alignment") {
        if (type != kU32 || v.i <= 0 || (v.i & (v.i - 1)) != 0)
          fail(DCPP_ERR_INVALID_ARG, bad + "general.alignment must be a power-of-two u32");
        alignment_ = static_cast<uint64_t>(v.i);
      }
      kv_.emplace_back(std::move(key), std::move(v));
    }
    if (n_tensors > (size_ - c.pos) / 24) c.truncated("the tensor infos");
    tensors_.reserve(n_tensors);
    for (uint64_t t = 0; t < n_tensors; ++t) {
      GGUFTensorInfo ti;
      ti.name = c.str("a tensor name");
      const uint32_t nd = c.get<uint32_t>("a tensor's dimension count");
      if (nd == 0 || nd > kMaxDims)
        fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "' has " + std::to_string(nd) + " dimensions");
      ti.ne.assign(kMaxDims, 1);
      for (uint32_t d = 0; d < nd; ++d) {
        const uint64_t e = c.get<uint64_t>("a tensor dimension");
        if (e > (1ull << 40)) fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "' has an invalid dimension");
        ti.ne[d] = static_cast<int64_t>(e);
      }
      ti.type = static_cast<int>(c.get<uint32_t>("a tensor type"));
      ti.offset = c.get<uint64_t>("a tensor offset");
      const GGUFTypeSize ts = gguf_type_size(ti.type);
      if (ts.block == 0)
        fail(DCPP_ERR_UNSUPPORTED, bad + "tensor '" + ti.name + "' has unknown ggml type " + std::to_string(ti.type));
      if (ti.ne[0] % ts.block != 0)
        fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "': row length " + std::to_string(ti.ne[0]) +
                                       " is not a multiple of the block size " + std::to_string(ts.block));
      uint64_t rows = 1;
      for (int d = 1; d < kMaxDims; ++d) {
        if (ti.ne[d] != 0 && rows > (1ull << 50) / static_cast<uint64_t>(ti.ne[d]))
          fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "' is too large");
        rows *= static_cast<uint64_t>(ti.ne[d]);
      }
      ti.nbytes = rows * static_cast<uint64_t>(ti.ne[0] / ts.block) * static_cast<uint64_t>(ts.bytes);
      if (index_.count(ti.name)) fail(DCPP_ERR_INVALID_ARG, bad + "duplicate tensor name '" + ti.name + "'");
      index_[ti.name] = static_cast<int64_t>(tensors_.size());
      tensors_.push_back(std::move(ti));
    }
    data_offset_ = (c.pos + alignment_ - 1) / alignment_ * alignment_;
    for (auto& ti : tensors_) {
      if (ti.offset % alignment_ != 0)
        fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "' data is not aligned to " + std::to_string(alignment_));
      if (data_offset_ > size_ || ti.offset > size_ - data_offset_ || ti.nbytes > size_ - data_offset_ - ti.offset)
        fail(DCPP_ERR_INVALID_ARG, bad + "tensor '" + ti.name + "' data is not within the file bounds");
      ti.offset += data_offset_;
    }
  } catch (...) {
    munmap(const_cast<uint8_t*>(base_), size_);
    base_ = nullptr;
    throw;
  }
}

GGUFFile::~GGUFFile() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
}

const GGUFValue* GGUFFile::find_kv(const std::string& key) const {
  for (const auto& kv : kv_)
    if (kv.first == key) return &kv.second;
  return nullptr;
}

int64_t GGUFFile::find_tensor(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? -1 : it->second;
}

int64_t gguf_bind_all(const GGUFFile& file, const GGUFSetParam& set_param, int64_t* unused) {
  int64_t bound = 0, skipped = 0;
  for (const auto& t : file.tensors()) {
    try {
      set_param(t.name, t.type, t.shape(), file.data(t), static_cast<size_t>(t.nbytes));
      ++bound;
    } catch (const Error& e) {
      if (e.status != DCPP_ERR_NOT_FOUND) throw;
      ++skipped;
    }
  }
  if (unused) *unused = skipped;
  return bound;
}

}  // namespace dcpp

// ------------------------------------------------------------------ C ABI
namespace {

const dcpp::GGUFValue* kv_value(const dcpp_gguf* f, const char* key, int64_t index, dcpp_status* st) {
  *st = DCPP_OK;
  if (!f || !f->file || !key) {
    *st = DCPP_ERR_INVALID_ARG;
    return nullptr;
  }
  const dcpp::GGUFValue* v = f->file->find_kv(key);
  if (!v) {
    *st = DCPP_ERR_NOT_FOUND;
    return nullptr;
  }
  const bool array = v->type == dcpp::kArray;
  if ((index < 0) == array || (array && static_cast<uint64_t>(index) >= v->count)) {
    *st = DCPP_ERR_INVALID_ARG;
    return nullptr;
  }
  return v;
}

}  // namespace

extern "C" {

dcpp_status dcpp_gguf_open(const char* path, dcpp_gguf** out, char* err, size_t err_cap) {
  if (!out) return DCPP_ERR_INVALID_ARG;
  *out = nullptr;
  auto report = [&](const std::string& m) {
    if (err && err_cap) {
      const size_t n = std::min(err_cap - 1, m.size());
      memcpy(err, m.data(), n);
      err[n] = 0;
    }
  };
  if (!path) {
    report("dcpp_gguf_open: null path");
    return DCPP_ERR_INVALID_ARG;
  }
  try {
    auto* g = new dcpp_gguf();
    try {
      g->file.reset(new dcpp::GGUFFile(path));
    } catch (...) {
      delete g;
      throw;
    }
    *out = g;
    report("");
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    report(e.what());
    return e.status;
  } catch (const std::exception& e) {
    report(e.what());
    return DCPP_ERR_INVALID_ARG;
  }
}

void dcpp_gguf_close(dcpp_gguf* f) { delete f; }

dcpp_status dcpp_gguf_info(const dcpp_gguf* f, uint32_t* version, uint64_t* alignment, uint64_t* data_offset,
                           int64_t* n_tensors, int64_t* n_kv) {
  if (!f || !f->file) return DCPP_ERR_INVALID_ARG;
  if (version) *version = f->file->version();
  if (alignment) *alignment = f->file->alignment();
  if (data_offset) *data_offset = f->file->data_offset();
  if (n_tensors) *n_tensors = static_cast<int64_t>(f->file->tensors().size());
  if (n_kv) *n_kv = static_cast<int64_t>(f->file->metadata().size());
  return DCPP_OK;
}

dcpp_status dcpp_gguf_tensor(const dcpp_gguf* f, int64_t i, const char** name, int* type, int* n_dims, int64_t ne[4],
                             uint64_t* offset, uint64_t* nbytes, const void** data) {
  if (!f || !f->file || i < 0 || i >= static_cast<int64_t>(f->file->tensors().size())) return DCPP_ERR_INVALID_ARG;
  const auto& t = f->file->tensors()[static_cast<size_t>(i)];
  if (name) *name = t.name.c_str();
  if (type) *type = t.type;
  if (n_dims) {
    int n = 1;
    for (int d = 0; d < 4; ++d)
      if (t.ne[d] != 1) n = d + 1;
    *n_dims = n;
  }
  if (ne)
    for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
  if (offset) *offset = t.offset;
  if (nbytes) *nbytes = t.nbytes;
  if (data) *data = f->file->data(t);
  return DCPP_OK;
}

int64_t dcpp_gguf_find_tensor(const dcpp_gguf* f, const char* name) {
  if (!f || !f->file || !name) return -1;
  return f->file->find_tensor(name);
}

dcpp_status dcpp_gguf_kv(const dcpp_gguf* f, int64_t i, const char** key, uint32_t* type, uint32_t* elem_type,
                         uint64_t* count) {
  if (!f || !f->file || i < 0 || i >= static_cast<int64_t>(f->file->metadata().size())) return DCPP_ERR_INVALID_ARG;
  const auto& kv = f->file->metadata()[static_cast<size_t>(i)];
  if (key) *key = kv.first.c_str();
  if (type) *type = kv.second.type;
  if (elem_type) *elem_type = kv.second.type == dcpp::kArray ? kv.second.elem_type : 0;
  if (count) *count = kv.second.type == dcpp::kArray ? kv.second.count : 0;
  return DCPP_OK;
}

dcpp_status dcpp_gguf_get_int(const dcpp_gguf* f, const char* key, int64_t index, int64_t* out) {
  dcpp_status st;
  const dcpp::GGUFValue* v = kv_value(f, key, index, &st);
  if (!v) return st;
  const uint32_t t = v->type == dcpp::kArray ? v->elem_type : v->type;
  if (!out || t == dcpp::kString || dcpp::is_float(t)) return DCPP_ERR_INVALID_ARG;
  *out = index < 0 ? v->i : v->ai[static_cast<size_t>(index)];
  return DCPP_OK;
}

dcpp_status dcpp_gguf_get_float(const dcpp_gguf* f, const char* key, int64_t index, double* out) {
  dcpp_status st;
  const dcpp::GGUFValue* v = kv_value(f, key, index, &st);
  if (!v) return st;
  const uint32_t t = v->type == dcpp::kArray ? v->elem_type : v->type;
  if (!out || !dcpp::is_float(t)) return DCPP_ERR_INVALID_ARG;
  *out = index < 0 ? v->f : v->af[static_cast<size_t>(index)];
  return DCPP_OK;
}

dcpp_status dcpp_gguf_get_string(const dcpp_gguf* f, const char* key, int64_t index, char* buf, size_t cap) {
  dcpp_status st;
  const dcpp::GGUFValue* v = kv_value(f, key, index, &st);
  if (!v) return st;
  const uint32_t t = v->type == dcpp::kArray ? v->elem_type : v->type;
  if (!buf || t != dcpp::kString) return DCPP_ERR_INVALID_ARG;
  const std::string& s = index < 0 ? v->s : v->as[static_cast<size_t>(index)];
  if (cap < s.size() + 1) return DCPP_ERR_INVALID_ARG;
  memcpy(buf, s.data(), s.size());
  buf[s.size()] = 0;
  return DCPP_OK;
}

}  // extern "C"
