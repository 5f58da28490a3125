// GGUF checkpoint reader: the on-disk format the reference's models load
// (GGUFLoaderVisitor, src/ggml/GGUFLoaderVisitor.cpp:15-429, which parses
// metadata with ggml's gguf_init_from_file and streams each tensor's bytes
// from the file).  Here the file is memory-mapped once and every tensor is
// handed to a model's set_param straight from the mapping: the block bytes
// go to the device without an intermediate host copy.
//
// Format (GGUF v2 / v3, little-endian): magic "GGUF", u32 version, u64
// tensor count, u64 metadata count; metadata entries (string key, u32 value
// type, value); tensor infos (string name, u32 n_dims, u64 ne[n_dims], u32
// ggml type, u64 offset relative to the data section); the data section
// starts at the next multiple of general.alignment (default 32).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace dcpp {

// One metadata value.  Arrays keep their element type and their elements
// (numbers as int64 / double, strings as std::string).
struct GGUFValue {
  uint32_t type = 0;       // GGUF value type (0 u8 ... 12 f64)
  uint32_t elem_type = 0;  // arrays: element type
  int64_t i = 0;           // integer and bool values
  double f = 0.0;          // float values
  std::string s;           // string values
  std::vector<int64_t> ai;
  std::vector<double> af;
  std::vector<std::string> as;
  uint64_t count = 0;      // arrays: number of elements
};

struct GGUFTensorInfo {
  std::string name;
  int type = 0;                 // ggml type id
  std::vector<int64_t> ne;      // ggml order: ne[0] is the row length
  uint64_t offset = 0;          // absolute offset of the data in the file
  uint64_t nbytes = 0;          // bytes of the data (0 when the type's block size is unknown)
  // The shape the reference binds (GGUFLoaderVisitor.cpp:244-266): trailing
  // unit dimensions dropped, reversed to row-major (PyTorch) order.
  std::vector<int64_t> shape() const;
};

// Block size (elements) and block bytes of a ggml type; {0, 0} if unknown.
struct GGUFTypeSize {
  int64_t block = 0;
  int64_t bytes = 0;
};
GGUFTypeSize gguf_type_size(int type);

class GGUFFile {
 public:
  // path: a .gguf file, or a directory holding one (the first *.gguf in
  // name order is used; the reference takes the first its directory
  // iterator returns, find_first_gguf, GGUFLoaderVisitor.cpp:113-129).
  explicit GGUFFile(const std::string& path);
  ~GGUFFile();
  GGUFFile(const GGUFFile&) = delete;
  GGUFFile& operator=(const GGUFFile&) = delete;

  const std::string& path() const { return path_; }
  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  uint64_t data_offset() const { return data_offset_; }
  uint64_t file_size() const { return size_; }
  const std::vector<GGUFTensorInfo>& tensors() const { return tensors_; }
  const std::vector<std::pair<std::string, GGUFValue>>& metadata() const { return kv_; }
  const GGUFValue* find_kv(const std::string& key) const;
  int64_t find_tensor(const std::string& name) const;  // -1 if absent
  // Pointer to a tensor's bytes inside the mapping (valid while open).
  const uint8_t* data(const GGUFTensorInfo& t) const { return base_ + t.offset; }

 private:
  std::string path_;
  const uint8_t* base_ = nullptr;
  uint64_t size_ = 0;
  uint32_t version_ = 0;
  uint64_t alignment_ = 32;
  uint64_t data_offset_ = 0;
  std::vector<std::pair<std::string, GGUFValue>> kv_;
  std::vector<GGUFTensorInfo> tensors_;
  std::map<std::string, int64_t> index_;
};

// Binds every tensor of `file` through `set_param(name, type, shape, data,
// nbytes)`.  A tensor the model does not know (set_param throws
// DCPP_ERR_NOT_FOUND) is skipped and counted, as the reference leaves it to
// validate() (GGUFLoaderVisitor.cpp:175-189), which only reports.  Any other
// error is rethrown with the tensor's name.  Returns the number bound.
using GGUFSetParam =
    std::function<void(const std::string&, int, const std::vector<int64_t>&, const void*, size_t)>;
int64_t gguf_bind_all(const GGUFFile& file, const GGUFSetParam& set_param, int64_t* unused);

}  // namespace dcpp

struct dcpp_gguf {
  std::unique_ptr<dcpp::GGUFFile> file;
};
