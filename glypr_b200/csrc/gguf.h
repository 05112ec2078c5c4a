// GGUF v2/v3 reader (memory-mapped, read-only).  Parses the metadata and tensor table the
// way candle's gguf_file::Content does for glypr (crates/glypr-core/src/lib.rs:176-209,
// model.rs:229-488): little-endian header, key/value metadata, tensor infos (ne[0] is the
// innermost dimension), data section aligned to general.alignment (default 32).
#pragma once
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <string_view>
#include <vector>

namespace glp {

enum GgmlType : uint32_t { kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ8_0 = 8, kGgmlBF16 = 30 };

struct GgufValue {
  int type = -1;       // gguf value type
  double num = 0;      // numeric scalars (bool as 0/1)
  std::string str;
  int arr_type = -1;
  uint64_t arr_len = 0;
  std::vector<double> arr;  // numeric / bool array elements
  std::vector<std::string_view> strs;  // string array elements (views into the mapped file)
};

struct GgufTensor {
  std::string name;
  std::vector<int64_t> ne;
  uint32_t type = 0;
  uint64_t offset = 0;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto e : ne) n *= e;
    return n;
  }
};

class GgufFile {
 public:
  GgufFile() = default;
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  // Returns false and sets *err on any I/O or format error (truncated or corrupt files
  // are rejected before any tensor is touched).
  bool open(const char* path, std::string* err);

  const GgufValue* find(const std::string& key) const {
    auto it = kv_.find(key);
    return it == kv_.end() ? nullptr : &it->second;
  }
  const GgufTensor* tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
  }
  // scalar lookups with the reference's type rules (config.rs:253-280): false = no value
  bool get_u32(const std::string& key, uint32_t* out) const;
  bool get_f64(const std::string& key, double* out) const;
  // element i of an integer array (false when the key is absent, not an array, i is past its
  // end or its elements are not integers)
  bool get_array_u32(const std::string& key, size_t i, uint32_t* out) const;

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, GgufValue> kv_;
  std::map<std::string, GgufTensor> tensors_;
};

size_t ggml_nbytes(uint32_t type, int64_t numel);

}  // namespace glp
