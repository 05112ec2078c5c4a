#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace glp {

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <class T>
  T get() {
    T v{};
    if (!ok || static_cast<size_t>(end - p) < sizeof(T)) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

bool read_scalar(Cursor& c, int type, double* num, std::string* s) {
  switch (type) {
    case 0: *num = c.get<uint8_t>(); break;
    case 1: *num = c.get<int8_t>(); break;
    case 2: *num = c.get<uint16_t>(); break;
    case 3: *num = c.get<int16_t>(); break;
    case 4: *num = c.get<uint32_t>(); break;
    case 5: *num = c.get<int32_t>(); break;
    case 6: *num = c.get<float>(); break;
    case 7: *num = c.get<uint8_t>() ? 1.0 : 0.0; break;
    case 8: *s = c.str(); break;
    case 10: *num = static_cast<double>(c.get<uint64_t>()); break;
    case 11: *num = static_cast<double>(c.get<int64_t>()); break;
    case 12: *num = c.get<double>(); break;
    default: return false;
  }
  return c.ok;
}

}  // namespace

size_t ggml_nbytes(uint32_t type, int64_t numel) {
  switch (type) {
    case kGgmlF32: return 4 * static_cast<size_t>(numel);
    case kGgmlF16:
    case kGgmlBF16: return 2 * static_cast<size_t>(numel);
    case kGgmlQ8_0: return numel % 32 ? 0 : static_cast<size_t>(numel / 32) * 34;
    default: return 0;
  }
}

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

bool GgufFile::open(const char* path, std::string* err) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    *err = std::string("cannot open GGUF file: ") + path;
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    *err = std::string("GGUF file too small: ") + path;
    return false;
  }
  size_ = static_cast<size_t>(st.st_size);
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    *err = "mmap failed";
    return false;
  }
  Cursor c{static_cast<const uint8_t*>(map_), static_cast<const uint8_t*>(map_) + size_};
  if (c.get<uint32_t>() != 0x46554747u) {
    *err = "not a GGUF file (bad magic)";
    return false;
  }
  const uint32_t version = c.get<uint32_t>();
  if (version < 2 || version > 3) {
    *err = "unsupported GGUF version " + std::to_string(version);
    return false;
  }
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  if (!c.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) {
    *err = "corrupt GGUF header";
    return false;
  }
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    GgufValue v;
    v.type = static_cast<int>(c.get<uint32_t>());
    if (!c.ok) break;
    if (v.type == 9) {
      v.arr_type = static_cast<int>(c.get<uint32_t>());
      v.arr_len = c.get<uint64_t>();
      if (!c.ok || v.arr_len > size_) {
        c.ok = false;
        break;
      }
      for (uint64_t j = 0; j < v.arr_len; ++j) {
        if (v.arr_type == 8) {  // strings stay in the mapping
          const uint64_t n = c.get<uint64_t>();
          if (!c.ok || static_cast<uint64_t>(c.end - c.p) < n) {
            c.ok = false;
            break;
          }
          v.strs.emplace_back(reinterpret_cast<const char*>(c.p), n);
          c.p += n;
          continue;
        }
        double x = 0;
        std::string s;
        if (!read_scalar(c, v.arr_type, &x, &s)) {
          c.ok = false;
          break;
        }
        v.arr.push_back(x);
      }
    } else if (!read_scalar(c, v.type, &v.num, &v.str)) {
      c.ok = false;
    }
    if (!c.ok) break;
    kv_[key] = std::move(v);
  }
  if (!c.ok) {
    *err = "truncated or corrupt GGUF metadata";
    return false;
  }
  uint64_t align = 32;
  if (auto* a = find("general.alignment")) align = static_cast<uint64_t>(a->num);
  if (align == 0 || (align & (align - 1))) {
    *err = "bad general.alignment";
    return false;
  }
  std::vector<std::string> order;
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok || nd == 0 || nd > 4) {
      c.ok = false;
      break;
    }
    for (uint32_t d = 0; d < nd; ++d) t.ne.push_back(static_cast<int64_t>(c.get<uint64_t>()));
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) break;
    order.push_back(t.name);
    tensors_[t.name] = std::move(t);
  }
  if (!c.ok) {
    *err = "truncated or corrupt GGUF tensor table";
    return false;
  }
  const size_t header = static_cast<size_t>(c.p - static_cast<const uint8_t*>(map_));
  const size_t data0 = (header + align - 1) / align * align;
  for (const auto& name : order) {
    GgufTensor& t = tensors_[name];
    for (auto e : t.ne)
      if (e <= 0) {
        *err = "bad tensor shape: " + name;
        return false;
      }
    t.nbytes = ggml_nbytes(t.type, t.numel());
    if (t.nbytes == 0) {
      *err = "unsupported tensor type " + std::to_string(t.type) + " for " + name;
      return false;
    }
    if (t.offset > size_ || data0 + t.offset + t.nbytes > size_) {
      *err = "tensor data out of file bounds: " + name;
      return false;
    }
    t.data = static_cast<const uint8_t*>(map_) + data0 + t.offset;
  }
  return true;
}

// Integer GGUF value types (u8, i8, u16, i16, u32, i32, u64, i64): the ones the reference's
// get_u32 converts (config.rs:253-265, `v as u32`, wrapping negatives); any other type yields
// no value, so the caller's default applies.
static bool gguf_int_type(int t) { return (t >= 0 && t <= 5) || t == 10 || t == 11; }

static uint32_t gguf_as_u32(double v) { return static_cast<uint32_t>(static_cast<int64_t>(v)); }

bool GgufFile::get_u32(const std::string& key, uint32_t* out) const {
  const GgufValue* v = find(key);
  if (!v || !gguf_int_type(v->type)) return false;
  *out = gguf_as_u32(v->num);
  return true;
}

bool GgufFile::get_array_u32(const std::string& key, size_t i, uint32_t* out) const {
  const GgufValue* v = find(key);
  if (!v || v->type != 9 || i >= v->arr.size() || !gguf_int_type(v->arr_type)) return false;
  *out = gguf_as_u32(v->arr[i]);
  return true;
}

// f32 and f64 only (config.rs:274-280)
bool GgufFile::get_f64(const std::string& key, double* out) const {
  const GgufValue* v = find(key);
  if (!v || (v->type != 6 && v->type != 12)) return false;
  *out = v->num;
  return true;
}

}  // namespace glp
