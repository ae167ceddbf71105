#include "gguf.h"

#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace specb200 {

namespace {

// GGUF value type ids.
enum : int {
  T_U8 = 0, T_I8 = 1, T_U16 = 2, T_I16 = 3, T_U32 = 4, T_I32 = 5, T_F32 = 6, T_BOOL = 7,
  T_STR = 8, T_ARR = 9, T_U64 = 10, T_I64 = 11, T_F64 = 12,
};

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  bool need(size_t n) {
    if ((size_t)(end - p) < n) ok = false;
    return ok;
  }
  template <class T>
  T rd() {
    T v{};
    if (!need(sizeof(T))) return v;
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = rd<uint64_t>();
    if (!ok || !need(n)) return {};
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

int scalar_size(int t) {
  switch (t) {
    case T_U8: case T_I8: case T_BOOL: return 1;
    case T_U16: case T_I16: return 2;
    case T_U32: case T_I32: case T_F32: return 4;
    case T_U64: case T_I64: case T_F64: return 8;
  }
  return 0;
}

double read_num(Cursor& c, int t, GgufValue* v) {
  switch (t) {
    case T_U8: { uint8_t x = c.rd<uint8_t>(); if (v) v->u = x, v->i = x; return x; }
    case T_I8: { int8_t x = c.rd<int8_t>(); if (v) v->i = x, v->u = (uint64_t)x; return x; }
    case T_U16: { uint16_t x = c.rd<uint16_t>(); if (v) v->u = x, v->i = x; return x; }
    case T_I16: { int16_t x = c.rd<int16_t>(); if (v) v->i = x, v->u = (uint64_t)x; return x; }
    case T_U32: { uint32_t x = c.rd<uint32_t>(); if (v) v->u = x, v->i = x; return x; }
    case T_I32: { int32_t x = c.rd<int32_t>(); if (v) v->i = x, v->u = (uint64_t)x; return x; }
    case T_F32: { float x = c.rd<float>(); if (v) v->f = x; return x; }
    case T_BOOL: { uint8_t x = c.rd<uint8_t>(); if (v) v->u = x, v->i = x; return x; }
    case T_U64: { uint64_t x = c.rd<uint64_t>(); if (v) v->u = x, v->i = (int64_t)x; return (double)x; }
    case T_I64: { int64_t x = c.rd<int64_t>(); if (v) v->i = x, v->u = (uint64_t)x; return (double)x; }
    case T_F64: { double x = c.rd<double>(); if (v) v->f = x; return x; }
  }
  c.ok = false;
  return 0;
}

int ggml_block_elems(int t) {
  switch (t) {
    case 12: case 13: case 14: return 256;  // Q4_K Q5_K Q6_K
    case 8: return 32;                      // Q8_0
    case 0: case 1: case 30: return 1;      // F32 F16 BF16
  }
  return 0;
}
int ggml_block_bytes(int t) {
  switch (t) {
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
    case 8: return 34;
    case 0: return 4;
    case 1: case 30: return 2;
  }
  return 0;
}

}  // namespace

GgufFile::~GgufFile() {
  if (base_) munmap(const_cast<uint8_t*>(base_), size_);
  if (fd_ >= 0) close(fd_);
}

std::string GgufFile::open(const std::string& path) {
  fd_ = ::open(path.c_str(), O_RDONLY);
  if (fd_ < 0) return "cannot open " + path + ": " + strerror(errno);
  struct stat st;
  if (fstat(fd_, &st) != 0) return "cannot stat " + path;
  size_ = (size_t)st.st_size;
  if (size_ < 24) return "file too small to be GGUF: " + path;
  void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (m == MAP_FAILED) return "mmap failed: " + path;
  base_ = static_cast<const uint8_t*>(m);
  Cursor c{base_, base_ + size_};
  const uint32_t magic = c.rd<uint32_t>();
  if (magic != 0x46554747u) return "bad GGUF magic in " + path;
  version_ = c.rd<uint32_t>();
  if (version_ < 2 || version_ > 3) return "unsupported GGUF version " + std::to_string(version_);
  const uint64_t n_tensors = c.rd<uint64_t>();
  const uint64_t n_kv = c.rd<uint64_t>();
  for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
    const std::string key = c.str();
    GgufValue v;
    v.type = (int)c.rd<uint32_t>();
    if (v.type == T_STR) {
      v.s = c.str();
    } else if (v.type == T_ARR) {
      v.arr_type = (int)c.rd<uint32_t>();
      v.arr_len = c.rd<uint64_t>();
      for (uint64_t j = 0; j < v.arr_len && c.ok; ++j) {
        if (v.arr_type == T_STR) {
          c.str();
        } else if (scalar_size(v.arr_type)) {
          const double x = read_num(c, v.arr_type, nullptr);
          if (v.arr_num.size() < 4096) v.arr_num.push_back(x);
        } else {
          return "nested GGUF arrays are not supported (key " + key + ")";
        }
      }
    } else if (scalar_size(v.type)) {
      read_num(c, v.type, &v);
    } else {
      return "unknown GGUF value type for key " + key;
    }
    kv_[key] = std::move(v);
  }
  for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
    GgufTensor t;
    t.name = c.str();
    const uint32_t nd = c.rd<uint32_t>();
    if (nd > 4) return "tensor " + t.name + " has too many dims";
    for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(c.rd<uint64_t>());
    t.type = (int)c.rd<uint32_t>();
    t.offset = c.rd<uint64_t>();
    const int be = ggml_block_elems(t.type), bb = ggml_block_bytes(t.type);
    if (!be) return "tensor " + t.name + " has unsupported ggml type " + std::to_string(t.type);
    uint64_t n = 1;
    for (auto d : t.dims) n *= d;
    if (t.dims.empty() || t.dims[0] % be) return "tensor " + t.name + " row is not a whole number of blocks";
    t.nbytes = n / be * bb;
    tensors_[t.name] = std::move(t);
  }
  if (!c.ok) return "truncated GGUF header in " + path;
  uint32_t align = 32;
  uint32_t a;
  if (get_u32("general.alignment", a) && a) align = a;
  const uint64_t hdr = (uint64_t)(c.p - base_);
  data_off_ = (hdr + align - 1) / align * align;
  for (auto& kvp : tensors_) {
    const GgufTensor& t = kvp.second;
    if (data_off_ + t.offset + t.nbytes > size_) return "tensor " + t.name + " extends past end of file";
  }
  return {};
}

const GgufValue* GgufFile::get(const std::string& key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}

bool GgufFile::get_u32(const std::string& key, uint32_t& out) const {
  const GgufValue* v = get(key);
  if (!v || v->type == T_STR || v->type == T_ARR || v->type == T_F32 || v->type == T_F64) return false;
  out = (uint32_t)v->u;
  return true;
}

bool GgufFile::get_f32(const std::string& key, float& out) const {
  const GgufValue* v = get(key);
  if (!v) return false;
  if (v->type == T_F32 || v->type == T_F64) out = (float)v->f;
  else if (v->type == T_STR || v->type == T_ARR) return false;
  else out = (float)v->i;
  return true;
}

bool GgufFile::get_str(const std::string& key, std::string& out) const {
  const GgufValue* v = get(key);
  if (!v || v->type != T_STR) return false;
  out = v->s;
  return true;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace specb200
