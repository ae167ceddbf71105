// Minimal GGUF (v2/v3) reader: metadata, tensor directory, mmap'd data.
//
// Reads the same keys and tensor names as the reference's loaders
// (crates/speculate/src/model/quantized_llama_local.rs:229-281,
//  crates/speculate/src/model/quantized_qwen2_local.rs:220-275; vocab size
//  from `tokenizer.ggml.tokens`, quantized_llama.rs:75-80).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace specb200 {

struct GgufValue {
  int type = -1;          // GGUF value type id
  uint64_t u = 0;         // unsigned / bool
  int64_t i = 0;          // signed
  double f = 0.0;         // float
  std::string s;          // string
  int arr_type = -1;      // array element type
  uint64_t arr_len = 0;   // array length
  std::vector<double> arr_num;  // numeric array elements (strings are skipped)
};

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> dims;  // dims[0] = columns (K), dims[1] = rows (N)
  int type = 0;
  uint64_t offset = 0;          // relative to the data section
  uint64_t nbytes = 0;
};

class GgufFile {
 public:
  ~GgufFile();
  // Returns an empty string on success, else an error message.
  std::string open(const std::string& path);
  const GgufValue* get(const std::string& key) const;
  bool get_u32(const std::string& key, uint32_t& out) const;
  bool get_f32(const std::string& key, float& out) const;
  bool get_str(const std::string& key, std::string& out) const;
  const GgufTensor* tensor(const std::string& name) const;
  const uint8_t* data(const GgufTensor& t) const { return base_ + data_off_ + t.offset; }
  uint32_t version() const { return version_; }

 private:
  int fd_ = -1;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  uint64_t data_off_ = 0;
  uint32_t version_ = 0;
  std::map<std::string, GgufValue> kv_;
  std::map<std::string, GgufTensor> tensors_;
};

}  // namespace specb200
