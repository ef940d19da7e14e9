// gguf.h -- read-only GGUF (v1-v3) container: metadata and tensor table over mmap.
//
// Same format contract as the reference loader (src/gguf.cc:69-160): magic
// "GGUF", v1 counts are u32 and v2/v3 counts u64, tensor data aligned to
// general.alignment (default 32), dims[0] is the fastest-varying dimension so a
// 2-D weight is row-major [dims[1], dims[0]].  Arrays are kept as file
// offsets and decoded on demand (the tokenizer arrays hold 150k strings).
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace rpgb {

enum GgmlType : uint32_t {
  kGgmlF32 = 0,
  kGgmlF16 = 1,
  kGgmlQ8_0 = 8,
  kGgmlQ4_K = 12,
  kGgmlQ5_K = 13,
  kGgmlQ6_K = 14,
};

// The quantised matrix types the kernels run: Q4_K and Q6_K (the reference's
// GPU set, src/gpu_model.cu:26-38) plus Q5_K and Q8_0.
inline bool MatrixTypeSupported(uint32_t t) {
  return t == kGgmlQ4_K || t == kGgmlQ6_K || t == kGgmlQ5_K || t == kGgmlQ8_0;
}

// Bytes per 256-element super-block (or per element for F32/F16).
int64_t GgmlRowBytes(uint32_t type, int64_t n_elems);
const char* GgmlTypeName(uint32_t type);

struct GgufTensor {
  std::string name;
  std::vector<int64_t> dims;
  uint32_t type = 0;
  int64_t offset = 0;  // absolute file offset of the data
  int64_t n_elements = 0;
  int64_t n_bytes = 0;
  int64_t cols() const { return dims.empty() ? 0 : dims[0]; }
  int64_t rows() const { return dims.size() >= 2 ? dims[1] : 1; }
};

class GgufFile {
 public:
  GgufFile() = default;
  ~GgufFile();
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;

  void Open(const std::string& path);

  const std::string& path() const { return path_; }
  int64_t size() const { return size_; }
  const uint8_t* data() const { return base_; }

  bool Has(const std::string& key) const { return meta_.count(key) != 0; }
  int64_t GetInt(const std::string& key, int64_t def) const;
  double GetFloat(const std::string& key, double def) const;
  bool GetBool(const std::string& key, bool def) const;
  std::string GetStr(const std::string& key, const std::string& def = "") const;
  std::vector<std::string> GetStrArray(const std::string& key) const;
  std::vector<int64_t> GetIntArray(const std::string& key) const;
  int64_t ArrayLen(const std::string& key) const;

  const std::vector<GgufTensor>& tensors() const { return tensors_; }
  const GgufTensor* Find(const std::string& name) const;
  const uint8_t* TensorData(const GgufTensor& t) const { return base_ + t.offset; }

 private:
  struct Meta {
    uint32_t type = 0;
    int64_t i = 0;
    double f = 0;
    std::string s;
    uint32_t elem_type = 0;  // arrays
    uint64_t count = 0;
    int64_t pos = 0;  // arrays: file offset of the first element
  };
  std::string path_;
  int fd_ = -1;
  uint8_t* base_ = nullptr;
  int64_t size_ = 0;
  std::unordered_map<std::string, Meta> meta_;
  std::vector<GgufTensor> tensors_;
  std::unordered_map<std::string, size_t> index_;
};

}  // namespace rpgb
