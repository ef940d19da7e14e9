#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "common.h"

namespace rpgb {

namespace {

enum MetaType : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6,
  kBool = 7, kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

int ScalarSize(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return -1;
  }
}

class Cursor {
 public:
  Cursor(const uint8_t* p, int64_t n) : p_(p), n_(n) {}
  void Need(int64_t k) const {
    RPGB_CHECK(pos_ + k <= n_, "GGUF truncated at byte %lld (need %lld more)",
               static_cast<long long>(pos_), static_cast<long long>(k));
  }
  template <typename T>
  T Get() {
    Need(sizeof(T));
    T v;
    std::memcpy(&v, p_ + pos_, sizeof(T));
    pos_ += sizeof(T);
    return v;
  }
  std::string Str() {
    const uint64_t n = Get<uint64_t>();
    RPGB_CHECK(n < (1ull << 31), "GGUF string length %llu is implausible",
               static_cast<unsigned long long>(n));
    Need(static_cast<int64_t>(n));
    std::string s(reinterpret_cast<const char*>(p_ + pos_), static_cast<size_t>(n));
    pos_ += static_cast<int64_t>(n);
    return s;
  }
  void Skip(int64_t k) {
    Need(k);
    pos_ += k;
  }
  int64_t pos() const { return pos_; }
  void Seek(int64_t p) { pos_ = p; }

 private:
  const uint8_t* p_;
  int64_t n_;
  int64_t pos_ = 0;
};

int64_t ReadScalarInt(Cursor& c, uint32_t t) {
  switch (t) {
    case kU8: return c.Get<uint8_t>();
    case kI8: return c.Get<int8_t>();
    case kU16: return c.Get<uint16_t>();
    case kI16: return c.Get<int16_t>();
    case kU32: return c.Get<uint32_t>();
    case kI32: return c.Get<int32_t>();
    case kU64: return static_cast<int64_t>(c.Get<uint64_t>());
    case kI64: return c.Get<int64_t>();
    case kBool: return c.Get<uint8_t>() != 0;
    default: Throw("GGUF metadata type %u is not an integer", t);
  }
}

}  // namespace

int64_t GgmlRowBytes(uint32_t type, int64_t n) {
  switch (type) {
    case kGgmlF32: return n * 4;
    case kGgmlF16: return n * 2;
    case kGgmlQ4_K:
      RPGB_CHECK(n % 256 == 0, "Q4_K row of %lld elements is not a multiple of 256", static_cast<long long>(n));
      return n / 256 * 144;
    case kGgmlQ6_K:
      RPGB_CHECK(n % 256 == 0, "Q6_K row of %lld elements is not a multiple of 256", static_cast<long long>(n));
      return n / 256 * 210;
    case kGgmlQ5_K:
      RPGB_CHECK(n % 256 == 0, "Q5_K row of %lld elements is not a multiple of 256", static_cast<long long>(n));
      return n / 256 * 176;
    case kGgmlQ8_0:
      RPGB_CHECK(n % 32 == 0, "Q8_0 row of %lld elements is not a multiple of 32", static_cast<long long>(n));
      return n / 32 * 34;
    default:
      Throw("ggml type %u (%s) is not supported by this engine (F32, F16, Q4_K, Q5_K, Q6_K and Q8_0 are)", type,
            GgmlTypeName(type));
  }
}

const char* GgmlTypeName(uint32_t type) {
  switch (type) {
    case 0: return "F32";
    case 1: return "F16";
    case 2: return "Q4_0";
    case 3: return "Q4_1";
    case 6: return "Q5_0";
    case 7: return "Q5_1";
    case 8: return "Q8_0";
    case 10: return "Q2_K";
    case 11: return "Q3_K";
    case 12: return "Q4_K";
    case 13: return "Q5_K";
    case 14: return "Q6_K";
    case 15: return "Q8_K";
    case 30: return "BF16";
    default: return "unknown";
  }
}

GgufFile::~GgufFile() {
  if (base_ != nullptr) munmap(base_, static_cast<size_t>(size_));
  if (fd_ >= 0) close(fd_);
}

void GgufFile::Open(const std::string& path) {
  path_ = path;
  fd_ = open(path.c_str(), O_RDONLY);
  RPGB_CHECK(fd_ >= 0, "cannot open %s", path.c_str());
  struct stat st;
  RPGB_CHECK(fstat(fd_, &st) == 0, "cannot stat %s", path.c_str());
  size_ = st.st_size;
  RPGB_CHECK(size_ >= 24, "%s is too small to be a GGUF file", path.c_str());
  void* p = mmap(nullptr, static_cast<size_t>(size_), PROT_READ, MAP_PRIVATE, fd_, 0);
  RPGB_CHECK(p != MAP_FAILED, "cannot mmap %s", path.c_str());
  base_ = static_cast<uint8_t*>(p);

  Cursor c(base_, size_);
  const uint32_t magic = c.Get<uint32_t>();
  RPGB_CHECK(magic == 0x46554747u, "%s: bad magic 0x%08X (not GGUF)", path.c_str(), magic);
  const uint32_t version = c.Get<uint32_t>();
  RPGB_CHECK(version >= 1 && version <= 3, "GGUF version %u is not supported", version);
  uint64_t n_tensors, n_kv;
  if (version == 1) {
    n_tensors = c.Get<uint32_t>();
    n_kv = c.Get<uint32_t>();
  } else {
    n_tensors = c.Get<uint64_t>();
    n_kv = c.Get<uint64_t>();
  }
  RPGB_CHECK(n_tensors < (1u << 20) && n_kv < (1u << 20), "GGUF header counts are implausible");

  for (uint64_t i = 0; i < n_kv; ++i) {
    const std::string key = c.Str();
    Meta m;
    m.type = c.Get<uint32_t>();
    if (m.type == kString) {
      m.s = c.Str();
    } else if (m.type == kF32) {
      m.f = c.Get<float>();
    } else if (m.type == kF64) {
      m.f = c.Get<double>();
    } else if (m.type == kArray) {
      m.elem_type = c.Get<uint32_t>();
      m.count = c.Get<uint64_t>();
      RPGB_CHECK(m.count < (1ull << 32), "GGUF array %s is implausibly long", key.c_str());
      m.pos = c.pos();
      if (m.elem_type == kString) {
        for (uint64_t k = 0; k < m.count; ++k) {
          const uint64_t n = c.Get<uint64_t>();
          c.Skip(static_cast<int64_t>(n));
        }
      } else {
        const int sz = ScalarSize(m.elem_type);
        RPGB_CHECK(sz > 0, "GGUF array %s has unsupported element type %u", key.c_str(), m.elem_type);
        c.Skip(static_cast<int64_t>(m.count) * sz);
      }
    } else {
      m.i = ReadScalarInt(c, m.type);
      m.f = static_cast<double>(m.i);
    }
    meta_[key] = std::move(m);
  }

  const int64_t alignment = GetInt("general.alignment", 32);
  RPGB_CHECK(alignment > 0 && alignment % 8 == 0, "GGUF alignment %lld is invalid", static_cast<long long>(alignment));

  tensors_.reserve(static_cast<size_t>(n_tensors));
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor t;
    t.name = c.Str();
    const uint32_t nd = c.Get<uint32_t>();
    RPGB_CHECK(nd >= 1 && nd <= 4, "tensor %s has %u dims", t.name.c_str(), nd);
    t.n_elements = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t v = c.Get<uint64_t>();
      RPGB_CHECK(v > 0 && v < (1ull << 40), "tensor %s dim %u is invalid", t.name.c_str(), d);
      t.dims.push_back(static_cast<int64_t>(v));
      t.n_elements *= static_cast<int64_t>(v);
    }
    t.type = c.Get<uint32_t>();
    t.offset = static_cast<int64_t>(c.Get<uint64_t>());
    tensors_.push_back(std::move(t));
  }
  const int64_t data_start = (c.pos() + alignment - 1) / alignment * alignment;
  for (size_t i = 0; i < tensors_.size(); ++i) {
    GgufTensor& t = tensors_[i];
    t.offset += data_start;
    if (t.type == kGgmlF32 || t.type == kGgmlF16 || MatrixTypeSupported(t.type)) {
      t.n_bytes = GgmlRowBytes(t.type, t.cols()) * (t.n_elements / t.cols());
      RPGB_CHECK(t.offset + t.n_bytes <= size_, "tensor %s runs past the end of the file", t.name.c_str());
    } else {
      t.n_bytes = -1;  // unsupported types are rejected only if the model uses them
    }
    RPGB_CHECK(index_.emplace(t.name, i).second, "duplicate tensor name %s", t.name.c_str());
  }
}

int64_t GgufFile::GetInt(const std::string& key, int64_t def) const {
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type == kString || it->second.type == kArray) return def;
  if (it->second.type == kF32 || it->second.type == kF64) return static_cast<int64_t>(it->second.f);
  return it->second.i;
}

double GgufFile::GetFloat(const std::string& key, double def) const {
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type == kString || it->second.type == kArray) return def;
  return it->second.f;
}

bool GgufFile::GetBool(const std::string& key, bool def) const {
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type == kString || it->second.type == kArray) return def;
  return it->second.i != 0;
}

std::string GgufFile::GetStr(const std::string& key, const std::string& def) const {
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type != kString) return def;
  return it->second.s;
}

int64_t GgufFile::ArrayLen(const std::string& key) const {
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type != kArray) return -1;
  return static_cast<int64_t>(it->second.count);
}

std::vector<std::string> GgufFile::GetStrArray(const std::string& key) const {
  std::vector<std::string> out;
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type != kArray || it->second.elem_type != kString) return out;
  Cursor c(base_, size_);
  c.Seek(it->second.pos);
  out.reserve(static_cast<size_t>(it->second.count));
  for (uint64_t i = 0; i < it->second.count; ++i) out.push_back(c.Str());
  return out;
}

std::vector<int64_t> GgufFile::GetIntArray(const std::string& key) const {
  std::vector<int64_t> out;
  const auto it = meta_.find(key);
  if (it == meta_.end() || it->second.type != kArray || it->second.elem_type == kString) return out;
  Cursor c(base_, size_);
  c.Seek(it->second.pos);
  out.reserve(static_cast<size_t>(it->second.count));
  for (uint64_t i = 0; i < it->second.count; ++i) out.push_back(ReadScalarInt(c, it->second.elem_type));
  return out;
}

const GgufTensor* GgufFile::Find(const std::string& name) const {
  const auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

}  // namespace rpgb
