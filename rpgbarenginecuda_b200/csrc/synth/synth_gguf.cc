// synth_gguf.cc -- seeded synthetic Qwen3 GGUF models in the Q4_K_M mix.
//
// There is no public checkpoint on this machine and the reference repository
// ships no quantiser (its src/quant.cc only dequantises), so the benchmark
// models are generated here: weights are N(0, 0.02) fp32, norms 1 + N(0, 0.05),
// quantised per 256-element super-block by the encoders below, and written as a
// GGUF v3 file that the reference's loader (src/gguf.cc:69-160,
// src/model_meta.cc:11-77, src/gpu_model.cu:148-246) accepts unchanged.
//
// The encoders invert the bit layouts the reference decodes:
//   Q4_K  src/quant.cc:159-167 (6-bit scale/min packing), src/quant.cc:252-277
//   Q6_K  src/quant.cc:321-354
// Their only contract is "DequantizeRow(encode(x)) is close to x"; tests check
// that round trip against the reference's own dequantiser.
//
// Random numbers are counter based (SplitMix64 of (seed, tensor, index)), so a
// model is bit-identical for a given seed regardless of thread count.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kTypeF32 = 0;
constexpr uint32_t kTypeQ8_0 = 8;
constexpr uint32_t kTypeQ4K = 12;
constexpr uint32_t kTypeQ5K = 13;
constexpr uint32_t kTypeQ6K = 14;
constexpr int kQK = 256;

// ---------------------------------------------------------------- randomness

inline uint64_t Mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint64_t HashName(const std::string& s) {
  uint64_t h = 1469598103934665603ull;
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

// Standard normal pair for counter `i` of stream `key` (Box-Muller in double).
inline void NormalPair(uint64_t key, uint64_t i, double* a, double* b) {
  const uint64_t r1 = Mix64(key + 2 * i);
  const uint64_t r2 = Mix64(key + 2 * i + 1);
  // (0, 1] so the log is finite.
  const double u1 = (static_cast<double>(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);
  const double u2 = static_cast<double>(r2 >> 11) * (1.0 / 9007199254740992.0);
  const double rad = std::sqrt(-2.0 * std::log(u1));
  const double th = 6.283185307179586476925 * u2;
  *a = rad * std::cos(th);
  *b = rad * std::sin(th);
}

// Fills out[0..n) with mean + std * N(0,1), elements [off, off+n) of the stream.
void FillNormal(uint64_t key, int64_t off, int64_t n, float mean, float stdv, float* out) {
  int64_t i = 0;
  while (i < n) {
    const int64_t e = off + i;
    double a, b;
    NormalPair(key, static_cast<uint64_t>(e >> 1), &a, &b);
    const double v = (e & 1) ? b : a;
    out[i] = static_cast<float>(mean + stdv * v);
    ++i;
  }
}

// ---------------------------------------------------------------- f16

// fp32 -> fp16 with round-to-nearest-even (same rounding as __float2half_rn).
uint16_t F32ToF16Rne(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // rounds to inf
  if (ax < 0x38800000u) {                                               // subnormal half
    if (ax < 0x33000000u) return static_cast<uint16_t>(sign);           // < 2^-25 -> 0
    const uint32_t e = ax >> 23;
    const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e;  // value = m * 2^(e-150); half ulp = 2^-24
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t h = ((ax >> 13) - (112u << 10));
  const uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(sign | h);
}

float F16ToF32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu;
  uint32_t out;
  if (e == 0) {
    if (m == 0) {
      out = sign;
    } else {
      int ee = 113;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        --ee;
      }
      out = sign | (static_cast<uint32_t>(ee) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    out = sign | 0x7F800000u | (m << 13);
  } else {
    out = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

inline int Clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// ---------------------------------------------------------------- Q4_K / Q5_K encoder
//
// Block (144 B): d f16 | dmin f16 | scales[12] | qs[128].
// Element e of sub-block j (32 wide) decodes as (d*sc_j)*q - (dmin*m_j), q in
// [0,15], sc_j and m_j 6-bit.  Encoding: per sub-block take [lo, hi] with lo <= 0,
// the 4-bit step (hi-lo)/15 and offset -lo; the super-block stores d and dmin as
// the largest step / offset over 63, then everything is requantised against the
// f16-rounded d and dmin so the stored q match the decoder exactly.
// Q5_K (176 B: d | dmin | scales[12] | qh[32] | qs[128]) is the same with
// 5-bit q in [0, 31]: low nibbles packed as Q4_K's, the fifth bit of column
// 64 g + l in bit 2 g of qh[l] and of column 64 g + 32 + l in bit 2 g + 1.
void EncodeQ45KBlock(const float* x, uint8_t* out, bool five) {
  const int levels = five ? 31 : 15;
  float step[8], off[8];
  for (int j = 0; j < 8; ++j) {
    float lo = 0.0f, hi = 0.0f;
    for (int l = 0; l < 32; ++l) {
      const float v = x[32 * j + l];
      lo = v < lo ? v : lo;
      hi = v > hi ? v : hi;
    }
    step[j] = (hi - lo) / static_cast<float>(levels);
    off[j] = -lo;
  }
  float smax = 0.0f, omax = 0.0f;
  for (int j = 0; j < 8; ++j) {
    smax = step[j] > smax ? step[j] : smax;
    omax = off[j] > omax ? off[j] : omax;
  }
  const uint16_t dh = F32ToF16Rne(smax / 63.0f);
  const uint16_t mh = F32ToF16Rne(omax / 63.0f);
  const float d = F16ToF32(dh);
  const float dmin = F16ToF32(mh);

  int sc[8], mn[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d > 0.0f ? Clampi(static_cast<int>(std::lround(step[j] / d)), 0, 63) : 0;
    mn[j] = dmin > 0.0f ? Clampi(static_cast<int>(std::lround(off[j] / dmin)), 0, 63) : 0;
    // A step that rounds to zero would make the whole sub-block decode to -offset.
    if (sc[j] == 0 && step[j] > 0.0f && d > 0.0f) sc[j] = 1;
  }

  std::memcpy(out + 0, &dh, 2);
  std::memcpy(out + 2, &mh, 2);
  uint8_t* s = out + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = static_cast<uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }

  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    const float ds = d * static_cast<float>(sc[j]);
    const float dm = dmin * static_cast<float>(mn[j]);
    for (int l = 0; l < 32; ++l) {
      const float v = x[32 * j + l];
      const int qi = ds > 0.0f ? static_cast<int>(std::lround((v + dm) / ds)) : 0;
      q[32 * j + l] = static_cast<uint8_t>(Clampi(qi, 0, levels));
    }
  }
  uint8_t* qs = out + (five ? 48 : 16);
  for (int g = 0; g < 4; ++g) {
    for (int l = 0; l < 32; ++l) {
      qs[32 * g + l] = static_cast<uint8_t>((q[64 * g + l] & 15) | ((q[64 * g + 32 + l] & 15) << 4));
    }
  }
  if (five) {
    uint8_t* qh = out + 16;
    for (int l = 0; l < 32; ++l) {
      uint8_t h = 0;
      for (int g = 0; g < 4; ++g) {
        h |= static_cast<uint8_t>(((q[64 * g + l] >> 4) & 1) << (2 * g));
        h |= static_cast<uint8_t>(((q[64 * g + 32 + l] >> 4) & 1) << (2 * g + 1));
      }
      qh[l] = h;
    }
  }
}
void EncodeQ4KBlock(const float* x, uint8_t* out) { EncodeQ45KBlock(x, out, false); }
void EncodeQ5KBlock(const float* x, uint8_t* out) { EncodeQ45KBlock(x, out, true); }

// ---------------------------------------------------------------- Q8_0 encoder
//
// Block of 32 (34 B): d f16 | qs[32] int8, decoding as q * d; d = max|x| / 127
// rounded to f16, q requantised against the rounded d.
void EncodeQ80Block(const float* x, uint8_t* out) {
  float amax = 0.0f;
  for (int l = 0; l < 32; ++l) amax = std::fabs(x[l]) > amax ? std::fabs(x[l]) : amax;
  const uint16_t dh = F32ToF16Rne(amax / 127.0f);
  const float d = F16ToF32(dh);
  std::memcpy(out, &dh, 2);
  for (int l = 0; l < 32; ++l) {
    const int qi = d > 0.0f ? static_cast<int>(std::lround(x[l] / d)) : 0;
    out[2 + l] = static_cast<uint8_t>(static_cast<int8_t>(Clampi(qi, -127, 127)));
  }
}

void EncodeQ6KBlock(const float* x, uint8_t* out);

// Encodes n elements (a multiple of 256) of type `type` into out.
void EncodeRow(uint32_t type, const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / kQK; ++b) {
    if (type == kTypeQ4K) {
      EncodeQ4KBlock(x + b * kQK, out + b * 144);
    } else if (type == kTypeQ5K) {
      EncodeQ5KBlock(x + b * kQK, out + b * 176);
    } else if (type == kTypeQ6K) {
      EncodeQ6KBlock(x + b * kQK, out + b * 210);
    } else {
      for (int k = 0; k < 8; ++k) EncodeQ80Block(x + b * kQK + 32 * k, out + (b * 8 + k) * 34);
    }
  }
}

// ---------------------------------------------------------------- Q6_K encoder
//
// Block (210 B): ql[128] | qh[64] | sc[16] int8 | d f16.  Element e of 16-wide
// sub-block s decodes as (d*sc_s)*(q-32), q a 6-bit unsigned value.
void EncodeQ6KBlock(const float* x, uint8_t* out) {
  float amax[16];
  float gmax = 0.0f;
  for (int s = 0; s < 16; ++s) {
    float a = 0.0f;
    for (int l = 0; l < 16; ++l) {
      const float v = std::fabs(x[16 * s + l]);
      a = v > a ? v : a;
    }
    amax[s] = a / 31.0f;  // per-sub-block step
    gmax = amax[s] > gmax ? amax[s] : gmax;
  }
  const uint16_t dh = F32ToF16Rne(gmax / 127.0f);
  const float d = F16ToF32(dh);
  int8_t sc[16];
  for (int s = 0; s < 16; ++s) {
    int v = d > 0.0f ? static_cast<int>(std::lround(amax[s] / d)) : 0;
    if (v == 0 && amax[s] > 0.0f && d > 0.0f) v = 1;
    sc[s] = static_cast<int8_t>(Clampi(v, -128, 127));
  }
  uint8_t u[256];
  for (int s = 0; s < 16; ++s) {
    const float step = d * static_cast<float>(sc[s]);
    for (int l = 0; l < 16; ++l) {
      const float v = x[16 * s + l];
      const int qi = step > 0.0f ? static_cast<int>(std::lround(v / step)) : 0;
      u[16 * s + l] = static_cast<uint8_t>(Clampi(qi, -32, 31) + 32);
    }
  }
  uint8_t* ql = out;
  uint8_t* qh = out + 128;
  for (int hh = 0; hh < 2; ++hh) {
    const uint8_t* uu = u + 128 * hh;
    for (int l = 0; l < 32; ++l) {
      const uint8_t u1 = uu[l], u2 = uu[32 + l], u3 = uu[64 + l], u4 = uu[96 + l];
      ql[64 * hh + l] = static_cast<uint8_t>((u1 & 15) | ((u3 & 15) << 4));
      ql[64 * hh + 32 + l] = static_cast<uint8_t>((u2 & 15) | ((u4 & 15) << 4));
      qh[32 * hh + l] = static_cast<uint8_t>((u1 >> 4) | ((u2 >> 4) << 2) | ((u3 >> 4) << 4) |
                                             ((u4 >> 4) << 6));
    }
  }
  std::memcpy(out + 192, sc, 16);
  std::memcpy(out + 208, &dh, 2);
}

// ---------------------------------------------------------------- GGUF writer

struct Buf {
  std::vector<uint8_t> b;
  void Raw(const void* p, size_t n) {
    const uint8_t* q = static_cast<const uint8_t*>(p);
    b.insert(b.end(), q, q + n);
  }
  void U32(uint32_t v) { Raw(&v, 4); }
  void I32(int32_t v) { Raw(&v, 4); }
  void U64(uint64_t v) { Raw(&v, 8); }
  void F32(float v) { Raw(&v, 4); }
  void Str(const std::string& s) {
    U64(s.size());
    Raw(s.data(), s.size());
  }
};

enum : uint32_t { kMU32 = 4, kMI32 = 5, kMF32 = 6, kMBool = 7, kMStr = 8, kMArr = 9 };

struct TensorPlan {
  std::string name;
  uint32_t type;
  int64_t rows;  // 1 for vectors
  int64_t cols;
  int kind;  // 0 = weight N(0, 0.02), 1 = norm 1 + N(0, 0.05)
  uint64_t offset = 0;
  uint64_t nbytes = 0;
};

uint64_t RowBytes(uint32_t type, int64_t cols) {
  if (type == kTypeF32) return static_cast<uint64_t>(cols) * 4;
  const uint64_t nb = static_cast<uint64_t>(cols / kQK);
  switch (type) {
    case kTypeQ4K: return nb * 144u;
    case kTypeQ5K: return nb * 176u;
    case kTypeQ6K: return nb * 210u;
    default: return nb * 8u * 34u;  // Q8_0
  }
}

// GPT-2 byte-level alphabet: byte -> code point.
uint32_t ByteToCp(int b) {
  static uint32_t table[256];
  static bool init = false;
  if (!init) {
    int n = 0;
    for (int i = 0; i < 256; ++i) {
      const bool direct = (i >= 33 && i <= 126) || (i >= 161 && i <= 172) || (i >= 174 && i <= 255);
      table[i] = direct ? static_cast<uint32_t>(i) : static_cast<uint32_t>(256 + n++);
    }
    init = true;
  }
  return table[b];
}

std::string Utf8(uint32_t cp) {
  std::string s;
  if (cp < 0x80) {
    s.push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    s.push_back(static_cast<char>(0xC0 | (cp >> 6)));
    s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    s.push_back(static_cast<char>(0xE0 | (cp >> 12)));
    s.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
  return s;
}

// A small byte-level BPE vocabulary: 256 byte tokens, a few hundred merges over
// lowercase letters (with and without the leading-space marker), fillers, and
// the Qwen chat specials at the top of the id range.
void BuildTokenizer(int32_t vocab, std::vector<std::string>* toks, std::vector<int32_t>* types,
                    std::vector<std::string>* merges, int32_t* eos, int32_t* pad) {
  toks->clear();
  types->clear();
  merges->clear();
  for (int b = 0; b < 256; ++b) {
    toks->push_back(Utf8(ByteToCp(b)));
    types->push_back(6);  // BYTE
  }
  const std::string sp = Utf8(ByteToCp(' '));
  const char* common = "etaoinshrdlu";
  // 1) space + letter
  for (char c = 'a'; c <= 'z'; ++c) {
    merges->push_back(sp + " " + std::string(1, c));
    toks->push_back(sp + std::string(1, c));
    types->push_back(1);
  }
  // 2) letter + letter over the common letters
  for (const char* a = common; *a; ++a) {
    for (const char* b = common; *b; ++b) {
      merges->push_back(std::string(1, *a) + " " + std::string(1, *b));
      toks->push_back(std::string(1, *a) + std::string(1, *b));
      types->push_back(1);
    }
  }
  // 3) (space + letter) + common letter
  for (char c = 'a'; c <= 'z'; ++c) {
    for (const char* b = common; *b; ++b) {
      merges->push_back(sp + std::string(1, c) + " " + std::string(1, *b));
      toks->push_back(sp + std::string(1, c) + std::string(1, *b));
      types->push_back(1);
    }
  }
  const int32_t special_base = vocab - 293;
  while (static_cast<int32_t>(toks->size()) < special_base) {
    char nm[32];
    std::snprintf(nm, sizeof(nm), "tok%d", static_cast<int>(toks->size()));
    toks->push_back(nm);
    types->push_back(1);
  }
  struct Sp {
    int off;
    const char* s;
    int type;
  };
  const Sp named[] = {
      {0, "<|endoftext|>", 3},   {1, "<|im_start|>", 3},   {2, "<|im_end|>", 3},
      {14, "<tool_call>", 4},    {15, "</tool_call>", 4},  {22, "<tool_response>", 4},
      {23, "</tool_response>", 4}, {24, "<think>", 4},       {25, "</think>", 4},
  };
  for (int i = special_base; i < vocab; ++i) {
    const int off = i - special_base;
    const char* nm = nullptr;
    int ty = 5;
    for (const Sp& s : named) {
      if (s.off == off) {
        nm = s.s;
        ty = s.type;
      }
    }
    char buf[48];
    if (nm == nullptr) {
      std::snprintf(buf, sizeof(buf), off < 26 ? "<|reserved_%d|>" : "[PAD%d]", i);
      nm = buf;
      ty = off < 26 ? 3 : 5;
    }
    toks->push_back(nm);
    types->push_back(ty);
  }
  *eos = special_base + 2;  // <|im_end|>
  *pad = special_base + 0;  // <|endoftext|>
}

}  // namespace

extern "C" {

// Model shape for rpgs_write_qwen3_gguf.
struct rpgs_config {
  int32_t n_layers;
  int32_t hidden;
  int32_t ffn;
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t vocab;
  int32_t context;
  float rope_theta;
  float rms_eps;
  uint64_t seed;
  // Q6_K for attn_v / ffn_down on layers with (layer % 2 == q6k_parity); Q4_K otherwise.
  int32_t q6k_parity;
  // standard deviations of the weights and of the norms around 1 (0: the
  // defaults 0.02 and 0.05)
  float weight_std;
  float norm_std;
  // type mix: 0 Q4_K_M (Q4_K, Q6_K), 1 Q5_K_M (Q5_K in place of Q4_K), 2 Q8_0 everywhere
  int32_t mix;
};

int rpgs_quantize_q4k(const float* x, int64_t n, uint8_t* out) {
  if (n <= 0 || n % kQK != 0) return -1;
  for (int64_t b = 0; b < n / kQK; ++b) EncodeQ4KBlock(x + b * kQK, out + b * 144);
  return 0;
}

int rpgs_quantize_q5k(const float* x, int64_t n, uint8_t* out) {
  if (n <= 0 || n % kQK != 0) return -1;
  EncodeRow(kTypeQ5K, x, n, out);
  return 0;
}

int rpgs_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
  if (n <= 0 || n % kQK != 0) return -1;
  EncodeRow(kTypeQ8_0, x, n, out);
  return 0;
}

int rpgs_quantize_q6k(const float* x, int64_t n, uint8_t* out) {
  if (n <= 0 || n % kQK != 0) return -1;
  for (int64_t b = 0; b < n / kQK; ++b) EncodeQ6KBlock(x + b * kQK, out + b * 210);
  return 0;
}

void rpgs_normal(uint64_t seed, int64_t offset, int64_t n, float mean, float stdv, float* out) {
  FillNormal(Mix64(seed), offset, n, mean, stdv, out);
}

uint16_t rpgs_f32_to_f16(float f) { return F32ToF16Rne(f); }

int rpgs_write_qwen3_gguf(const char* path, const rpgs_config* cfg, char* err, int errlen) {
  auto fail = [&](const char* msg) {
    if (err != nullptr && errlen > 0) std::snprintf(err, static_cast<size_t>(errlen), "%s", msg);
    return -1;
  };
  const rpgs_config c = *cfg;
  if (c.hidden % kQK || c.ffn % kQK || (c.n_heads * c.head_dim) % kQK)
    return fail("hidden, ffn and q_dim must be multiples of 256");
  if (c.vocab < 2048) return fail("vocab must be at least 2048");

  const int64_t q_dim = static_cast<int64_t>(c.n_heads) * c.head_dim;
  const int64_t kv_dim = static_cast<int64_t>(c.n_kv_heads) * c.head_dim;

  if (c.mix < 0 || c.mix > 2) return fail("mix must be 0 (Q4_K_M), 1 (Q5_K_M) or 2 (Q8_0)");
  const uint32_t t4 = c.mix == 0 ? kTypeQ4K : (c.mix == 1 ? kTypeQ5K : kTypeQ8_0);
  const uint32_t t6 = c.mix == 2 ? kTypeQ8_0 : kTypeQ6K;
  std::vector<TensorPlan> plan;
  plan.push_back({"token_embd.weight", t6, c.vocab, c.hidden, 0});
  plan.push_back({"output_norm.weight", kTypeF32, 1, c.hidden, 1});
  for (int l = 0; l < c.n_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const bool q6 = (l % 2) == c.q6k_parity;
    plan.push_back({p + "attn_norm.weight", kTypeF32, 1, c.hidden, 1});
    plan.push_back({p + "attn_q.weight", t4, q_dim, c.hidden, 0});
    plan.push_back({p + "attn_k.weight", t4, kv_dim, c.hidden, 0});
    plan.push_back({p + "attn_v.weight", q6 ? t6 : t4, kv_dim, c.hidden, 0});
    plan.push_back({p + "attn_output.weight", t4, c.hidden, q_dim, 0});
    plan.push_back({p + "attn_q_norm.weight", kTypeF32, 1, c.head_dim, 1});
    plan.push_back({p + "attn_k_norm.weight", kTypeF32, 1, c.head_dim, 1});
    plan.push_back({p + "ffn_norm.weight", kTypeF32, 1, c.hidden, 1});
    plan.push_back({p + "ffn_gate.weight", t4, c.ffn, c.hidden, 0});
    plan.push_back({p + "ffn_up.weight", t4, c.ffn, c.hidden, 0});
    plan.push_back({p + "ffn_down.weight", q6 ? t6 : t4, c.hidden, c.ffn, 0});
  }

  const uint64_t align = 32;
  uint64_t off = 0;
  for (TensorPlan& t : plan) {
    t.nbytes = RowBytes(t.type, t.cols) * static_cast<uint64_t>(t.rows);
    t.offset = off;
    off += (t.nbytes + align - 1) / align * align;
  }

  std::vector<std::string> toks, merges;
  std::vector<int32_t> types;
  int32_t eos = 0, pad = 0;
  BuildTokenizer(c.vocab, &toks, &types, &merges, &eos, &pad);

  Buf h;
  h.U32(0x46554747u);  // "GGUF"
  h.U32(3);
  h.U64(plan.size());
  const int n_kv = 22;
  h.U64(n_kv);
  auto kv_str = [&](const char* k, const std::string& v) {
    h.Str(k);
    h.U32(kMStr);
    h.Str(v);
  };
  auto kv_u32 = [&](const char* k, uint32_t v) {
    h.Str(k);
    h.U32(kMU32);
    h.U32(v);
  };
  auto kv_f32 = [&](const char* k, float v) {
    h.Str(k);
    h.U32(kMF32);
    h.F32(v);
  };
  char name[96];
  std::snprintf(name, sizeof(name), "synthetic-qwen3-%dL-%d-seed%llu", c.n_layers, c.hidden,
                static_cast<unsigned long long>(c.seed));
  kv_str("general.architecture", "qwen3");                      // 1
  kv_str("general.name", name);                                 // 2
  kv_u32("general.alignment", static_cast<uint32_t>(align));    // 3
  kv_u32("qwen3.block_count", c.n_layers);                      // 4
  kv_u32("qwen3.context_length", c.context);                    // 5
  kv_u32("qwen3.embedding_length", c.hidden);                   // 6
  kv_u32("qwen3.feed_forward_length", c.ffn);                   // 7
  kv_u32("qwen3.attention.head_count", c.n_heads);              // 8
  kv_u32("qwen3.attention.head_count_kv", c.n_kv_heads);        // 9
  kv_u32("qwen3.attention.key_length", c.head_dim);             // 10
  kv_u32("qwen3.attention.value_length", c.head_dim);           // 11
  kv_f32("qwen3.rope.freq_base", c.rope_theta);                 // 12
  kv_f32("qwen3.attention.layer_norm_rms_epsilon", c.rms_eps);  // 13
  kv_str("tokenizer.ggml.model", "gpt2");                       // 14
  kv_str("tokenizer.ggml.pre", "qwen2");                        // 15
  h.Str("tokenizer.ggml.tokens");                               // 16
  h.U32(kMArr);
  h.U32(kMStr);
  h.U64(toks.size());
  for (const std::string& s : toks) h.Str(s);
  h.Str("tokenizer.ggml.token_type");  // 17
  h.U32(kMArr);
  h.U32(kMI32);
  h.U64(types.size());
  for (int32_t t : types) h.I32(t);
  h.Str("tokenizer.ggml.merges");  // 18
  h.U32(kMArr);
  h.U32(kMStr);
  h.U64(merges.size());
  for (const std::string& s : merges) h.Str(s);
  kv_u32("tokenizer.ggml.eos_token_id", static_cast<uint32_t>(eos));      // 19
  kv_u32("tokenizer.ggml.padding_token_id", static_cast<uint32_t>(pad));  // 20
  kv_u32("tokenizer.ggml.bos_token_id", static_cast<uint32_t>(pad));      // 21
  h.Str("tokenizer.ggml.add_bos_token");                                  // 22
  h.U32(kMBool);
  const uint8_t f = 0;
  h.Raw(&f, 1);

  for (const TensorPlan& t : plan) {
    h.Str(t.name);
    const bool vec = t.rows == 1 && t.kind == 1;
    h.U32(vec ? 1 : 2);
    h.U64(static_cast<uint64_t>(t.cols));
    if (!vec) h.U64(static_cast<uint64_t>(t.rows));
    h.U32(t.type);
    h.U64(t.offset);
  }
  while (h.b.size() % align) h.b.push_back(0);

  FILE* fp = std::fopen(path, "wb");
  if (fp == nullptr) return fail("cannot open the output file");
  bool ok = std::fwrite(h.b.data(), 1, h.b.size(), fp) == h.b.size();

  unsigned nthreads = std::thread::hardware_concurrency();
  if (nthreads == 0) nthreads = 4;
  if (nthreads > 32) nthreads = 32;

  std::vector<uint8_t> data;
  uint64_t written = 0;
  for (size_t ti = 0; ti < plan.size() && ok; ++ti) {
    const TensorPlan& t = plan[ti];
    const uint64_t key = Mix64(c.seed ^ HashName(t.name));
    data.assign(t.nbytes, 0);
    const uint64_t rb = RowBytes(t.type, t.cols);
    auto work = [&](unsigned tid) {
      std::vector<float> row(static_cast<size_t>(t.cols));
      for (int64_t r = tid; r < t.rows; r += nthreads) {
        const float mean = t.kind == 1 ? 1.0f : 0.0f;
        const float stdv = t.kind == 1 ? (c.norm_std > 0.0f ? c.norm_std : 0.05f)
                                       : (c.weight_std > 0.0f ? c.weight_std : 0.02f);
        FillNormal(key, r * t.cols, t.cols, mean, stdv, row.data());
        uint8_t* dst = data.data() + static_cast<uint64_t>(r) * rb;
        if (t.type == kTypeF32) {
          std::memcpy(dst, row.data(), rb);
        } else {
          EncodeRow(t.type, row.data(), t.cols, dst);
        }
      }
    };
    std::vector<std::thread> th;
    for (unsigned i = 0; i < nthreads; ++i) th.emplace_back(work, i);
    for (std::thread& x : th) x.join();
    // pad up to this tensor's offset
    while (written < t.offset && ok) {
      const uint8_t z = 0;
      ok = std::fwrite(&z, 1, 1, fp) == 1;
      ++written;
    }
    ok = ok && std::fwrite(data.data(), 1, data.size(), fp) == data.size();
    written += data.size();
  }
  ok = (std::fclose(fp) == 0) && ok;
  if (!ok) return fail("short write");
  return 0;
}

}  // extern "C"
