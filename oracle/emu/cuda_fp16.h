// SIMT emulation layer: IEEE binary16 storage type.  TEST INFRASTRUCTURE ONLY
// (see cuda_runtime_api.h).  Conversions are written from the IEEE 754
// definition: float -> half rounds to nearest, ties to even, with overflow to
// infinity and gradual underflow; half -> float is exact.
#ifndef RPG_ORACLE_EMU_CUDA_FP16_H_
#define RPG_ORACLE_EMU_CUDA_FP16_H_

#include <cmath>
#include <cstdint>
#include <cstring>

struct __half {
  uint16_t bits;
};

inline uint16_t RpgEmuF32ToF16Bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);  // >= 65520 rounds to infinity
  if (ax < 0x38800000u) {
    // below 2^-14: a multiple of 2^-24; scaling by 2^24 is exact and the
    // default rounding mode (nearest, ties to even) gives the count (1024 is
    // the smallest normal, whose bit pattern is that same integer)
    float a;
    std::memcpy(&a, &ax, 4);
    return static_cast<uint16_t>(sign | static_cast<uint32_t>(std::nearbyint(a * 16777216.0f)));
  }
  const uint32_t e = (ax >> 23) - 127u + 15u;
  const uint32_t m = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(sign | h);
}

inline float RpgEmuF16BitsToF32(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  uint32_t x;
  if (e == 0) {
    float v = static_cast<float>(m) * (1.0f / 16777216.0f);
    std::memcpy(&x, &v, 4);
    x |= sign;
  } else if (e == 31) {
    x = sign | 0x7F800000u | (m << 13);
  } else {
    x = sign | ((e - 15u + 127u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

inline __half __float2half_rn(float f) { return __half{RpgEmuF32ToF16Bits(f)}; }
inline __half __float2half(float f) { return __float2half_rn(f); }
inline float __half2float(__half h) { return RpgEmuF16BitsToF32(h.bits); }
inline unsigned short __half_as_ushort(__half h) { return h.bits; }
inline __half __ushort_as_half(unsigned short b) { return __half{b}; }

#endif  // RPG_ORACLE_EMU_CUDA_FP16_H_
