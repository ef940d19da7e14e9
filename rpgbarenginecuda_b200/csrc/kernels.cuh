// kernels.cuh -- device helpers shared by the sm_100a kernels.
//
// Dequantisation follows the reference's per-element definitions exactly
// (src/quant_gpu.cuh:92-161, src/quant.cc:252-277 and 321-354):
//   Q4_K  w = (d*sc)*q - (dmin*m)   with each product rounded separately
//   Q6_K  w = (d*sc)*(q - 32)
// The fused dot products below regroup the same terms per 32-element (Q4_K)
// or 16-element (Q6_K) sub-block: (d*sc) * sum(q*x) - (dmin*m) * sum(x).  That
// is a different rounding order from the reference's per-element dequant, so
// matvec parity is a tolerance check; the element-wise entry points
// (DeqQ4K/DeqQ6K) are bit-exact.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "model.h"

namespace rpgb {
namespace dev {

__device__ __forceinline__ float Half(uint32_t h16) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h16))); }

// Byte K of w placed in the mantissa of 2^23: returns 8388608 + byte exactly.
template <int K>
__device__ __forceinline__ float ByteBiased(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | K));
}

__device__ __forceinline__ uint32_t ByteOf(uint32_t w, int i) { return (w >> (8 * i)) & 0xFFu; }

// 6-bit scale and min of Q4_K sub-block j (0..7); sy/sz/sw are the 12 packed
// scale bytes (bytes 4..15 of the block).  Same bit layout as
// GetScaleMinK4 (src/quant.cc:159-167).
__device__ __forceinline__ void Q4kScaleMin(uint32_t sy, uint32_t sz, uint32_t sw, int j, int* sc, int* m) {
  const int i = j & 3;
  const uint32_t by = ByteOf(sy, i), bz = ByteOf(sz, i), bw = ByteOf(sw, i);
  if (j < 4) {
    *sc = static_cast<int>(by & 63u);
    *m = static_cast<int>(bz & 63u);
  } else {
    *sc = static_cast<int>((bw & 0x0Fu) | ((by >> 6) << 4));
    *m = static_cast<int>((bw >> 4) | ((bz >> 6) << 4));
  }
}

// Signed scale byte i (0..15) out of a 16-byte Q6_K scale record.
__device__ __forceinline__ int Q6kScale(const uint4& s, int i) {
  const uint32_t w = i < 4 ? s.x : (i < 8 ? s.y : (i < 12 ? s.z : s.w));
  return static_cast<int>(static_cast<int8_t>(ByteOf(w, i & 3)));
}

// ------------------------------------------------------------------ element dequant (bit-exact)

// Element e (0..255) of Q4_K block `blk` of a repacked matrix.
__device__ __forceinline__ float DeqQ4K(const DevMat& w, int64_t blk, int e) {
  const uint8_t* hd = w.s + blk * 16;
  const uint32_t d_dm = *reinterpret_cast<const uint32_t*>(hd);
  const uint4 h = *reinterpret_cast<const uint4*>(hd);
  const int sub = e >> 5, l = e & 31;
  int sc, m;
  Q4kScaleMin(h.y, h.z, h.w, sub, &sc, &m);
  const uint8_t byte = w.q[blk * 128 + (sub >> 1) * 32 + l];
  const int raw = (sub & 1) ? (byte >> 4) : (byte & 15);
  const float d = Half(d_dm & 0xFFFFu), dmin = Half(d_dm >> 16);
  const float d1 = __fmul_rn(d, static_cast<float>(sc));
  const float m1 = __fmul_rn(dmin, static_cast<float>(m));
  return __fsub_rn(__fmul_rn(d1, static_cast<float>(raw)), m1);
}

// Element e (0..255) of Q6_K block `blk` of a repacked matrix.
__device__ __forceinline__ float DeqQ6K(const DevMat& w, int64_t blk, int e) {
  const int hh = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
  const uint8_t* base = w.q + blk * 192;
  const uint8_t byte = base[hh * 64 + l + ((quarter & 1) ? 32 : 0)];
  const int nib = quarter < 2 ? (byte & 15) : (byte >> 4);
  const int hi = (base[128 + hh * 32 + l] >> (2 * quarter)) & 3;
  const int raw = (nib | (hi << 4)) - 32;
  const int8_t sc = static_cast<int8_t>(w.s[blk * 16 + hh * 8 + (l >> 4) + 2 * quarter]);
  const float d = Half(w.d[blk]);
  return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(raw));
}

__device__ __forceinline__ float DeqElem(const DevMat& w, int64_t row, int col) {
  const int64_t blk = row * w.nb + (col >> 8);
  return w.type == 12u ? DeqQ4K(w, blk, col & 255) : DeqQ6K(w, blk, col & 255);
}

// ------------------------------------------------------------------ reductions

__device__ __forceinline__ float WarpSum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ double WarpSumD(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ float WarpMax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Block-wide double sum; every thread gets the total.  `sh` holds >= 32 doubles.
// The summation order is fixed (warp butterfly, then warps in index order).
__device__ __forceinline__ double BlockSumD(double v, double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = WarpSumD(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += sh[i];
  return t;
}

__device__ __forceinline__ float BlockMax(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = WarpMax(v);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = sh[0];
  for (int i = 1; i < nw; ++i) t = fmaxf(t, sh[i]);
  return t;
}

// Order-preserving float -> uint32 key (same mapping as the reference sampler,
// src/sampler_gpu.cu:74-82).
__device__ __forceinline__ uint32_t OrderKey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float FromOrderKey(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Counter-based uniform u = H(seed, counter): the reference's SplitMix64
// construction (src/sampler_gpu.cu:42-56), restated.
__host__ __device__ __forceinline__ uint64_t SplitMix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__host__ __device__ __forceinline__ float CounterUniform(uint64_t seed, uint64_t counter) {
  const uint32_t bits = static_cast<uint32_t>(SplitMix64(seed + 0x9E3779B97F4A7C15ull * counter) >> 40);
  return static_cast<float>(bits) * (1.0f / 16777216.0f);
}

// Streaming 16-byte load for weights read once per step (skip L1 allocation).
__device__ __forceinline__ uint4 LdStream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace dev
}  // namespace rpgb
