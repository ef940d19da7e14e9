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

#include "kernels.h"
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

// ------------------------------------------------------------------ weight layout
//
// Matrices are 16-row tiles; block group (tile, super-block b) holds the 16
// GGUF blocks in the byte order documented at RepackTile (model.cu).  Lane
// L = 4g + t of a warp owns tile rows g and g + 8 in the integer MMA
// fragments; the accessors below address single elements for the bit-exact
// dequant paths.
__host__ __device__ __forceinline__ int GroupBytesOf(uint32_t type) {
  return type == 12u ? 2304 : (type == 14u ? 3360 : kByteGroupBytes);
}

__device__ __forceinline__ const uint8_t* GroupPtr(const DevMat& w, int64_t row, int b) {
  return w.q + ((row >> 4) * w.nb + b) * GroupBytesOf(w.type);
}

// 4-bit value of element e (0..255) of Q4_K tile row r (0..15).
__device__ __forceinline__ int Q4kNibble(const uint8_t* grp, int r, int e) {
  const int j = e >> 5, p = e & 31;
  const int c = j >> 1, h = p >> 4, t = (p >> 2) & 3, ee = p & 3;
  const int g = r & 7, rs = r >> 3;
  const uint8_t byte = grp[(c * 32 + 4 * g + t) * 16 + (2 * h + rs) * 4 + ee];
  return (j & 1) ? (byte >> 4) : (byte & 15);
}

// 6-bit value of element e (0..255) of a Q6_K tile row r (0..15).
__device__ __forceinline__ int Q6kValue(const uint8_t* grp, int r, int e) {
  const int j = e >> 4, pos = e & 15;
  const int c = j >> 2, h = j & 1, hb = (j >> 1) & 1;
  const int m = 2 * c + h, t = pos >> 2, ee = pos & 3;
  const int g = r & 7, rs = r >> 3;
  const uint8_t* w = grp + ((m >> 2) * 32 + 4 * g + t) * 48 + (m & 3) * 12;
  if (hb == 0) return (rs == 0 ? w[ee] : w[4 + ee]) & 63;
  if (rs == 0) return w[8 + ee] & 63;
  return (w[ee] >> 6) | ((w[4 + ee] >> 6) << 2) | ((w[8 + ee] >> 6) << 4);
}

// Byte of element e (0..255) of tile row r (0..15) in a Q5_K / Q8_0 group.
__device__ __forceinline__ uint8_t ByteGroupValue(const uint8_t* grp, int r, int e) {
  const int c = e >> 6, half = (e >> 5) & 1, h = (e >> 4) & 1, t = (e >> 2) & 3, ee = e & 3;
  const int g = r & 7, rs = r >> 3;
  return grp[(c * 32 + 4 * g + t) * 32 + 4 * (4 * h + 2 * half + rs) + ee];
}

// ------------------------------------------------------------------ element dequant (bit-exact)

// Element e (0..255) of Q4_K block b of `row`.
__device__ __forceinline__ float DeqQ4K(const DevMat& w, int64_t row, int b, int e) {
  const uint8_t* grp = GroupPtr(w, row, b);
  const int r = static_cast<int>(row & 15);
  const uint4 h = *reinterpret_cast<const uint4*>(grp + 2048 + 16 * r);
  int sc, m;
  Q4kScaleMin(h.y, h.z, h.w, e >> 5, &sc, &m);
  const int raw = Q4kNibble(grp, r, e);
  const float d = Half(h.x & 0xFFFFu), dmin = Half(h.x >> 16);
  const float d1 = __fmul_rn(d, static_cast<float>(sc));
  const float m1 = __fmul_rn(dmin, static_cast<float>(m));
  return __fsub_rn(__fmul_rn(d1, static_cast<float>(raw)), m1);
}

// Element e (0..255) of Q6_K block b of `row`.
__device__ __forceinline__ float DeqQ6K(const DevMat& w, int64_t row, int b, int e) {
  const uint8_t* grp = GroupPtr(w, row, b);
  const int r = static_cast<int>(row & 15);
  const int raw = Q6kValue(grp, r, e) - 32;
  const int8_t sc = static_cast<int8_t>(grp[3072 + 16 * r + (e >> 4)]);
  const float d = Half(*reinterpret_cast<const uint16_t*>(grp + 3328 + 2 * (2 * (r & 7) + (r >> 3))));
  return __fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(raw));
}

// Element e (0..255) of Q5_K block b of `row` (src/quant.cc:281-313).
__device__ __forceinline__ float DeqQ5K(const DevMat& w, int64_t row, int b, int e) {
  const uint8_t* grp = GroupPtr(w, row, b);
  const int r = static_cast<int>(row & 15);
  const uint4 h = *reinterpret_cast<const uint4*>(grp + 4096 + 16 * r);
  int sc, m;
  Q4kScaleMin(h.y, h.z, h.w, e >> 5, &sc, &m);
  const int raw = ByteGroupValue(grp, r, e);
  const float d = Half(h.x & 0xFFFFu), dmin = Half(h.x >> 16);
  const float d1 = __fmul_rn(d, static_cast<float>(sc));
  const float m1 = __fmul_rn(dmin, static_cast<float>(m));
  return __fsub_rn(__fmul_rn(d1, static_cast<float>(raw)), m1);
}

// Element e (0..255) of the 256 columns b of a Q8_0 `row` (src/quant.cc:132-141).
__device__ __forceinline__ float DeqQ8(const DevMat& w, int64_t row, int b, int e) {
  const uint8_t* grp = GroupPtr(w, row, b);
  const int r = static_cast<int>(row & 15);
  const int8_t q = static_cast<int8_t>(ByteGroupValue(grp, r, e));
  const float d = Half(*reinterpret_cast<const uint16_t*>(grp + 4096 + 16 * r + 2 * (e >> 5)));
  return __fmul_rn(static_cast<float>(q), d);
}

__device__ __forceinline__ float DeqElem(const DevMat& w, int64_t row, int col) {
  switch (w.type) {
    case 12u: return DeqQ4K(w, row, col >> 8, col & 255);
    case 13u: return DeqQ5K(w, row, col >> 8, col & 255);
    case 8u: return DeqQ8(w, row, col >> 8, col & 255);
    default: return DeqQ6K(w, row, col >> 8, col & 255);
  }
}

// ------------------------------------------------------------------ async copy / PDL primitives

__device__ __forceinline__ uint32_t SmemAddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void MbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(SmemAddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void MbarInitFence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void MbarExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(SmemAddr(bar)), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> shared, completion counted on `bar` (16-byte aligned,
// size a multiple of 16).  No multicast.
__device__ __forceinline__ void BulkG2S(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   SmemAddr(dst)),
               "l"(src), "r"(bytes), "r"(SmemAddr(bar))
               : "memory");
}
__device__ __forceinline__ void PrefetchL2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void FenceProxyAsync() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ bool MbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  // The suspend-time hint (ns) lets a waiting warp sleep until the phase
  // completes instead of re-issuing the test, which frees issue slots for
  // the warps that have data.
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(SmemAddr(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false after `limit` attempts (each suspends for at
// most ~20 us) instead of waiting forever.
__device__ __forceinline__ bool MbarWait(uint64_t* bar, uint32_t parity, uint32_t limit = 1u << 16) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (MbarTryWait(bar, parity)) return true;
  }
  return false;
}
// Programmatic dependent launch: let the next kernel in the stream start its
// prologue / wait until the previous kernel's results are visible.  Both are
// no-ops for a launch without the programmatic-serialization attribute.
__device__ __forceinline__ void GridLaunchDependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void GridWait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ timeline trace

__device__ __forceinline__ uint64_t GlobalTimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Records one TraceRec per block (thread 0) when the trace buffer is set:
// construct at kernel entry, call Ready() after GridWait(); Mark(k) notes the
// time of phase k (1..4).  Everything is written when the scope ends (every
// return path included), with one atomic per block, so the marks do not slow
// the block down.
struct TraceScope {
  static constexpr int kMaxMarks = 4;
  const Trace& t;
  uint64_t t0 = 0, tr = 0;
  uint64_t mt[kMaxMarks];
  uint32_t mk[kMaxMarks];
  int nm = 0;
  __device__ explicit TraceScope(const Trace& tr_) : t(tr_) {
    if (t.rec != nullptr && threadIdx.x == 0) t0 = GlobalTimer();
  }
  __device__ void Ready() {
    if (t.rec != nullptr && threadIdx.x == 0) tr = GlobalTimer();
  }
  // Phase mark k: a record whose block field carries k << 24 and whose t_end
  // is the time of the mark (thread 0's view; callers place marks after a
  // barrier so the whole block has reached them).
  __device__ void Mark(uint32_t k) {
    if (t.rec != nullptr && threadIdx.x == 0 && nm < kMaxMarks) {
      mt[nm] = GlobalTimer();
      mk[nm] = k;
      ++nm;
    }
  }
  __device__ ~TraceScope() {
    if (t.rec != nullptr && threadIdx.x == 0) {
      const uint64_t t1 = GlobalTimer();
      const uint32_t i = atomicAdd(t.count, 1u + static_cast<uint32_t>(nm));
      Put(i, 0u, t1);
      for (int j = 0; j < nm; ++j) Put(i + 1 + j, mk[j], mt[j]);
    }
  }
  __device__ void Put(uint32_t i, uint32_t k, uint64_t t1) const {
    if (i < t.cap) {
      TraceRec r;
      r.id = static_cast<uint32_t>(t.id);
      r.block = (blockIdx.x + gridDim.x * blockIdx.y) | (k << 24);
      r.t_start = t0;
      r.t_ready = tr ? tr : t0;
      r.t_end = t1;
      t.rec[i] = r;
    }
  }
};

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
