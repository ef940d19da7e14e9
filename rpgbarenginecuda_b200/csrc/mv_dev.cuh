// mv_dev.cuh -- the integer tensor-core pieces of the decode matvec, shared
// by the standalone matvec kernel (k_matvec.cu) and the decode loop kernel
// (k_step.cu).
//
// A (tile, super-block) unit is one block group of the repacked layout
// (Q4_K 2304 B, Q6_K 3360 B) in shared memory; x is split per super-block
// into four signed 8-bit digits laid out as the B fragments of
// mma.sync.m16n8k32 (PutDigits).  Lane L = 4g + t accumulates rows g and
// g + 8 of the tile (rg, rg8); FlushPiece folds the four lanes of a row and
// stores the piece into the block's reduction buffer.
#pragma once

#include <cstdint>

#include "kernels.cuh"

namespace rpgb {
namespace mv {

constexpr int kTile = 16;

__device__ __forceinline__ uint4 Lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

// Predicated 16-byte shared load into four loop-carried registers (registers
// of lanes with pred == 0 keep their value).
__device__ __forceinline__ void Lds128If(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t pred,
                                         uint32_t saddr) {
  asm volatile(
      "{ .reg .pred p; setp.ne.u32 p, %4, 0;\n"
      "  @p ld.shared.v4.u32 {%0,%1,%2,%3}, [%5]; }"
      : "+r"(r0), "+r"(r1), "+r"(r2), "+r"(r3)
      : "r"(pred), "r"(saddr));
}

__device__ __forceinline__ void MmaU8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void MmaS8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// PRMT in its default mode: selector nibble bits 0-2 pick a byte of {b, a},
// bit 3 replicates that byte's sign (the __byte_perm intrinsic masks bit 3
// away, so signed extraction needs the instruction itself).
__device__ __forceinline__ uint32_t Prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ int ByteU(uint32_t w, uint32_t sel) { return static_cast<int>(Prmt(w, 0u, sel)); }

// Per-lane constants of the fragment geometry.
struct LaneK {
  int g, tig, p;
  uint32_t sel_q4[2];  // Q4_K scale byte of sub-block 2c + p inside SC_lo / SC_hi (c & 1 = 0, 1)
  uint32_t sel_m[2];   // Q4_K min bytes of sub-blocks 2 tig, 2 tig + 1
  uint32_t sel_q6[2];  // Q6_K signed scale byte h + 2p of word c (h = 0, 1), sign-extended
  float w4[2];         // Q4_K digit weights of the lane's two columns (1/16 for the high nibble half)
  float w6g[2], w6g8[2];  // Q6_K digit weights for rows g and g + 8 (1/4 for a3)
};

__device__ __forceinline__ LaneK MakeLane(int lane) {
  LaneK k;
  k.g = lane >> 2;
  k.tig = lane & 3;
  k.p = k.tig >> 1;
  for (int c = 0; c < 2; ++c) k.sel_q4[c] = 0x4440u | static_cast<uint32_t>(2 * c + k.p);
  k.sel_m[0] = 0x4440u | static_cast<uint32_t>(2 * (k.tig & 1));
  k.sel_m[1] = 0x4440u | static_cast<uint32_t>(2 * (k.tig & 1) + 1);
  for (int h = 0; h < 2; ++h) {
    const uint32_t b = static_cast<uint32_t>(h + 2 * k.p), s = b | 8u;
    k.sel_q6[h] = b | (s << 4) | (s << 8) | (s << 12);
  }
  const float w0 = (k.tig & 1) ? 1.0f / 8192.0f : 1.0f;
  const float w1 = (k.tig & 1) ? 1.0f / 1048576.0f : 1.0f / 64.0f;
  const float f4 = k.p ? 1.0f / 16.0f : 1.0f;
  const float f6 = k.p ? 0.25f : 1.0f;
  k.w4[0] = w0 * f4;
  k.w4[1] = w1 * f4;
  k.w6g[0] = w0;
  k.w6g[1] = w1;
  k.w6g8[0] = w0 * f6;
  k.w6g8[1] = w1 * f6;
  return k;
}

// One Q4_K (tile, super-block) unit: adds the lane's share of rows g, g + 8.
__device__ __forceinline__ void UnitQ4K(const uint8_t* grp, const uint32_t (&bA)[8], const uint32_t (&bB)[8],
                                        const float* sx, float s, const LaneK& k, int lane, float& rg, float& rg8) {
  const uint4 R0 = Lds128(grp + 2048 + 16 * k.g);
  const uint4 R1 = Lds128(grp + 2048 + 16 * (k.g + 8));
  const uint32_t sclo0 = R0.y & 0x3F3F3F3Fu, sclo1 = R1.y & 0x3F3F3F3Fu;
  const uint32_t schi0 = (R0.w & 0x0F0F0F0Fu) | ((R0.y >> 2) & 0x30303030u);
  const uint32_t schi1 = (R1.w & 0x0F0F0F0Fu) | ((R1.y >> 2) & 0x30303030u);
  int acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint4 W = Lds128(grp + (c * 32 + lane) * 16);
    int d[4] = {0, 0, 0, 0};
    MmaU8(d, W.x & 0x0F0F0F0Fu, W.y & 0x0F0F0F0Fu, W.x & 0xF0F0F0F0u, W.y & 0xF0F0F0F0u, bA[2 * c], bB[2 * c]);
    MmaU8(d, W.z & 0x0F0F0F0Fu, W.w & 0x0F0F0F0Fu, W.z & 0xF0F0F0F0u, W.w & 0xF0F0F0F0u, bA[2 * c + 1],
          bB[2 * c + 1]);
    const int s0 = ByteU(c < 2 ? sclo0 : schi0, k.sel_q4[c & 1]);
    const int s1 = ByteU(c < 2 ? sclo1 : schi1, k.sel_q4[c & 1]);
    acc[0] += s0 * d[0];
    acc[1] += s0 * d[1];
    acc[2] += s1 * d[2];
    acc[3] += s1 * d[3];
  }
  // min term of sub-blocks 2 tig and 2 tig + 1
  const uint32_t mlo0 = R0.z & 0x3F3F3F3Fu, mlo1 = R1.z & 0x3F3F3F3Fu;
  const uint32_t mhi0 = ((R0.w >> 4) & 0x0F0F0F0Fu) | ((R0.z >> 2) & 0x30303030u);
  const uint32_t mhi1 = ((R1.w >> 4) & 0x0F0F0F0Fu) | ((R1.z >> 2) & 0x30303030u);
  const uint32_t m0 = k.p ? mhi0 : mlo0, m1 = k.p ? mhi1 : mlo1;
  const float2 sxv = *reinterpret_cast<const float2*>(sx + 2 * k.tig);
  const float mn0 =
      static_cast<float>(ByteU(m0, k.sel_m[0])) * sxv.x + static_cast<float>(ByteU(m0, k.sel_m[1])) * sxv.y;
  const float mn1 =
      static_cast<float>(ByteU(m1, k.sel_m[0])) * sxv.x + static_cast<float>(ByteU(m1, k.sel_m[1])) * sxv.y;
  const float d0 = dev::Half(R0.x & 0xFFFFu), dm0 = dev::Half(R0.x >> 16);
  const float d1 = dev::Half(R1.x & 0xFFFFu), dm1 = dev::Half(R1.x >> 16);
  const float f0 = s * k.w4[0], f1 = s * k.w4[1];
  rg += d0 * (static_cast<float>(acc[0]) * f0 + static_cast<float>(acc[1]) * f1) - dm0 * mn0;
  rg8 += d1 * (static_cast<float>(acc[2]) * f0 + static_cast<float>(acc[3]) * f1) - dm1 * mn1;
}

// One Q6_K (tile, super-block) unit.
__device__ __forceinline__ void UnitQ6K(const uint8_t* grp, const uint32_t (&bA)[8], const uint32_t (&bB)[8], float s,
                                        const LaneK& k, int lane, float& rg, float& rg8) {
  const uint4 S0 = Lds128(grp + 3072 + 16 * k.g);
  const uint4 S1 = Lds128(grp + 3072 + 16 * (k.g + 8));
  const uint32_t dd = *reinterpret_cast<const uint32_t*>(grp + 3328 + 4 * k.g);
  const uint32_t s0w[4] = {S0.x, S0.y, S0.z, S0.w}, s1w[4] = {S1.x, S1.y, S1.z, S1.w};
  int acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint8_t* base = grp + (q * 32 + lane) * 48;
    const uint4 V0 = Lds128(base), V1 = Lds128(base + 16), V2 = Lds128(base + 32);
    const uint32_t v[12] = {V0.x, V0.y, V0.z, V0.w, V1.x, V1.y, V1.z, V1.w, V2.x, V2.y, V2.z, V2.w};
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) {
      const int m = 4 * q + mm, c = m >> 1, h = m & 1;
      const uint32_t X = v[3 * mm], Y = v[3 * mm + 1], Z = v[3 * mm + 2];
      const uint32_t a0 = X & 0x3F3F3F3Fu, a1 = Y & 0x3F3F3F3Fu, a2 = Z & 0x3F3F3F3Fu;
      const uint32_t a3 = ((X >> 4) & 0x0C0C0C0Cu) | ((Y >> 2) & 0x30303030u) | (Z & 0xC0C0C0C0u);
      int d[4] = {0, 0, 0, 0};
      // -32 per weight (x4 for the a3 quarter): d = -32 * sum(B) first
      MmaS8(d, 0xE0E0E0E0u, 0xE0E0E0E0u, 0xE0E0E0E0u, 0x80808080u, bA[m], bB[m]);
      MmaU8(d, a0, a1, a2, a3, bA[m], bB[m]);
      const int sc0 = static_cast<int>(Prmt(s0w[c], 0u, k.sel_q6[h]));
      const int sc1 = static_cast<int>(Prmt(s1w[c], 0u, k.sel_q6[h]));
      acc[0] += sc0 * d[0];
      acc[1] += sc0 * d[1];
      acc[2] += sc1 * d[2];
      acc[3] += sc1 * d[3];
    }
  }
  const float dg = dev::Half(dd & 0xFFFFu), dg8 = dev::Half(dd >> 16);
  rg += dg * s * (static_cast<float>(acc[0]) * k.w6g[0] + static_cast<float>(acc[1]) * k.w6g[1]);
  rg8 += dg8 * s * (static_cast<float>(acc[2]) * k.w6g8[0] + static_cast<float>(acc[3]) * k.w6g8[1]);
}

// One Q5_K (tile, super-block) unit: the Q4_K unit with the 5-bit values
// stored one per byte (no nibble masks, both halves at weight 1).
__device__ __forceinline__ void UnitQ5K(const uint8_t* grp, const uint32_t (&bA)[8], const uint32_t (&bB)[8],
                                        const float* sx, float s, const LaneK& k, int lane, float& rg, float& rg8) {
  const uint4 R0 = Lds128(grp + 4096 + 16 * k.g);
  const uint4 R1 = Lds128(grp + 4096 + 16 * (k.g + 8));
  const uint32_t sclo0 = R0.y & 0x3F3F3F3Fu, sclo1 = R1.y & 0x3F3F3F3Fu;
  const uint32_t schi0 = (R0.w & 0x0F0F0F0Fu) | ((R0.y >> 2) & 0x30303030u);
  const uint32_t schi1 = (R1.w & 0x0F0F0F0Fu) | ((R1.y >> 2) & 0x30303030u);
  int acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint8_t* base = grp + (c * 32 + lane) * 32;
    const uint4 W0 = Lds128(base), W1 = Lds128(base + 16);
    int d[4] = {0, 0, 0, 0};
    MmaU8(d, W0.x, W0.y, W0.z, W0.w, bA[2 * c], bB[2 * c]);
    MmaU8(d, W1.x, W1.y, W1.z, W1.w, bA[2 * c + 1], bB[2 * c + 1]);
    const int s0 = ByteU(c < 2 ? sclo0 : schi0, k.sel_q4[c & 1]);
    const int s1 = ByteU(c < 2 ? sclo1 : schi1, k.sel_q4[c & 1]);
    acc[0] += s0 * d[0];
    acc[1] += s0 * d[1];
    acc[2] += s1 * d[2];
    acc[3] += s1 * d[3];
  }
  const uint32_t mlo0 = R0.z & 0x3F3F3F3Fu, mlo1 = R1.z & 0x3F3F3F3Fu;
  const uint32_t mhi0 = ((R0.w >> 4) & 0x0F0F0F0Fu) | ((R0.z >> 2) & 0x30303030u);
  const uint32_t mhi1 = ((R1.w >> 4) & 0x0F0F0F0Fu) | ((R1.z >> 2) & 0x30303030u);
  const uint32_t m0 = k.p ? mhi0 : mlo0, m1 = k.p ? mhi1 : mlo1;
  const float2 sxv = *reinterpret_cast<const float2*>(sx + 2 * k.tig);
  const float mn0 =
      static_cast<float>(ByteU(m0, k.sel_m[0])) * sxv.x + static_cast<float>(ByteU(m0, k.sel_m[1])) * sxv.y;
  const float mn1 =
      static_cast<float>(ByteU(m1, k.sel_m[0])) * sxv.x + static_cast<float>(ByteU(m1, k.sel_m[1])) * sxv.y;
  const float d0 = dev::Half(R0.x & 0xFFFFu), dm0 = dev::Half(R0.x >> 16);
  const float d1 = dev::Half(R1.x & 0xFFFFu), dm1 = dev::Half(R1.x >> 16);
  const float f0 = s * k.w6g[0], f1 = s * k.w6g[1];
  rg += d0 * (static_cast<float>(acc[0]) * f0 + static_cast<float>(acc[1]) * f1) - dm0 * mn0;
  rg8 += d1 * (static_cast<float>(acc[2]) * f0 + static_cast<float>(acc[3]) * f1) - dm1 * mn1;
}

// One Q8_0 (tile, 256 columns) unit: signed bytes times the signed digits;
// each 32-column block has its own f16 scale, so the block sums are scaled
// in FP32 (they are exact integers below 2^24).
__device__ __forceinline__ void UnitQ8(const uint8_t* grp, const uint32_t (&bA)[8], const uint32_t (&bB)[8], float s,
                                       const LaneK& k, int lane, float& rg, float& rg8) {
  const uint4 S0 = Lds128(grp + 4096 + 16 * k.g);
  const uint4 S1 = Lds128(grp + 4096 + 16 * (k.g + 8));
  const uint32_t s0w[4] = {S0.x, S0.y, S0.z, S0.w}, s1w[4] = {S1.x, S1.y, S1.z, S1.w};
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint8_t* base = grp + (c * 32 + lane) * 32;
    const uint4 W0 = Lds128(base), W1 = Lds128(base + 16);
    int d[4] = {0, 0, 0, 0};
    MmaS8(d, W0.x, W0.y, W0.z, W0.w, bA[2 * c], bB[2 * c]);
    MmaS8(d, W1.x, W1.y, W1.z, W1.w, bA[2 * c + 1], bB[2 * c + 1]);
    // this lane's columns are block 2c + p of rows g and g + 8: f16 at word c, half p
    const float q0 = dev::Half(k.p ? s0w[c] >> 16 : s0w[c] & 0xFFFFu);
    const float q1 = dev::Half(k.p ? s1w[c] >> 16 : s1w[c] & 0xFFFFu);
    a0 += q0 * (static_cast<float>(d[0]) * k.w6g[0] + static_cast<float>(d[1]) * k.w6g[1]);
    a1 += q1 * (static_cast<float>(d[2]) * k.w6g[0] + static_cast<float>(d[3]) * k.w6g[1]);
  }
  rg += s * a0;
  rg8 += s * a1;
}

// One unit of a matrix of type `type` (ggml codes 12 Q4_K, 13 Q5_K, 14 Q6_K, 8 Q8_0).
__device__ __forceinline__ void UnitOf(uint32_t type, const uint8_t* grp, const uint32_t (&bA)[8],
                                       const uint32_t (&bB)[8], const float* sx, float s, const LaneK& k, int lane,
                                       float& rg, float& rg8) {
  if (type == 12u) {
    UnitQ4K(grp, bA, bB, sx, s, k, lane, rg, rg8);
  } else if (type == 14u) {
    UnitQ6K(grp, bA, bB, s, k, lane, rg, rg8);
  } else if (type == 13u) {
    UnitQ5K(grp, bA, bB, sx, s, k, lane, rg, rg8);
  } else {
    UnitQ8(grp, bA, bB, s, k, lane, rg, rg8);
  }
}

__device__ __forceinline__ void FlushPiece(float* red, int piece, const LaneK& k, float& rg, float& rg8) {
  rg += __shfl_xor_sync(0xFFFFFFFFu, rg, 1);
  rg += __shfl_xor_sync(0xFFFFFFFFu, rg, 2);
  rg8 += __shfl_xor_sync(0xFFFFFFFFu, rg8, 1);
  rg8 += __shfl_xor_sync(0xFFFFFFFFu, rg8, 2);
  if (k.tig == 0) {
    red[piece * kTile + k.g] = rg;
    red[piece * kTile + k.g + 8] = rg8;
  }
  rg = rg8 = 0.f;
}


// x -> digits.  v[8] = positions 8 lane .. 8 lane + 7 of super-block b (the
// RMSNorm weight already applied).  Stores the B fragments of b (1024 bytes at
// bfrag + 1024 b), the eight 32-column sums of b (sx[8 b ..]) used by the Q4_K
// min term and the digit scale s (sscale[b]).
//
// s = 2^(e(max|v|) - 5) so |v / s| < 64; Y = round(v / s * 2^20) splits
// exactly into balanced digits x0 (|x0| <= 64), x1 (6 bits), x2, x3 (7 bits).
__device__ __forceinline__ void PutDigits(const float (&v)[8], int b, int lane, uint8_t* bfrag, float* sx,
                                          float* sscale) {
  float mx = 0.f, su = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mx = fmaxf(mx, fabsf(v[i]));
    su += v[i];
  }
  mx = dev::WarpMax(mx);
  const int E = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
  float s = 0.f, inv20 = 0.f;
  if (E >= 25 && E < 255) {
    s = __uint_as_float(static_cast<uint32_t>(E - 5) << 23);
    inv20 = __uint_as_float(static_cast<uint32_t>(279 - E) << 23);
  }
  int d0[8], d1[8], d2[8], d3[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int Y = __float2int_rn(v[i] * inv20);
    d3[i] = (Y << 25) >> 25;
    Y = (Y - d3[i]) >> 7;
    d2[i] = (Y << 25) >> 25;
    Y = (Y - d2[i]) >> 7;
    d1[i] = (Y << 26) >> 26;
    d0[i] = (Y - d1[i]) >> 6;
  }
  auto pack = [](int a, int b_, int c, int d) {
    return __byte_perm(__byte_perm(a, b_, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
  };
  const uint32_t dw[4][2] = {{pack(d0[0], d0[1], d0[2], d0[3]), pack(d0[4], d0[5], d0[6], d0[7])},
                             {pack(d1[0], d1[1], d1[2], d1[3]), pack(d1[4], d1[5], d1[6], d1[7])},
                             {pack(d2[0], d2[1], d2[2], d2[3]), pack(d2[4], d2[5], d2[6], d2[7])},
                             {pack(d3[0], d3[1], d3[2], d3[3]), pack(d3[4], d3[5], d3[6], d3[7])}};
  // positions 8 lane .. 8 lane + 7 = 64c + 32hb + 16h + 8(lane & 1) + i
  const int c = lane >> 3, hb = (lane >> 2) & 1, h = (lane >> 1) & 1, tb = 2 * (lane & 1);
  const int m = 2 * c + h;
  uint32_t* bw = reinterpret_cast<uint32_t*>(bfrag + static_cast<size_t>(b) * 1024);
#pragma unroll
  for (int dg = 0; dg < 4; ++dg) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int Lp = 4 * (dg + 4 * hb) + tb + j;
      bw[((m >> 2) * 32 + Lp) * 4 + (m & 3)] = dw[dg][j];
    }
  }
  su += __shfl_xor_sync(0xFFFFFFFFu, su, 1);
  su += __shfl_xor_sync(0xFFFFFFFFu, su, 2);
  if ((lane & 3) == 0) sx[b * 8 + (lane >> 2)] = su;
  if (lane == 0) sscale[b] = s;
}

// The B fragments of super-block b for this lane: lanes g < 4 own columns
// 0-3 (B rows 0..15, register b0), lanes g >= 4 columns 4-7 (rows 16..31,
// register b1); the other register stays 0.
__device__ __forceinline__ void LoadB(const uint8_t* bfrag, int b, int lane, uint32_t lo_half, uint32_t (&bA)[8],
                                      uint32_t (&bB)[8]) {
  const uint32_t baddr = dev::SmemAddr(bfrag + static_cast<size_t>(b) * 1024 + lane * 16);
  const uint32_t hi_half = 1u - lo_half;
  Lds128If(bA[0], bA[1], bA[2], bA[3], lo_half, baddr);
  Lds128If(bA[4], bA[5], bA[6], bA[7], lo_half, baddr + 512);
  Lds128If(bB[0], bB[1], bB[2], bB[3], hi_half, baddr);
  Lds128If(bB[4], bB[5], bB[6], bB[7], hi_half, baddr + 512);
}

}  // namespace mv
}  // namespace rpgb
