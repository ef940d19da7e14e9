// k_flash.cu -- prefill attention on the 5th-generation tensor cores
// (tcgen05, flash-attention style).
//
// Replaces AttentionFromCacheKernel for prompts (src/kernels_gpu.cu:737-823,
// GpuAttentionFromCache at 1038-1087): causal GQA over the fp16 KV cache,
// scale 1/sqrt(128), softmax with max subtraction, output = P V / sum P.
//
// One block per (tile of 128 / G query tokens, KV head h): its 128 rows are
// the (q head, token) pairs of the G q heads sharing h, so every K/V tile is
// read once per query tile instead of once per token; the rows are the 128
// TMEM lanes of the score tile S = Q K^T and of the output accumulator
// O += P V, both tcgen05 MMAs with operands in shared memory.  K and V are
// fp16 already (exact); Q and P are split into two fp16 terms (hi + lo), so
// scores and outputs keep about 22 significant bits (the reference computes
// them in FP32).  FlashTcKernel below has the pipeline.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "tc_dev.cuh"

namespace rpgb {
namespace {

constexpr int kD = 128;
constexpr int kKT = 64;        // key positions per stage
constexpr int kRows = 128;  // (q head, token) rows per block
constexpr uint32_t kHalfTile = kKT * 64 * 2;  // 64 positions x 64 dims fp16 = 8 KB (one swizzled box)

struct FlashArgs {
  const float* q;  // [n][q_stride], normalised and rotated
  int32_t q_stride;
  float* out;  // [n][q_dim]
  int32_t n, n_heads;
  int64_t pos0;  // position of query 0
  float scale;
  unsigned* err;
  // key splits (gridDim.z > 1): unnormalised O [split][n][q_dim] and
  // {row max, row sum} [split][n][n_heads][2]
  float* part_o;
  float* part_ml;
};

__device__ __forceinline__ uint32_t PackHalf2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// fp16 hi/lo split of a pair of floats.
__device__ __forceinline__ void SplitPair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = PackHalf2(a - hf.x, b - hf.y);
}

__device__ __forceinline__ void TmaLoad3D(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dev::SmemAddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(dev::SmemAddr(bar))
      : "memory");
}

// ------------------------------------------------------------------ tcgen05 version
//
// One block of 10 warps per (128 / G query tokens, KV head); its 128 rows
// are (q head g, token) pairs, head-major (row r = g * 128 / G + token), and
// they are the 128 TMEM lanes:
//  * warp 8 streams K and V tiles of 64 positions (3-D TMA, 128-byte
//    swizzle, two stages);
//  * warp 9 issues S = Q K^T (M 128, N 64: Qh K + Ql K, 16 MMAs) into one of
//    two 64-column TMEM tiles, one tile ahead of the softmax, then
//    O += P V (M 128, N 128: Ph Vt + Pl Vt, 8 MMAs) into a 128-column TMEM
//    accumulator;
//  * warps 0-7, two per row (warp w and w + 4 share TMEM lanes 32 (w % 4) ..
//    and take 32 of the 64 keys and 64 of the 128 dims each) read their S
//    half-row, apply the causal mask and the online softmax in log2 units
//    (the row maximum exchanged through shared memory), rescale their O
//    half-row in TMEM when the maximum grew, write P = Ph + Pl (fp16 terms)
//    into a K-major swizzled tile, and transpose V into a K-major tile Vt
//    (thread = dim), which the MMA needs as its B operand.
// Q (times scale * log2 e) is split into Qh + Ql fp16 terms once per block.
// Every mbarrier wait is bounded; a wait that gives up sets *err (64).
constexpr int kTcWarps = 10;  // 8 softmax warps, the TMA warp, the MMA warp
constexpr int kSoftThreads = 256;
constexpr uint32_t kQBox = 128 * 128;          // 128 rows x 64 dims fp16 (one swizzled box)
constexpr uint32_t kTcQ = 2 * kQBox;            // 128 rows x 128 dims
constexpr uint32_t kTcStage = 4 * kHalfTile;    // K dims 0-63, K dims 64-127, V dims 0-63, V dims 64-127
constexpr uint32_t kTcTile = 128 * 128;         // 128 rows x 64 keys fp16 (P, Vt)
constexpr size_t kTcSmem = 2 * kTcQ + 2 * kTcStage + 3 * kTcTile + 1024;

__device__ __forceinline__ uint32_t Swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kTcWarps * 32, 1)
    FlashTcKernel(const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV, const FlashArgs a) {
  using namespace tc;
  constexpr int kTQ = kRows / G;  // query tokens per block
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t kv_full[2], kv_empty[2], s_full[2], s_free[2], p_full, o_done, fin;
  __shared__ uint32_t s_tmem;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQh = smem;
  uint8_t* sQl = sQh + kTcQ;
  uint8_t* sKV = sQl + kTcQ;
  uint8_t* sVt = sKV + 2 * kTcStage;
  uint8_t* sPh = sVt + kTcTile;
  uint8_t* sPl = sPh + kTcTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y;
  // the last query tiles see the most keys (causal): they are launched first
  const int tok0 = (gridDim.x - 1 - blockIdx.x) * kTQ;
  const int64_t last_tok = (tok0 + kTQ < a.n ? tok0 + kTQ : a.n) - 1;
  const int64_t kend = a.pos0 + last_tok + 1;
  const int tiles = static_cast<int>((kend + kKT - 1) / kKT);
  const int n_split = static_cast<int>(gridDim.z), z = static_cast<int>(blockIdx.z);
  const int t_lo = static_cast<int>(static_cast<int64_t>(z) * tiles / n_split);
  const int nsteps = static_cast<int>(static_cast<int64_t>(z + 1) * tiles / n_split) - t_lo;

  if (warp == 0) TmemAlloc(&s_tmem, 256u);  // O: columns 0-127, S tiles: 128-191, 192-255
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      dev::MbarInit(kv_full + b, 1);
      dev::MbarInit(kv_empty + b, 1);
      dev::MbarInit(s_full + b, 1);
      dev::MbarInit(s_free + b, kSoftThreads);
    }
    dev::MbarInit(&p_full, kSoftThreads);
    dev::MbarInit(&o_done, 1);
    dev::MbarInit(&fin, 1);
    dev::MbarInitFence();
  }
  // ---- Q rows (warps 0-7: thread = row, half hh of the dims): q * scale * log2 e as fp16 hi + lo, swizzled
  const int row = tid & 127, hh = (tid >> 7) & 1;
  const int g = row / kTQ, tl = row - g * kTQ;
  const int qh = h * G + g;
  const int64_t qpos = a.pos0 + tok0 + tl;
  if (warp < 8) {
    const bool valid = tok0 + tl < a.n;
    const float* q = a.q + static_cast<int64_t>(valid ? tok0 + tl : 0) * a.q_stride + qh * kD;
    const float qs = a.scale * 1.4426950408889634f;
#pragma unroll 4
    for (int c = 8 * hh; c < 8 * hh + 8; ++c) {  // 8 dims per chunk
      const float4 x0 = *reinterpret_cast<const float4*>(q + 8 * c);
      const float4 x1 = *reinterpret_cast<const float4*>(q + 8 * c + 4);
      const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      uint32_t hi[4], lo[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float u0 = valid ? v[2 * i] * qs : 0.f, u1 = valid ? v[2 * i + 1] * qs : 0.f;
        SplitPair(u0, u1, hi[i], lo[i]);
      }
      const uint32_t off = (c >> 3) * kQBox + Swz(row, c & 7);
      *reinterpret_cast<uint4*>(sQh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(sQl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    dev::FenceProxyAsync();  // generic-proxy writes, read by the MMAs (async proxy)
  }
  FenceBeforeSync();
  __syncthreads();
  FenceAfterSync();
  const uint32_t tmem = s_tmem;

  if (warp == 8) {
    if (lane == 0) {
      // ---- producer: K and V tiles t_lo .. t_lo + nsteps - 1
      int issued = 0;
      for (int i = 0; i < nsteps; ++i) {
        const int b = i & 1;
        if (i >= 2 && !dev::MbarWait(kv_empty + b, static_cast<uint32_t>(((i >> 1) - 1) & 1))) {
          atomicOr(a.err, 64u);
          break;
        }
        uint8_t* st = sKV + b * kTcStage;
        const int y = (t_lo + i) * kKT;
        dev::MbarExpectTx(kv_full + b, kTcStage);
        TmaLoad3D(st, &mK, 0, y, h, kv_full + b);
        TmaLoad3D(st + kHalfTile, &mK, 64, y, h, kv_full + b);
        TmaLoad3D(st + 2 * kHalfTile, &mV, 0, y, h, kv_full + b);
        TmaLoad3D(st + 3 * kHalfTile, &mV, 64, y, h, kv_full + b);
        issued = i + 1;
      }
      for (int i = issued - 2 > 0 ? issued - 2 : 0; i < issued; ++i) {  // copies land before exit
        dev::MbarWait(kv_full + (i & 1), static_cast<uint32_t>((i >> 1) & 1));
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      // ---- MMA issuer
      constexpr uint32_t id_s = InstrDesc(128, kKT), id_o = InstrDesc(128, kD);
      const uint64_t dQh = DescSw128(sQh), dQl = DescSw128(sQl);
      const uint64_t dPh = DescSw128(sPh), dPl = DescSw128(sPl), dVt = DescSw128(sVt);
      bool bad = false;
      auto issue_s = [&](int j) {
        const int b = j & 1;
        if (!dev::MbarWait(kv_full + b, static_cast<uint32_t>((j >> 1) & 1)) ||
            (j >= 2 && !dev::MbarWait(s_free + b, static_cast<uint32_t>(((j >> 1) - 1) & 1)))) {
          atomicOr(a.err, 64u);
          bad = true;
          return;
        }
        FenceAfterSync();
        const uint8_t* st = sKV + b * kTcStage;
        const uint32_t ts = tmem + 128u + static_cast<uint32_t>(b) * kKT;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t adv = static_cast<uint64_t>((kk & 3) * 2);  // 16 fp16 = 32 bytes along K
          const uint64_t dK = DescSw128(st + (kk >> 2) * kHalfTile) + adv;
          Mma(ts, dQh + (kk >> 2) * (kQBox >> 4) + adv, dK, id_s, kk > 0 ? 1u : 0u);
          Mma(ts, dQl + (kk >> 2) * (kQBox >> 4) + adv, dK, id_s, 1u);
        }
        MmaCommit(s_full + b);
      };
      if (nsteps > 0) issue_s(0);
      for (int j = 0; j < nsteps && !bad; ++j) {
        if (j + 1 < nsteps) {
          issue_s(j + 1);
          if (bad) break;
        }
        if (!dev::MbarWait(&p_full, static_cast<uint32_t>(j & 1))) {
          atomicOr(a.err, 64u);
          break;
        }
        FenceAfterSync();
#pragma unroll
        for (int kk = 0; kk < kKT / 16; ++kk) {
          const uint64_t adv = static_cast<uint64_t>(kk * 2);
          Mma(tmem, dPh + adv, dVt + adv, id_o, (j > 0 || kk > 0) ? 1u : 0u);
          Mma(tmem, dPl + adv, dVt + adv, id_o, 1u);
        }
        MmaCommit(&o_done);
        MmaCommit(kv_empty + (j & 1));
      }
      // every MMA issued by this thread has completed before the block may exit
      MmaCommit(&fin);
      dev::MbarWait(&fin, 0u);
    }
  } else {
    // ---- softmax, P, Vt and the output (warps 0-7: thread = row, half hh of
    // the 64 keys of S and of the 128 dims of O)
    __shared__ float s_mx[2][2][128];  // [tile parity][half][row]
    __shared__ float s_l[128];
    const uint32_t lrow = static_cast<uint32_t>(32 * (warp & 3)) << 16;  // this warp's TMEM lanes
    constexpr int kHK = kKT / 2;  // keys per half
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // A wait that gives up clears ok (warp-uniform); the loop still runs
    // every iteration's named barrier, so the other half never waits alone.
    for (int j = 0; j < nsteps; ++j) {
      const int b = j & 1;
      if (ok && !__all_sync(0xFFFFFFFFu, dev::MbarWait(s_full + b, static_cast<uint32_t>((j >> 1) & 1)))) ok = false;
      float p[kHK];
      float mx = -INFINITY;
      if (ok) {
        FenceAfterSync();
#pragma unroll
        for (int c0 = 0; c0 < kHK; c0 += 16) {
          uint32_t v[16];
          TmemLoad16(tmem + lrow + 128u + static_cast<uint32_t>(b * kKT + hh * kHK + c0), v);
#pragma unroll
          for (int i = 0; i < 16; ++i) p[c0 + i] = __uint_as_float(v[i]);
        }
        FenceBeforeSync();
        MbarArrive(s_free + b);
        // causal mask: keys past this row's position (lim = last visible key of the half)
        const int64_t rel = qpos - (static_cast<int64_t>(t_lo + j) * kKT + hh * kHK);
        const int lim = rel < -1 ? -1 : (rel > kHK ? kHK : static_cast<int>(rel));
        if (__any_sync(0xFFFFFFFFu, lim < kHK - 1)) {
#pragma unroll
          for (int c = 0; c < kHK; ++c) p[c] = c > lim ? -INFINITY : p[c];
        }
#pragma unroll
        for (int c = 0; c < kHK; ++c) mx = fmaxf(mx, p[c]);
      }
      // the row maximum over both halves
      s_mx[b][hh][row] = mx;
      asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
      if (!ok) continue;
      mx = fmaxf(mx, s_mx[b][hh ^ 1][row]);
      const float m_new = fmaxf(m_run, mx);
      const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
      float ps = 0.f;
      if (m_new == -INFINITY) {  // no visible key yet in this row
#pragma unroll
        for (int c = 0; c < kHK; ++c) p[c] = 0.f;
      } else {
#pragma unroll
        for (int c = 0; c < kHK; ++c) {
          p[c] = exp2f(p[c] - m_new);  // exp2(-inf) = 0 for masked keys
          ps += p[c];
        }
      }
      l_run = l_run * alpha + ps;  // this half's share of the row sum
      m_run = m_new;
      if (j > 0) {
        if (!__all_sync(0xFFFFFFFFu, dev::MbarWait(&o_done, static_cast<uint32_t>((j - 1) & 1)))) {
          ok = false;
          continue;
        }
        FenceAfterSync();
        if (__any_sync(0xFFFFFFFFu, alpha != 1.f)) {
#pragma unroll 2
          for (int c0 = 64 * hh; c0 < 64 * hh + 64; c0 += 16) {
            uint32_t v[16];
            TmemLoad16(tmem + lrow + static_cast<uint32_t>(c0), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            TmemStore16(tmem + lrow + static_cast<uint32_t>(c0), v);
          }
          TmemStoreWait();
        }
      }
#pragma unroll
      for (int c = 0; c < kHK / 8; ++c) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) SplitPair(p[8 * c + 2 * i], p[8 * c + 2 * i + 1], hi[i], lo[i]);
        *reinterpret_cast<uint4*>(sPh + Swz(row, 4 * hh + c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(sPl + Swz(row, 4 * hh + c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      if (!__all_sync(0xFFFFFFFFu, dev::MbarWait(kv_full + b, static_cast<uint32_t>((j >> 1) & 1)))) {
        ok = false;
        continue;
      }
      {
        // V^T: thread = dim d (row), keys of half hh
        const int d = row, box = d >> 6, col = d & 63, cc = col >> 3;
        const uint8_t* vb = sKV + b * kTcStage + 2 * kHalfTile + box * kHalfTile + (col & 7) * 2 + 32 * hh * 128;
        // key k = 32 hh + 8 c + i sits in swizzled chunk cc ^ i of its row
        const uint8_t* vi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) vi[i] = vb + ((cc ^ i) << 4);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t lo16 = *reinterpret_cast<const uint16_t*>(vi[2 * i] + (8 * c + 2 * i) * 128);
            const uint32_t hi16 = *reinterpret_cast<const uint16_t*>(vi[2 * i + 1] + (8 * c + 2 * i + 1) * 128);
            w[i] = lo16 | (hi16 << 16);
          }
          *reinterpret_cast<uint4*>(sVt + Swz(d, 4 * hh + c)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      dev::FenceProxyAsync();  // P and Vt (generic writes) are read by the MMAs
      FenceBeforeSync();
      MbarArrive(&p_full);
    }
    if (!ok && lane == 0) atomicOr(a.err, 64u);
    if (ok && nsteps > 0 &&
        !__all_sync(0xFFFFFFFFu, dev::MbarWait(&o_done, static_cast<uint32_t>((nsteps - 1) & 1)))) {
      ok = false;
      if (lane == 0) atomicOr(a.err, 64u);
    }
    FenceAfterSync();
    // the row sum over both halves (a failed half skips the exchange: the
    // other half's wait on the named barrier is then the block's own)
    if (hh == 1) s_l[row] = l_run;
    asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
    const float l_row = hh == 0 ? l_run + s_l[row] : s_l[row] + 0.f;
    asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
    if (hh == 0) s_l[row] = l_row;
    asm volatile("bar.sync 1, %0;" ::"r"(kSoftThreads) : "memory");
    const float l_all = s_l[row];
    // ---- O / l (or the unnormalised partial of this key split): dims of half hh
    const int t = tok0 + tl;
    const int q_dim = a.n_heads * kD;
    const bool store = ok && t < a.n && nsteps > 0;  // (every split holds at least two key tiles)
    if (n_split > 1) {
      float* po = a.part_o + (static_cast<int64_t>(z) * a.n + t) * q_dim + qh * kD;
      if (store && hh == 0) {
        float* pml = a.part_ml + ((static_cast<int64_t>(z) * a.n + t) * a.n_heads + qh) * 2;
        *reinterpret_cast<float2*>(pml) = make_float2(m_run * 0.6931471805599453f, l_all);
      }
#pragma unroll 2
      for (int c0 = 64 * hh; c0 < 64 * hh + 64; c0 += 16) {
        uint32_t v[16];
        TmemLoad16(tmem + lrow + static_cast<uint32_t>(c0), v);
        if (store) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            *reinterpret_cast<float4*>(po + c0 + i) = make_float4(
                __uint_as_float(v[i]), __uint_as_float(v[i + 1]), __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
          }
        }
      }
    } else {
      float* out = a.out + static_cast<int64_t>(t) * q_dim + qh * kD;
      const float inv = 1.0f / l_all;
#pragma unroll 2
      for (int c0 = 64 * hh; c0 < 64 * hh + 64; c0 += 16) {
        uint32_t v[16];
        TmemLoad16(tmem + lrow + static_cast<uint32_t>(c0), v);
        if (store) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            *reinterpret_cast<float4*>(out + c0 + i) =
                make_float4(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv,
                            __uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv);
          }
        }
      }
    }
  }
  FenceBeforeSync();
  __syncthreads();
  if (warp == 0) {
    FenceAfterSync();
    TmemDealloc(tmem, 256u);
  }
}

// out[t][head] = sum_z O_z e^(m_z - M) / sum_z l_z e^(m_z - M), M = max_z m_z;
// one warp per (token, head), four dimensions per lane.  A split that saw no
// key of the row carries m = -inf, l = 0 and adds nothing.
__global__ void __launch_bounds__(256) FlashMergeKernel(const float* __restrict__ part_o,
                                                        const float* __restrict__ part_ml, float* __restrict__ out,
                                                        int n, int n_heads, int n_split) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp;  // t * n_heads + head
  if (row >= static_cast<int64_t>(n) * n_heads) return;
  const int64_t rows = static_cast<int64_t>(n) * n_heads;
  const int t = static_cast<int>(row / n_heads), hd = static_cast<int>(row - static_cast<int64_t>(t) * n_heads);
  const int64_t q_dim = static_cast<int64_t>(n_heads) * kD;
  float M = -INFINITY;
  for (int z = 0; z < n_split; ++z) M = fmaxf(M, part_ml[(z * rows + row) * 2]);
  float L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int z = 0; z < n_split; ++z) {
    const float2 ml = *reinterpret_cast<const float2*>(part_ml + (z * rows + row) * 2);
    if (ml.x == -INFINITY) continue;
    const float w = expf(ml.x - M);
    L += ml.y * w;
    const float4 v = *reinterpret_cast<const float4*>(part_o + z * static_cast<int64_t>(n) * q_dim + t * q_dim +
                                                      hd * kD + 4 * lane);
    acc.x += v.x * w;
    acc.y += v.y * w;
    acc.z += v.z * w;
    acc.w += v.w * w;
  }
  const float inv = 1.0f / L;
  *reinterpret_cast<float4*>(out + t * q_dim + hd * kD + 4 * lane) =
      make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

PFN_cuTensorMapEncodeTiled_v12000 Encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  RPGB_CHECK(fn != nullptr, "flash attention: cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// The KV cache of one layer, [n_kv][max_seq][128] fp16, as a 3-D tensor map
// with 64-dim x 64-position boxes and the 128-byte swizzle.
CUtensorMap CacheMap(const __half* base, int n_kv, int max_seq) {
  CUtensorMap m;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(max_seq),
                              static_cast<cuuint64_t>(n_kv)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(max_seq) * kD * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kKT), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = Encode()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RPGB_CHECK(r == CUDA_SUCCESS, "flash attention: tensor map encoding failed (%d)", static_cast<int>(r));
  return m;
}

using FlashFn = void (*)(const CUtensorMap, const CUtensorMap, const FlashArgs);

FlashFn PickFlash(int group) {
  switch (group) {
    case 1: return FlashTcKernel<1>;
    case 2: return FlashTcKernel<2>;
    case 4: return FlashTcKernel<4>;
    case 8: return FlashTcKernel<8>;
  }
  Throw("flash attention: group size %d is not built", group);
}

}  // namespace

void PrepareFlashKernels() {
  for (int g : {1, 2, 4, 8}) {
    RPGB_CUDA(cudaFuncSetAttribute(PickFlash(g), cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTcSmem)));
  }
}

bool FlashSupports(int group, int head_dim) { return head_dim == kD && (group == 1 || group == 2 || group == 4 || group == 8); }

size_t FlashSplitFloats(int n_heads, int n_kv, int num_sms) {
  // splitting happens only while query tiles x KV heads x splits <= num_sms,
  // so split x token rows are at most num_sms / n_kv query tiles of 128 / G tokens
  const int group = n_heads / n_kv;
  const size_t rows = static_cast<size_t>(num_sms / n_kv + 1) * (kRows / group);
  return rows * (static_cast<size_t>(n_heads) * kD + 2 * static_cast<size_t>(n_heads));
}

void LaunchFlashPrefill(const AttnParams& p, int n_queries, int64_t pos0, int num_sms, cudaStream_t s) {
  RPGB_CHECK(n_queries > 0 && p.n_kv > 0 && p.n_heads % p.n_kv == 0, "flash attention: bad shape");
  RPGB_CHECK(p.err != nullptr, "flash attention: no error word");
  const int G = p.n_heads / p.n_kv;
  const CUtensorMap mK = CacheMap(p.kc, p.n_kv, p.max_seq), mV = CacheMap(p.vc, p.n_kv, p.max_seq);
  FlashArgs a;
  a.q = p.q;
  a.q_stride = p.q_stride;
  a.out = p.out;
  a.n = n_queries;
  a.n_heads = p.n_heads;
  a.pos0 = pos0;
  a.scale = p.scale;
  a.err = p.err;
  const int tq = kRows / G;
  const int qtiles = (n_queries + tq - 1) / tq;
  // key splits while the grid would fill at most half the SMs, each split at
  // least two 64-key tiles of the longest query tile
  int n_split = 1;
  const int base = qtiles * p.n_kv;
  const size_t q_dim = static_cast<size_t>(p.n_heads) * kD;
  if (p.part != nullptr && 2 * base <= num_sms) {
    const int64_t tiles = (pos0 + n_queries + kKT - 1) / kKT;
    n_split = static_cast<int>(std::min<int64_t>({static_cast<int64_t>(num_sms / base), tiles / 2,
                                                  static_cast<int64_t>(kMaxFlashSplits)}));
    n_split = std::max(n_split, 1);
    RPGB_CHECK(static_cast<size_t>(n_split) * n_queries * (q_dim + 2 * p.n_heads) <=
                   FlashSplitFloats(p.n_heads, p.n_kv, num_sms),
               "flash attention: split scratch too small");
  }
  a.part_o = n_split > 1 ? p.part : nullptr;
  a.part_ml = n_split > 1 ? p.part + static_cast<size_t>(n_split) * n_queries * q_dim : nullptr;
  const dim3 grid(qtiles, p.n_kv, n_split);
  PickFlash(G)<<<grid, kTcWarps * 32, kTcSmem, s>>>(mK, mV, a);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
  if (n_split > 1) {
    const int64_t rows = static_cast<int64_t>(n_queries) * p.n_heads;
    FlashMergeKernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, s>>>(a.part_o, a.part_ml, p.out, n_queries,
                                                                          p.n_heads, n_split);
    RPGB_CUDA(cudaGetLastError());
    CountLaunches(1);
  }
}

}  // namespace rpgb
