// k_flash.cu -- prefill attention on the tensor cores (flash-attention style).
//
// Replaces AttentionFromCacheKernel for prompts (src/kernels_gpu.cu:737-823,
// GpuAttentionFromCache at 1038-1087): causal GQA over the fp16 KV cache,
// scale 1/sqrt(128), softmax with max subtraction, output = P V / sum P.
//
// One block of 8 warps per (tile of 128 / G query tokens, KV head h): its
// 128 rows are the (token, q head) pairs of the G q heads sharing h, so every
// K/V tile is read once per query tile instead of once per token.  K and V
// tiles of 64 positions arrive by 3-D TMA (128-byte swizzle) in two stages;
// each warp owns 16 rows and computes
//   S = Q K^T   and   O += P V
// with mma.sync m16n8k16 (fp16 in, fp32 accumulate), keeping S, the online
// softmax state and O in registers.  K and V are fp16 already (exact); Q and
// P are split into two fp16 terms (hi + lo), so scores and outputs keep about
// 22 significant bits (the reference computes them in FP32).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"

namespace rpgb {
namespace {

constexpr int kD = 128;
constexpr int kKT = 64;        // key positions per stage
constexpr int kWarps = 8;
constexpr int kRows = 16 * kWarps;  // (token, q head) rows per block
constexpr uint32_t kHalfTile = kKT * 64 * 2;  // 64 positions x 64 dims fp16 = 8 KB (one swizzled box)
constexpr uint32_t kStageBytes = 4 * kHalfTile;  // K dims 0-63, K dims 64-127, V dims 0-63, V dims 64-127
constexpr size_t kSmem = 2 * kStageBytes + 1024;

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

__device__ __forceinline__ void MmaF16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void LdMatrixX4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void LdMatrixX4T(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void TmaLoad3D(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(dev::SmemAddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(dev::SmemAddr(bar))
      : "memory");
}

// Address of the 16-byte chunk `chunk` (0..15 over the 128 dims) of position
// `row` (0..63) in a stage half written by TMA with the 128-byte swizzle.
__device__ __forceinline__ uint32_t SwzAddr(uint32_t half_base, int row, int chunk) {
  const int sub = chunk >> 3, c = chunk & 7;
  return half_base + static_cast<uint32_t>(sub) * kHalfTile + static_cast<uint32_t>(row * 128 + ((c ^ (row & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kWarps * 32, 1)
    FlashPrefillKernel(const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mV,
                       const FlashArgs a) {
  constexpr int kTQ = kRows / G;           // query tokens per block
  constexpr int kWarpsPerHead = kWarps / G;  // warps per q head (16 tokens each)
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[2];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  const int h = blockIdx.y;
  // the last query tiles see the most keys (causal): they are launched first,
  // so the short tiles fill the final wave
  const int tok0 = (gridDim.x - 1 - blockIdx.x) * kTQ;
  const int gq = warp / kWarpsPerHead;                // q head within the group
  const int wt0 = tok0 + (warp % kWarpsPerHead) * 16;  // first token of this warp's rows
  const int qh = h * G + gq;

  // keys 0 .. pos0 + last token of the block, in 64-key tiles; split z of
  // gridDim.z takes tiles [t_lo, t_lo + nsteps)
  const int64_t last_tok = (tok0 + kTQ < a.n ? tok0 + kTQ : a.n) - 1;
  const int64_t kend = a.pos0 + last_tok + 1;
  const int tiles = static_cast<int>((kend + kKT - 1) / kKT);
  const int n_split = static_cast<int>(gridDim.z), z = static_cast<int>(blockIdx.z);
  const int t_lo = static_cast<int>(static_cast<int64_t>(z) * tiles / n_split);
  const int nsteps = static_cast<int>(static_cast<int64_t>(z + 1) * tiles / n_split) - t_lo;

  if (tid == 0) {
    dev::MbarInit(full + 0, 1);
    dev::MbarInit(full + 1, 1);
    dev::MbarInitFence();
    for (int st = 0; st < 2 && st < nsteps; ++st) {
      uint8_t* b = smem + st * kStageBytes;
      const int y = (t_lo + st) * kKT;
      dev::MbarExpectTx(full + st, kStageBytes);
      TmaLoad3D(b, &mK, 0, y, h, full + st);
      TmaLoad3D(b + kHalfTile, &mK, 64, y, h, full + st);
      TmaLoad3D(b + 2 * kHalfTile, &mV, 0, y, h, full + st);
      TmaLoad3D(b + 3 * kHalfTile, &mV, 64, y, h, full + st);
    }
  }

  // ---- Q fragments (A operand): rows g4 and g4 + 8 of this warp, hi and lo
  uint32_t qa_hi[8][4], qa_lo[8][4];
  {
    const int ta = wt0 + g4, tb = wt0 + g4 + 8;
    const float* qa = a.q + static_cast<int64_t>(ta < a.n ? ta : 0) * a.q_stride + qh * kD;
    const float* qb = a.q + static_cast<int64_t>(tb < a.n ? tb : 0) * a.q_stride + qh * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const float2 x0 = *reinterpret_cast<const float2*>(qa + 16 * ks + 2 * t4);
      const float2 x1 = *reinterpret_cast<const float2*>(qb + 16 * ks + 2 * t4);
      const float2 x2 = *reinterpret_cast<const float2*>(qa + 16 * ks + 8 + 2 * t4);
      const float2 x3 = *reinterpret_cast<const float2*>(qb + 16 * ks + 8 + 2 * t4);
      SplitPair(x0.x * a.scale, x0.y * a.scale, qa_hi[ks][0], qa_lo[ks][0]);
      SplitPair(x1.x * a.scale, x1.y * a.scale, qa_hi[ks][1], qa_lo[ks][1]);
      SplitPair(x2.x * a.scale, x2.y * a.scale, qa_hi[ks][2], qa_lo[ks][2]);
      SplitPair(x3.x * a.scale, x3.y * a.scale, qa_hi[ks][3], qa_lo[ks][3]);
    }
  }
  const int64_t pa = a.pos0 + wt0 + g4, pb = pa + 8;  // positions of the thread's two rows

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  __syncthreads();

  bool failed = false;
  for (int st = 0; st < nsteps; ++st) {
    const int stage = st & 1;
    const bool ok = dev::MbarWait(full + stage, static_cast<uint32_t>((st >> 1) & 1));
    if (!ok) {
      failed = true;
      if (tid == 0) atomicOr(a.err, 64u);
    }
    const uint32_t kb = dev::SmemAddr(smem + stage * kStageBytes);
    const uint32_t vb = kb + 2 * kHalfTile;
    const int64_t key0 = static_cast<int64_t>(t_lo + st) * kKT;
    // this warp's rows see no key of this stage: skip the math (stays in step for the barrier)
    const bool any = key0 <= a.pos0 + wt0 + 15;
    if (any) {
      // ---- S = Q K^T for 64 keys: 8 n-tiles of 8 keys
      float s[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          // matrices: keys 16np + {0..7, 0..7, 8..15, 8..15}, dims 16ks + {0..7, 8..15, 0..7, 8..15}
          const int mi = lane >> 3, row = 16 * np + ((mi >> 1) << 3) + (lane & 7);
          uint32_t b0, b1, b2, b3;
          LdMatrixX4(SwzAddr(kb, row, 2 * ks + (mi & 1)), b0, b1, b2, b3);
          MmaF16(s[2 * np], qa_hi[ks], b0, b1);
          MmaF16(s[2 * np], qa_lo[ks], b0, b1);
          MmaF16(s[2 * np + 1], qa_hi[ks], b2, b3);
          MmaF16(s[2 * np + 1], qa_lo[ks], b2, b3);
        }
      }
      // ---- causal mask and online softmax (rows g4: s[.][0..1], g4 + 8: s[.][2..3])
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int64_t k = key0 + 8 * nt + 2 * t4;
        if (k > pa) s[nt][0] = -INFINITY;
        if (k + 1 > pa) s[nt][1] = -INFINITY;
        if (k > pb) s[nt][2] = -INFINITY;
        if (k + 1 > pb) s[nt][3] = -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, 2));
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      const float al0 = m0 == -INFINITY ? 0.f : expf(m0 - n0);
      const float al1 = m1 == -INFINITY ? 0.f : expf(m1 - n1);
      m0 = n0;
      m1 = n1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][0] = s[nt][0] == -INFINITY ? 0.f : expf(s[nt][0] - n0);
        s[nt][1] = s[nt][1] == -INFINITY ? 0.f : expf(s[nt][1] - n0);
        s[nt][2] = s[nt][2] == -INFINITY ? 0.f : expf(s[nt][2] - n1);
        s[nt][3] = s[nt][3] == -INFINITY ? 0.f : expf(s[nt][3] - n1);
        ps0 += s[nt][0] + s[nt][1];
        ps1 += s[nt][2] + s[nt][3];
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al0;
        o[i][2] *= al1;
        o[i][3] *= al1;
      }
      // ---- O += P V: P (A operand, keys 16 kk .. +15) from the S tiles 2 kk, 2 kk + 1
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ph[4], pl[4];
        SplitPair(s[2 * kk][0], s[2 * kk][1], ph[0], pl[0]);
        SplitPair(s[2 * kk][2], s[2 * kk][3], ph[1], pl[1]);
        SplitPair(s[2 * kk + 1][0], s[2 * kk + 1][1], ph[2], pl[2]);
        SplitPair(s[2 * kk + 1][2], s[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          // matrices (transposed): keys 16kk + {0..7, 8..15, 0..7, 8..15}, dims 16dp + {0..7, 0..7, 8..15, 8..15}
          const int mi = lane >> 3, row = 16 * kk + ((mi & 1) << 3) + (lane & 7);
          uint32_t b0, b1, b2, b3;
          LdMatrixX4T(SwzAddr(vb, row, 2 * dp + (mi >> 1)), b0, b1, b2, b3);
          MmaF16(o[2 * dp], ph, b0, b1);
          MmaF16(o[2 * dp], pl, b0, b1);
          MmaF16(o[2 * dp + 1], ph, b2, b3);
          MmaF16(o[2 * dp + 1], pl, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && st + 2 < nsteps) {
      dev::FenceProxyAsync();
      uint8_t* b = smem + stage * kStageBytes;
      const int y = (t_lo + st + 2) * kKT;
      dev::MbarExpectTx(full + stage, kStageBytes);
      TmaLoad3D(b, &mK, 0, y, h, full + stage);
      TmaLoad3D(b + kHalfTile, &mK, 64, y, h, full + stage);
      TmaLoad3D(b + 2 * kHalfTile, &mV, 0, y, h, full + stage);
      TmaLoad3D(b + 3 * kHalfTile, &mV, 64, y, h, full + stage);
    }
  }

  if (failed && tid == 0) {  // copies that may still be landing in this block's shared memory
    for (int st = nsteps - 2 > 0 ? nsteps - 2 : 0; st < nsteps; ++st) {
      dev::MbarWait(full + (st & 1), static_cast<uint32_t>((st >> 1) & 1));
    }
  }

  // ---- O / l for the thread's rows
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
  const int ta = wt0 + g4, tb = ta + 8;
  const int q_dim = a.n_heads * kD;
  if (n_split > 1) {  // unnormalised partials; FlashMergeKernel combines the splits
    float* po = a.part_o + static_cast<int64_t>(z) * a.n * q_dim + qh * kD;
    float* pml = a.part_ml + (static_cast<int64_t>(z) * a.n * a.n_heads + qh) * 2;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      const int d = 8 * dt + 2 * t4;
      if (ta < a.n) *reinterpret_cast<float2*>(po + static_cast<int64_t>(ta) * q_dim + d) = make_float2(o[dt][0], o[dt][1]);
      if (tb < a.n) *reinterpret_cast<float2*>(po + static_cast<int64_t>(tb) * q_dim + d) = make_float2(o[dt][2], o[dt][3]);
    }
    if (t4 == 0) {
      if (ta < a.n) *reinterpret_cast<float2*>(pml + static_cast<int64_t>(ta) * a.n_heads * 2) = make_float2(m0, l0);
      if (tb < a.n) *reinterpret_cast<float2*>(pml + static_cast<int64_t>(tb) * a.n_heads * 2) = make_float2(m1, l1);
    }
    return;
  }
  const float i0 = 1.0f / l0, i1 = 1.0f / l1;
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    const int d = 8 * dt + 2 * t4;
    if (ta < a.n) {
      *reinterpret_cast<float2*>(a.out + static_cast<int64_t>(ta) * q_dim + qh * kD + d) =
          make_float2(o[dt][0] * i0, o[dt][1] * i0);
    }
    if (tb < a.n) {
      *reinterpret_cast<float2*>(a.out + static_cast<int64_t>(tb) * q_dim + qh * kD + d) =
          make_float2(o[dt][2] * i1, o[dt][3] * i1);
    }
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
    case 1: return FlashPrefillKernel<1>;
    case 2: return FlashPrefillKernel<2>;
    case 4: return FlashPrefillKernel<4>;
    case 8: return FlashPrefillKernel<8>;
  }
  Throw("flash attention: group size %d is not built", group);
}

}  // namespace

void PrepareFlashKernels() {
  for (int g : {1, 2, 4, 8}) {
    RPGB_CUDA(cudaFuncSetAttribute(PickFlash(g), cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem)));
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
  PickFlash(G)<<<grid, kWarps * 32, kSmem, s>>>(mK, mV, a);
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
