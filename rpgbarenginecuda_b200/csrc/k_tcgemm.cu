// k_tcgemm.cu -- prefill GEMM on the 5th-generation tensor cores (tcgen05).
//
// out[t, r] = sum_k X[t, k] * W[r, k] for a Q4_K / Q6_K weight matrix W, the
// prompt path of MatMulQ4KKernel / MatMulQ6KKernel with TILE = 8
// (src/kernels_gpu.cu:325-494) as used by GpuForwardFull.
//
// Precision.  The reference dequantises every weight in FP32 and sums FP32
// products.  Here both operands are split into two fp16 terms,
//   W = Wh + Wl,  X = Xh + Xl   (Wh = fp16(W), Wl = fp16(W - Wh), same for X)
// and the tensor cores accumulate Wh*Xh + Wh*Xl + Wl*Xh in FP32 (TMEM): about
// 22 significant bits of each operand survive, so results differ from the
// FP32 path at the 1e-6 relative level (the dropped Wl*Xl term is ~2^-22).
//
// (Dropping the Wl*Xh term -- weights rounded to fp16 -- was measured: two
// MMAs instead of three, but 1.8e-3 of full scale on the 1.7B model's logits
// after a 2811-token prefill, over the 1e-3 bound.)
//
// Pipeline (persistent: one block of 6 warps per SM walks 128 x 128 output
// tiles, token tiles fastest):
//  * DequantSplitKernel writes a matrix as Wh / Wl (row-major, fp16) with the
//    bit-exact per-element dequant formulas -- once at model load into the
//    model's own copy (Model::Load), or per call into the call's scratch for
//    a matrix without one; SplitKernel writes Xh / Xl (unless the producer
//    of X already wrote them: the prefill's RMSNorm does, and so does the
//    SiLU epilogue for ffn_down when given out_h / out_l);
//  * a GEMM with few output tiles, or whose whole tiles would leave a short
//    last wave, splits its K range (blockIdx-free: the work items carry the
//    split) and SplitReduceKernel adds the partials in split order;
//  * warp 0 streams 64-column k-slices of Wh, Wl, Xh, Xl into three
//    shared-memory stages with 2-D TMA tensor copies (128-byte swizzle);
//  * warp 1 issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N 128, K 16;
//    12 per k-slice) into one of two 128-column TMEM accumulators (tiles
//    alternate) and frees each stage with tcgen05.commit on its "empty"
//    mbarrier;
//  * warps 2-5 read their 32 TMEM lanes (= 32 weight rows) with tcgen05.ld
//    and apply the epilogue (store, residual add, or SiLU(gate) * up on
//    interleaved row pairs) with coalesced stores, while the MMAs of the
//    next tile run into the other accumulator.
// Every mbarrier wait is bounded; a wait that gives up sets *err, and the
// block still waits for its own copies and MMAs and frees its TMEM.
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

using namespace tc;

constexpr int kBM = 128;     // weight rows per tile (MMA M)
constexpr int kBN = 128;     // tokens per tile (MMA N)
constexpr int kBK = 64;      // k per stage: 64 fp16 = one 128-byte swizzle row
constexpr int kStages = 3;
constexpr int kThreads = 192;     // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kEpiThreads = 128;
constexpr uint32_t kTileBytes = kBM * kBK * 2;  // 16 KB, same for the B tiles (kBN == kBM)
constexpr uint32_t kStageBytes = 4 * kTileBytes;
constexpr size_t kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack

// ------------------------------------------------------------------ operand preparation

__device__ __forceinline__ void SplitStore8(const float (&v)[8], __half* hi, __half* lo) {
  __align__(16) __half h[8], l[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i] = __float2half_rn(v[i]);
    l[i] = __float2half_rn(v[i] - __half2float(h[i]));
  }
  *reinterpret_cast<uint4*>(hi) = *reinterpret_cast<const uint4*>(h);
  *reinterpret_cast<uint4*>(lo) = *reinterpret_cast<const uint4*>(l);
}

// W (repacked Q4_K / Q6_K) -> Wh, Wl [rows][K].  One thread per 8 consecutive
// columns of a row; the values are those of DeqQ4K / DeqQ6K (separately
// rounded products, as src/quant.cc).
__global__ void __launch_bounds__(256) DequantSplitKernel(const DevMat w, __half* __restrict__ hi,
                                                          __half* __restrict__ lo) {
  const int K = w.cols;
  const int64_t items = static_cast<int64_t>(w.rows) * (K / 8);
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = it / (K / 8);
    const int col = static_cast<int>(it - row * (K / 8)) * 8;
    const int b = col >> 8, kb = (col & 255) >> 5, lk = col & 31;
    const uint8_t* grp = dev::GroupPtr(w, row, b);
    const int r16 = static_cast<int>(row & 15), g = r16 & 7, rs = r16 >> 3;
    float v[8];
    if (w.type == 13u || w.type == 8u) {  // one byte per weight: element by element
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = dev::DeqElem(w, row, col + i);
    } else if (w.type == 12u) {
      const uint4 hd = *reinterpret_cast<const uint4*>(grp + 2048 + 16 * r16);
      int sc, m;
      dev::Q4kScaleMin(hd.y, hd.z, hd.w, kb, &sc, &m);
      const float d1 = __fmul_rn(dev::Half(hd.x & 0xFFFFu), static_cast<float>(sc));
      const float m1 = __fmul_rn(dev::Half(hd.x >> 16), static_cast<float>(m));
      const int c = kb >> 1, h = lk >> 4, t0 = (lk >> 2) & 3;
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(grp + (c * 32 + 4 * g + t0) * 16 + (2 * h + rs) * 4);
      const uint32_t qw[2] = {wp[0], wp[4]};
      const int sh = (kb & 1) * 4;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = static_cast<int>((qw[i >> 2] >> (8 * (i & 3) + sh)) & 15u);
        v[i] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
      }
    } else {
      const int j16 = 2 * kb + (lk >> 4);
      const int8_t sc = static_cast<int8_t>(grp[3072 + 16 * r16 + j16]);
      const float dd = dev::Half(*reinterpret_cast<const uint16_t*>(grp + 3328 + 2 * (2 * g + rs)));
      const float ds = __fmul_rn(dd, static_cast<float>(sc));
      const int c = j16 >> 2, h = j16 & 1, hb = (j16 >> 1) & 1, m = 2 * c + h;
      const int t0 = (lk & 15) >> 2;
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const uint32_t* wq =
            reinterpret_cast<const uint32_t*>(grp + ((m >> 2) * 32 + 4 * g + t0 + tt) * 48 + (m & 3) * 12);
        const uint32_t X = wq[0], Y = wq[1], Z = wq[2];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int q;
          if (hb == 0) {
            q = static_cast<int>(((rs == 0 ? X : Y) >> (8 * e)) & 63u);
          } else if (rs == 0) {
            q = static_cast<int>((Z >> (8 * e)) & 63u);
          } else {
            q = static_cast<int>(((X >> (8 * e + 6)) & 3u) | (((Y >> (8 * e + 6)) & 3u) << 2) |
                                 (((Z >> (8 * e + 6)) & 3u) << 4));
          }
          v[4 * tt + e] = __fmul_rn(ds, static_cast<float>(q - 32));
        }
      }
    }
    SplitStore8(v, hi + row * K + col, lo + row * K + col);
  }
}

// X [n][ldx] (first K columns) -> Xh, Xl [n][K].
__global__ void __launch_bounds__(256) SplitKernel(const float* __restrict__ X, int n, int ldx, int K,
                                                   __half* __restrict__ hi, __half* __restrict__ lo) {
  const int64_t items = static_cast<int64_t>(n) * (K / 8);
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = it / (K / 8);
    const int col = static_cast<int>(it - t * (K / 8)) * 8;
    const float4 a = *reinterpret_cast<const float4*>(X + t * ldx + col);
    const float4 b = *reinterpret_cast<const float4*>(X + t * ldx + col + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    SplitStore8(v, hi + t * K + col, lo + t * K + col);
  }
}

// ------------------------------------------------------------------ tcgen05 / TMA primitives

__device__ __forceinline__ void TmaLoad2D(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dev::SmemAddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(dev::SmemAddr(bar))
      : "memory");
}

// ------------------------------------------------------------------ the GEMM

struct TcArgs {
  int32_t n_tok, K;
  float* out;
  int32_t ldo, out_off;
  const float* resid;
  int32_t ldr;
  unsigned* err;
  // split-K (gridDim.z > 1): block z sums k-slices [z nk / S, (z + 1) nk / S)
  // and stores its raw tile into part[z][n_tok][rows]; SplitReduceKernel
  // adds the S partials in order and applies the epilogue
  float* part;
  int32_t rows;
  int32_t splits;
  // SiLU epilogue: fp16 hi/lo terms of the output instead of out (or null)
  __half* oh;
  __half* ol;
};

__device__ __forceinline__ void StoreSilu(const TcArgs& a, int64_t idx, float y) {
  if (a.oh != nullptr) {
    const __half h = __float2half_rn(y);
    a.oh[idx] = h;
    a.ol[idx] = __float2half_rn(y - __half2float(h));
  } else {
    a.out[idx] = y;
  }
}

// Work item it -> its output tile and K range (token tiles fastest, so the
// blocks running at one time share weight row tiles in L2).
struct TcItem {
  int tok0, row0, z, kb0, nk;
};
__device__ __forceinline__ TcItem ItemOf(const TcArgs& a, int it, int tok_tiles, int nk_all) {
  TcItem w;
  const int S = a.splits;
  w.z = it % S;
  const int tile = it / S;
  w.tok0 = (tile % tok_tiles) * kBN;
  w.row0 = (tile / tok_tiles) * kBM;
  w.kb0 = w.z * nk_all / S;
  w.nk = (w.z + 1) * nk_all / S - w.kb0;
  return w;
}

// Persistent, warp-specialised: warp 0 streams operands, warp 1 issues the
// MMAs, warps 2-5 run the epilogue.  Two 128-column TMEM accumulators let
// the epilogue of one tile overlap the main loop of the next.
template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    TcGemmKernel(const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                 const __grid_constant__ CUtensorMap mXh, const __grid_constant__ CUtensorMap mXl, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], accf[2], acce[2];
  __shared__ uint32_t s_tmem;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tok_tiles = (a.n_tok + kBN - 1) / kBN;
  const int items = tok_tiles * (a.rows / kBM) * a.splits;
  const int nk_all = a.K / kBK;

  if (warp == 0) {  // two accumulators: 2 x 128 TMEM columns x 128 lanes (fp32)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dev::SmemAddr(&s_tmem)),
                 "r"(256u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      dev::MbarInit(full + s, 1);
      dev::MbarInit(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      dev::MbarInit(accf + b, 1);
      dev::MbarInit(acce + b, kEpiThreads);
    }
    dev::MbarInitFence();
  }
  FenceBeforeSync();
  __syncthreads();
  FenceAfterSync();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: k-slices of Wh, Wl, Xh, Xl into the stages, item after item
      uint32_t q = 0;  // k-slices issued by this block
      bool bad = false;
      for (int it = blockIdx.x; it < items && !bad; it += gridDim.x) {
        const TcItem w = ItemOf(a, it, tok_tiles, nk_all);
        for (int kb = 0; kb < w.nk; ++kb, ++q) {
          const int s = static_cast<int>(q % kStages);
          if (q >= kStages && !dev::MbarWait(empty + s, (q / kStages - 1u) & 1u)) {
            atomicOr(a.err, 16u);
            bad = true;
            break;
          }
          uint8_t* st = smem + s * kStageBytes;
          const int kx = (w.kb0 + kb) * kBK;
          dev::MbarExpectTx(full + s, kStageBytes);
          TmaLoad2D(st, &mWh, kx, w.row0, full + s);
          TmaLoad2D(st + kTileBytes, &mWl, kx, w.row0, full + s);
          TmaLoad2D(st + 2 * kTileBytes, &mXh, kx, w.tok0, full + s);
          TmaLoad2D(st + 3 * kTileBytes, &mXl, kx, w.tok0, full + s);
        }
      }
      // the copies of the last stages land before the block may exit
      for (uint32_t k = q > kStages ? q - kStages : 0u; k < q; ++k) {
        dev::MbarWait(full + k % kStages, (k / kStages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      constexpr uint32_t idesc = InstrDesc(kBM, kBN);
      uint32_t q = 0, j = 0;
      bool bad = false;
      for (int it = blockIdx.x; it < items && !bad; it += gridDim.x, ++j) {
        const TcItem w = ItemOf(a, it, tok_tiles, nk_all);
        const uint32_t ab = j & 1u, use = j >> 1;
        if (use >= 1 && !dev::MbarWait(acce + ab, (use - 1u) & 1u)) {  // the epilogue has read this accumulator
          atomicOr(a.err, 16u);
          break;
        }
        FenceAfterSync();
        const uint32_t tacc = tmem + ab * 128u;
        for (int kb = 0; kb < w.nk; ++kb, ++q) {
          const int s = static_cast<int>(q % kStages);
          if (!dev::MbarWait(full + s, (q / kStages) & 1u)) {
            atomicOr(a.err, 16u);
            bad = true;
            break;
          }
          FenceAfterSync();
          const uint8_t* st = smem + s * kStageBytes;
          const uint64_t dWh = DescSw128(st), dWl = DescSw128(st + kTileBytes);
          const uint64_t dXh = DescSw128(st + 2 * kTileBytes), dXl = DescSw128(st + 3 * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t adv = static_cast<uint64_t>(kk * 32 >> 4);  // 16 fp16 = 32 bytes along K
            Mma(tacc, dWh + adv, dXh + adv, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            Mma(tacc, dWh + adv, dXl + adv, idesc, 1u);
            Mma(tacc, dWl + adv, dXh + adv, idesc, 1u);
          }
          MmaCommit(empty + s);  // the stage is free once these MMAs have read it
        }
        if (bad) break;
        MmaCommit(accf + ab);  // the accumulator is complete once every issued MMA is
      }
    }
  } else {
    // ---- epilogue: warp w reads TMEM lanes (weight rows) 32 (w % 4) .. + 31
    const int quarter = warp & 3;
    uint32_t j = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++j) {
      const TcItem w = ItemOf(a, it, tok_tiles, nk_all);
      const uint32_t ab = j & 1u, use = j >> 1;
      if (!dev::MbarWait(accf + ab, use & 1u)) {
        if (lane == 0) atomicOr(a.err, 32u);
        break;
      }
      FenceAfterSync();
      const int r = w.row0 + 32 * quarter + lane;
      for (int c0 = 0; c0 < kBN; c0 += 16) {
        uint32_t v[16];
        TmemLoad16(tmem + ab * 128u + (static_cast<uint32_t>(32 * quarter) << 16) + static_cast<uint32_t>(c0), v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int t = w.tok0 + c0 + jj;
          const float acc = __uint_as_float(v[jj]);
          if (a.splits > 1) {
            if (t < a.n_tok) a.part[(static_cast<int64_t>(w.z) * a.n_tok + t) * a.rows + r] = acc;
          } else if (EPI == static_cast<int>(Epi::kSilu)) {
            // rows 2i (gate) and 2i+1 (up) sit in neighbouring lanes
            const float u = __shfl_xor_sync(0xFFFFFFFFu, acc, 1);
            if (t < a.n_tok && (lane & 1) == 0) {
              StoreSilu(a, static_cast<int64_t>(t) * a.ldo + (r >> 1), (acc / (1.0f + expf(-acc))) * u);
            }
          } else if (t < a.n_tok) {
            if (EPI == static_cast<int>(Epi::kResid)) {
              float* o = a.out + static_cast<int64_t>(t) * a.ldo + r;
              *o = a.resid[static_cast<int64_t>(t) * a.ldr + r] + acc;
            } else {
              a.out[static_cast<int64_t>(t) * a.ldo + a.out_off + r] = acc;
            }
          }
        }
      }
      FenceBeforeSync();
      MbarArrive(acce + ab);  // this accumulator may be overwritten
    }
  }
  FenceBeforeSync();
  __syncthreads();
  if (warp == 0) {
    FenceAfterSync();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256u) : "memory");
  }
}

// Sum of the split-K partials in split order, then the GEMM's epilogue.
template <int EPI>
// With vec4 (16-byte aligned output, residual and offsets) the store and
// residual epilogues move four consecutive rows per thread.
__global__ void __launch_bounds__(256) SplitReduceKernel(const TcArgs a, int splits, bool vec4) {
  if (EPI != static_cast<int>(Epi::kSilu) && vec4) {
    const int64_t per4 = a.rows / 4;
    const int64_t items = static_cast<int64_t>(a.n_tok) * per4;
    const int64_t plane = static_cast<int64_t>(a.n_tok) * a.rows;
    for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
         it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t t = it / per4, i = (it - t * per4) * 4;
      float4 v = *reinterpret_cast<const float4*>(a.part + t * a.rows + i);
      for (int z = 1; z < splits; ++z) {
        const float4 w = *reinterpret_cast<const float4*>(a.part + z * plane + t * a.rows + i);
        v.x += w.x;
        v.y += w.y;
        v.z += w.z;
        v.w += w.w;
      }
      if (EPI == static_cast<int>(Epi::kResid)) {
        const float4 r = *reinterpret_cast<const float4*>(a.resid + t * a.ldr + i);
        *reinterpret_cast<float4*>(a.out + t * a.ldo + i) = make_float4(r.x + v.x, r.y + v.y, r.z + v.z, r.w + v.w);
      } else {
        *reinterpret_cast<float4*>(a.out + t * a.ldo + a.out_off + i) = v;
      }
    }
    return;
  }
  const int64_t per = EPI == static_cast<int>(Epi::kSilu) ? a.rows / 2 : a.rows;
  const int64_t items = static_cast<int64_t>(a.n_tok) * per;
  const int64_t plane = static_cast<int64_t>(a.n_tok) * a.rows;
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = it / per, i = it - t * per;
    if (EPI == static_cast<int>(Epi::kSilu)) {
      float g = 0.f, u = 0.f;
      for (int z = 0; z < splits; ++z) {
        const float2 gu = *reinterpret_cast<const float2*>(a.part + z * plane + t * a.rows + 2 * i);
        g += gu.x;
        u += gu.y;
      }
      StoreSilu(a, t * a.ldo + i, (g / (1.0f + expf(-g))) * u);
    } else {
      float v = 0.f;
      for (int z = 0; z < splits; ++z) v += a.part[z * plane + t * a.rows + i];
      if (EPI == static_cast<int>(Epi::kResid)) {
        a.out[t * a.ldo + i] = a.resid[t * a.ldr + i] + v;
      } else {
        a.out[t * a.ldo + a.out_off + i] = v;
      }
    }
  }
}

// ------------------------------------------------------------------ host side

// SMs of the current device (one persistent GEMM block per SM).
int DeviceSms() {
  int dev = 0, n = 0;
  RPGB_CUDA(cudaGetDevice(&dev));
  RPGB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 EncodeFn() {
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
  RPGB_CHECK(fn != nullptr, "tcgen05 gemm: cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Row-major fp16 [rows][K] as a 2-D tensor map with 64 x 128 boxes, 128-byte swizzle.
CUtensorMap MapOf(const __half* base, int64_t rows, int K) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(kBM)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = EncodeFn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides,
                                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RPGB_CHECK(r == CUDA_SUCCESS, "tcgen05 gemm: tensor map encoding failed (%d)", static_cast<int>(r));
  return m;
}

using TcFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const TcArgs);

TcFn PickTc(Epi epi) {
  switch (epi) {
    case Epi::kStore: return TcGemmKernel<0>;
    case Epi::kResid: return TcGemmKernel<1>;
    case Epi::kSilu: return TcGemmKernel<2>;
    default: Throw("tcgen05 gemm: unsupported epilogue");
  }
}

}  // namespace

void PrepareTcGemmKernels() {
  for (Epi e : {Epi::kStore, Epi::kResid, Epi::kSilu}) {
    RPGB_CUDA(cudaFuncSetAttribute(PickTc(e), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(kSmemBytes)));
  }
}

size_t TcGemmScratchHalves(int64_t rows, int64_t n_tok, int K, bool has_wh) {
  return (has_wh ? 0 : 2 * static_cast<size_t>(rows) * K) + 2 * static_cast<size_t>(n_tok) * K;
}

int TcGemmSplits(int64_t rows, int64_t n_tok, int K, int num_sms, size_t part_floats) {
  const int64_t tiles = (rows / kBM) * ((n_tok + kBN - 1) / kBN);
  const int nk = K / kBK;
  if (num_sms <= 0 || nk < 8) return 1;
  if (tiles * 2 > num_sms) {
    // many tiles: split in two when the last wave of whole tiles would be
    // short (two waves and a fifth of whole tiles take three tile times,
    // five waves of half tiles two and a half), if the partials fit
    const int64_t w1 = (tiles + num_sms - 1) / num_sms, w2 = (2 * tiles + num_sms - 1) / num_sms;
    const bool fits = static_cast<size_t>(2 * rows * n_tok) <= part_floats;
    return fits && nk >= 16 && 20 * w2 <= 17 * 2 * w1 ? 2 : 1;
  }
  // enough splits to fill the SMs, at least four k-slices each, and room
  // for the partial tiles
  int64_t sp = std::min<int64_t>(num_sms / tiles, nk / 4);
  const int64_t plane = rows * n_tok;
  if (plane > 0) sp = std::min<int64_t>(sp, static_cast<int64_t>(part_floats / static_cast<size_t>(plane)));
  return sp >= 2 ? static_cast<int>(sp) : 1;
}

size_t TcGemmPartFloats(int num_sms) { return static_cast<size_t>(num_sms) * kBM * kBN; }

void LaunchDequantSplit(const DevMat& w, __half* hi, __half* lo, cudaStream_t s) {
  const int64_t items = static_cast<int64_t>(w.rows) * (w.cols / 8);
  const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 148 * 16));
  DequantSplitKernel<<<blocks, 256, 0, s>>>(w, hi, lo);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

void LaunchTcGemm(const GemmParams& p, Epi epi, __half* scratch, size_t scratch_halves, cudaStream_t s) {
  const DevMat& w = p.w;
  const int K = w.cols;
  RPGB_CHECK(w.rows % kBM == 0, "tcgen05 gemm: rows %d not a multiple of %d", w.rows, kBM);
  RPGB_CHECK(K % 256 == 0, "tcgen05 gemm: cols %d not a multiple of 256", K);
  RPGB_CHECK(p.n_tok > 0 && p.ldx % 4 == 0, "tcgen05 gemm: bad activations");
  RPGB_CHECK(p.err != nullptr, "tcgen05 gemm: no error word");
  RPGB_CHECK((w.wh != nullptr && w.wl != nullptr) || w.q != nullptr, "tcgen05 gemm: matrix without weights");
  const bool has_wh = w.wh != nullptr && w.wl != nullptr;
  const size_t need = TcGemmScratchHalves(w.rows, p.n_tok, K, has_wh);
  RPGB_CHECK(scratch != nullptr && scratch_halves >= need, "tcgen05 gemm: scratch of %zu halves < %zu",
             scratch_halves, need);
  const __half* wh = w.wh;
  const __half* wl = w.wl;
  __half* xh = scratch;
  if (!has_wh) {
    LaunchDequantSplit(w, scratch, scratch + static_cast<size_t>(w.rows) * K, s);
    wh = scratch;
    wl = scratch + static_cast<size_t>(w.rows) * K;
    xh = scratch + 2 * static_cast<size_t>(w.rows) * K;
  }
  __half* xl = xh + static_cast<size_t>(p.n_tok) * K;
  if (p.xh != nullptr) {  // split by the kernel that produced the activations
    RPGB_CHECK(p.xl != nullptr, "tcgen05 gemm: activation terms incomplete");
    xh = const_cast<__half*>(p.xh);
    xl = const_cast<__half*>(p.xl);
  } else {
    const int64_t items = static_cast<int64_t>(p.n_tok) * (K / 8);
    const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 148 * 16));
    SplitKernel<<<blocks, 256, 0, s>>>(p.X, p.n_tok, p.ldx, K, xh, xl);
    RPGB_CUDA(cudaGetLastError());
  }
  const CUtensorMap mWh = MapOf(wh, w.rows, K), mWl = MapOf(wl, w.rows, K);
  const CUtensorMap mXh = MapOf(xh, p.n_tok, K), mXl = MapOf(xl, p.n_tok, K);
  TcArgs a;
  a.n_tok = p.n_tok;
  a.K = K;
  a.out = p.out;
  a.ldo = p.ldo;
  a.out_off = p.out_off;
  a.resid = p.resid;
  a.ldr = p.ldr;
  a.err = p.err;
  a.part = p.part;
  a.rows = w.rows;
  RPGB_CHECK((p.out_h == nullptr) == (p.out_l == nullptr) && (p.out_h == nullptr || epi == Epi::kSilu),
             "tcgen05 gemm: fp16 output terms are for the SiLU epilogue");
  a.oh = p.out_h;
  a.ol = p.out_l;
  const int num_sms = p.num_sms > 0 ? p.num_sms : DeviceSms();
  const int splits = TcGemmSplits(w.rows, p.n_tok, K, num_sms, p.part_floats);
  a.splits = splits;
  const int64_t items = static_cast<int64_t>((p.n_tok + kBN - 1) / kBN) * (w.rows / kBM) * splits;
  RPGB_CHECK(items < (static_cast<int64_t>(1) << 30), "tcgen05 gemm: too many tiles");
  const int grid = static_cast<int>(std::min<int64_t>(items, num_sms));
  PickTc(epi)<<<grid, kThreads, kSmemBytes, s>>>(mWh, mWl, mXh, mXl, a);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(2);
  if (splits > 1) {
    const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    const bool vec4 = epi != Epi::kSilu && a.ldo % 4 == 0 && a.out_off % 4 == 0 && al16(a.out) && al16(a.part) &&
                      (epi != Epi::kResid || (a.ldr % 4 == 0 && al16(a.resid)));
    const int64_t items = static_cast<int64_t>(p.n_tok) * w.rows / (vec4 ? 4 : 1);
    const int blocks = static_cast<int>(std::min<int64_t>((items + 255) / 256, 148 * 8));
    switch (epi) {
      case Epi::kStore: SplitReduceKernel<0><<<blocks, 256, 0, s>>>(a, splits, vec4); break;
      case Epi::kResid: SplitReduceKernel<1><<<blocks, 256, 0, s>>>(a, splits, vec4); break;
      case Epi::kSilu: SplitReduceKernel<2><<<blocks, 256, 0, s>>>(a, splits, false); break;
      default: Throw("tcgen05 gemm: unsupported epilogue");
    }
    RPGB_CUDA(cudaGetLastError());
    CountLaunches(1);
  }
}

}  // namespace rpgb
