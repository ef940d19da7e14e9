// k_gemm.cu -- prefill GEMM out[t, r] = sum_k X[t, k] * W[r, k], W Q4_K / Q6_K.
//
// Replaces the TILE = 8 path of MatMulQ4KKernel / MatMulQ6KKernel
// (src/kernels_gpu.cu:325-494) used by GpuForwardFull for prompts.  This is
// the FP32 SIMT tile (64 rows x 64 tokens x 32 k, 4x4 outputs per thread);
// every weight is dequantised with the reference's per-element formula, so
// results differ from the reference only by FP32 summation order.
#include "common.h"
#include "kernels.cuh"
#include "kernels.h"

namespace rpgb {
namespace {

constexpr int BM = 64, BN = 64, BK = 32;

template <int EPI>
__global__ void __launch_bounds__(256) GemmKernel(const GemmParams p) {
  __shared__ __align__(16) float Ws[BK][BM + 4];
  __shared__ __align__(16) float Xs[BK][BN + 4];
  const int tid = threadIdx.x;
  const int row0 = blockIdx.x * BM, tok0 = blockIdx.y * BN;
  const int ty = tid >> 4, tx = tid & 15;
  const DevMat& w = p.w;
  const int K = w.cols;
  const int lr = tid >> 2, lk = (tid & 3) * 8;
  const int64_t row = row0 + lr;
  const int tok = tok0 + lr;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }

  for (int kb = 0; kb < K / BK; ++kb) {
    float wv[8], xv[8];
    const int b = kb >> 3;
    const uint8_t* grp = dev::GroupPtr(w, row, b);
    const int r16 = static_cast<int>(row & 15), g = r16 & 7, rs = r16 >> 3;
    if (w.type == 13u || w.type == 8u) {  // one byte per weight: element by element
#pragma unroll
      for (int i = 0; i < 8; ++i) wv[i] = dev::DeqElem(w, row, kb * BK + lk + i);
    } else if (w.type == 12u) {
      const int j = kb & 7;
      const uint4 hd = *reinterpret_cast<const uint4*>(grp + 2048 + 16 * r16);
      int sc, m;
      dev::Q4kScaleMin(hd.y, hd.z, hd.w, j, &sc, &m);
      const float d1 = __fmul_rn(dev::Half(hd.x & 0xFFFFu), static_cast<float>(sc));
      const float m1 = __fmul_rn(dev::Half(hd.x >> 16), static_cast<float>(m));
      // positions lk .. lk+7 of sub-block j: words of lanes (g, t0) and (g, t0 + 1)
      const int c = j >> 1, h = lk >> 4, t0 = (lk >> 2) & 3;
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(grp + (c * 32 + 4 * g + t0) * 16 + (2 * h + rs) * 4);
      const uint32_t qw[2] = {wp[0], wp[4]};
      const int sh = (j & 1) * 4;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = static_cast<int>((qw[i >> 2] >> (8 * (i & 3) + sh)) & 15u);
        wv[i] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
      }
    } else {
      // Q6_K sub-block j16 = 2 (kb & 7) + (lk >> 4), positions (lk & 15) .. +7
      const int j16 = 2 * (kb & 7) + (lk >> 4);
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
          wv[4 * tt + e] = __fmul_rn(ds, static_cast<float>(q - 32));
        }
      }
    }
    if (tok < p.n_tok) {
      const float4* xp = reinterpret_cast<const float4*>(p.X + static_cast<int64_t>(tok) * p.ldx + kb * BK + lk);
      const float4 a = xp[0], b = xp[1];
      xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
      xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      Ws[lk + i][lr] = wv[i];
      Xs[lk + i][lr] = xv[i];
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < BK; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&Ws[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&Xs[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
    }
  }

#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int t = tok0 + tx * 4 + j;
    if (t >= p.n_tok) continue;
    const int r = row0 + ty * 4;
    if (EPI == static_cast<int>(Epi::kStore)) {
      float* o = p.out + static_cast<int64_t>(t) * p.ldo + p.out_off + r;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = acc[i][j];
    } else if (EPI == static_cast<int>(Epi::kResid)) {
      float* o = p.out + static_cast<int64_t>(t) * p.ldo + r;
      const float* rs = p.resid + static_cast<int64_t>(t) * p.ldr + r;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = rs[i] + acc[i][j];
    } else {
      float* o = p.out + static_cast<int64_t>(t) * p.ldo + r / 2;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float g = acc[2 * i][j], u = acc[2 * i + 1][j];
        o[i] = (g / (1.0f + expf(-g))) * u;
      }
    }
  }
}

}  // namespace

void LaunchGemm(const GemmParams& p, Epi epi, cudaStream_t s) {
  if (p.tc_scratch != nullptr && p.n_tok >= kTcMinTokens && p.w.rows % 128 == 0) {
    LaunchTcGemm(p, epi, p.tc_scratch, p.tc_scratch_halves, s);
    return;
  }
  RPGB_CHECK(p.w.q != nullptr, "gemm: the FP32 tile path needs the quantised matrix");
  RPGB_CHECK(p.out_h == nullptr, "gemm: fp16 output terms need the tensor-core path");
  RPGB_CHECK(p.w.rows % BM == 0, "gemm: rows %d not a multiple of %d", p.w.rows, BM);
  RPGB_CHECK(p.w.cols % 256 == 0, "gemm: cols %d not a multiple of 256", p.w.cols);
  RPGB_CHECK(p.n_tok > 0, "gemm: no tokens");
  const dim3 grid(p.w.rows / BM, (p.n_tok + BN - 1) / BN);
  RPGB_CHECK(grid.y < 65536, "gemm: too many tokens");
  switch (epi) {
    case Epi::kStore: GemmKernel<0><<<grid, 256, 0, s>>>(p); break;
    case Epi::kResid: GemmKernel<1><<<grid, 256, 0, s>>>(p); break;
    case Epi::kSilu: GemmKernel<2><<<grid, 256, 0, s>>>(p); break;
    default: Throw("gemm: unsupported epilogue");
  }
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

}  // namespace rpgb
