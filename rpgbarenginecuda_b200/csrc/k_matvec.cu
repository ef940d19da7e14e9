// k_matvec.cu -- decode (n = 1) dequant-fused matvec for Q4_K / Q6_K.
//
// Replaces MatMulQ4KKernel / MatMulQ6KKernel with TILE = 1 (src/kernels_gpu.cu:
// 325-494) and the surrounding RmsNorm / VecAdd / SiluMul / ArgMax launches of
// GpuForwardLayer (src/qwen3_gpu.cu:47-109): one launch computes
// prologue(x) -> W x -> epilogue.
//
// Work split: a warp owns `RW` consecutive output rows; each lane walks the
// row's 64-weight units (u = lane, lane+32, ...), so one warp-wide load
// instruction reads 32 consecutive 16-byte chunks of the repacked weights.  The
// activation vector (and per-32 sub-block sums for the Q4_K min term) lives in
// shared memory and is read once per unit for all RW rows.  Blocks are
// persistent (grid <= 2 x SMs) so the prologue runs once per block.
#include <cfloat>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"

namespace rpgb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// x (K floats) + sub-block sums (K/32 floats) for K up to 16384.
constexpr size_t kMaxMatvecSmem = (16384 + 512) * sizeof(float);

template <int RW>
__device__ __forceinline__ void DotQ4K(const DevMat& w, int lr0, const float* __restrict__ xs,
                                       const float* __restrict__ sx, int lane, float (&acc)[RW]) {
  const int nb = w.nb;
  const int units = nb * 4;
  for (int u = lane; u < units; u += 32) {
    const int b = u >> 2, j = u & 3;
    // Unit (b, j) = qs bytes [32j, 32j+32) of block b = sub-blocks 2j (low
    // nibbles) and 2j+1 (high nibbles), elements 64j .. 64j+63.
    const float4* xp = reinterpret_cast<const float4*>(xs + b * 256 + 64 * j);
    float4 xa[8], xb[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xa[i] = xp[i];
      xb[i] = xp[8 + i];
    }
    const float sxa = sx[b * 8 + 2 * j], sxb = sx[b * 8 + 2 * j + 1];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int64_t blk = static_cast<int64_t>(lr0 + r) * nb + b;
      const uint4 q0 = dev::LdStream(w.q + blk * 128 + 32 * j);
      const uint4 q1 = dev::LdStream(w.q + blk * 128 + 32 * j + 16);
      const uint4 hd = dev::LdStream(w.s + blk * 16);
      int sca, ma, scb, mb;
      dev::Q4kScaleMin(hd.y, hd.z, hd.w, 2 * j, &sca, &ma);
      dev::Q4kScaleMin(hd.y, hd.z, hd.w, 2 * j + 1, &scb, &mb);
      const float d = dev::Half(hd.x & 0xFFFFu), dmin = dev::Half(hd.x >> 16);
      const uint32_t wd[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t lo = wd[k] & 0x0F0F0F0Fu;
        const uint32_t hi = (wd[k] >> 4) & 0x0F0F0F0Fu;
        const float4 a = xa[k], c = xb[k];
        sa = fmaf(dev::ByteBiased<0>(lo) - 8388608.f, a.x, sa);
        sb = fmaf(dev::ByteBiased<0>(hi) - 8388608.f, c.x, sb);
        sa = fmaf(dev::ByteBiased<1>(lo) - 8388608.f, a.y, sa);
        sb = fmaf(dev::ByteBiased<1>(hi) - 8388608.f, c.y, sb);
        sa = fmaf(dev::ByteBiased<2>(lo) - 8388608.f, a.z, sa);
        sb = fmaf(dev::ByteBiased<2>(hi) - 8388608.f, c.z, sb);
        sa = fmaf(dev::ByteBiased<3>(lo) - 8388608.f, a.w, sa);
        sb = fmaf(dev::ByteBiased<3>(hi) - 8388608.f, c.w, sb);
      }
      const float da = d * static_cast<float>(sca), db = d * static_cast<float>(scb);
      const float ma_f = dmin * static_cast<float>(ma), mb_f = dmin * static_cast<float>(mb);
      acc[r] += da * sa + db * sb - (ma_f * sxa + mb_f * sxb);
    }
  }
}

template <int RW>
__device__ __forceinline__ void DotQ6K(const DevMat& w, int lr0, const float* __restrict__ xs, int lane,
                                       float (&acc)[RW]) {
  const int nb = w.nb;
  const int units = nb * 4;
  for (int u = lane; u < units; u += 32) {
    // Unit (b, hh, bb): elements 128hh + 32q + 16bb + i, q = 0..3, i = 0..15.
    const int b = u >> 2, hh = (u >> 1) & 1, bb = u & 1;
    const float* xb = xs + b * 256 + 128 * hh + 16 * bb;
    float4 xq[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int i = 0; i < 4; ++i) xq[q][i] = reinterpret_cast<const float4*>(xb + 32 * q)[i];
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      const int64_t blk = static_cast<int64_t>(lr0 + r) * nb + b;
      const uint8_t* base = w.q + blk * 192;
      const uint4 A = dev::LdStream(base + 64 * hh + 16 * bb);
      const uint4 B = dev::LdStream(base + 64 * hh + 32 + 16 * bb);
      const uint4 H = dev::LdStream(base + 128 + 32 * hh + 16 * bb);
      const uint4 S = dev::LdStream(w.s + blk * 16);
      const float d = dev::Half(__ldg(w.d + blk));
      const int si = 8 * hh + bb;
      const float d0 = d * static_cast<float>(dev::Q6kScale(S, si));
      const float d1 = d * static_cast<float>(dev::Q6kScale(S, si + 2));
      const float d2 = d * static_cast<float>(dev::Q6kScale(S, si + 4));
      const float d3 = d * static_cast<float>(dev::Q6kScale(S, si + 6));
      const uint32_t Aw[4] = {A.x, A.y, A.z, A.w};
      const uint32_t Bw[4] = {B.x, B.y, B.z, B.w};
      const uint32_t Hw[4] = {H.x, H.y, H.z, H.w};
      float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t u0 = (Aw[k] & 0x0F0F0F0Fu) | ((Hw[k] << 4) & 0x30303030u);
        const uint32_t u1 = (Bw[k] & 0x0F0F0F0Fu) | ((Hw[k] << 2) & 0x30303030u);
        const uint32_t u2 = ((Aw[k] >> 4) & 0x0F0F0F0Fu) | (Hw[k] & 0x30303030u);
        const uint32_t u3 = ((Bw[k] >> 4) & 0x0F0F0F0Fu) | ((Hw[k] >> 2) & 0x30303030u);
        // 8388640 = 2^23 + 32 turns the 6-bit value into (q - 32).
        t0 = fmaf(dev::ByteBiased<0>(u0) - 8388640.f, xq[0][k].x, t0);
        t1 = fmaf(dev::ByteBiased<0>(u1) - 8388640.f, xq[1][k].x, t1);
        t2 = fmaf(dev::ByteBiased<0>(u2) - 8388640.f, xq[2][k].x, t2);
        t3 = fmaf(dev::ByteBiased<0>(u3) - 8388640.f, xq[3][k].x, t3);
        t0 = fmaf(dev::ByteBiased<1>(u0) - 8388640.f, xq[0][k].y, t0);
        t1 = fmaf(dev::ByteBiased<1>(u1) - 8388640.f, xq[1][k].y, t1);
        t2 = fmaf(dev::ByteBiased<1>(u2) - 8388640.f, xq[2][k].y, t2);
        t3 = fmaf(dev::ByteBiased<1>(u3) - 8388640.f, xq[3][k].y, t3);
        t0 = fmaf(dev::ByteBiased<2>(u0) - 8388640.f, xq[0][k].z, t0);
        t1 = fmaf(dev::ByteBiased<2>(u1) - 8388640.f, xq[1][k].z, t1);
        t2 = fmaf(dev::ByteBiased<2>(u2) - 8388640.f, xq[2][k].z, t2);
        t3 = fmaf(dev::ByteBiased<2>(u3) - 8388640.f, xq[3][k].z, t3);
        t0 = fmaf(dev::ByteBiased<3>(u0) - 8388640.f, xq[0][k].w, t0);
        t1 = fmaf(dev::ByteBiased<3>(u1) - 8388640.f, xq[1][k].w, t1);
        t2 = fmaf(dev::ByteBiased<3>(u2) - 8388640.f, xq[2][k].w, t2);
        t3 = fmaf(dev::ByteBiased<3>(u3) - 8388640.f, xq[3][k].w, t3);
      }
      acc[r] += d0 * t0 + d1 * t1 + d2 * t2 + d3 * t3;
    }
  }
}

template <int RW, bool NORM, int EPI>
__global__ void __launch_bounds__(kThreads) MatvecKernel(const MvParams p) {
  extern __shared__ __align__(16) float smem[];
  __shared__ double red[32];
  __shared__ float s_bv[kWarps];
  __shared__ int s_bi[kWarps];
  __shared__ int s_last;

  const int K = p.seg[0].w.cols;
  float* xs = smem;
  float* sx = smem + K;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- prologue: x (optionally RMSNorm'ed) and 32-element sums into shared memory
  double ss = 0.0;
  for (int i = threadIdx.x * 4; i < K; i += kThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(p.x + i);
    *reinterpret_cast<float4*>(xs + i) = v;
    if (NORM) {
      ss += static_cast<double>(v.x) * v.x;
      ss += static_cast<double>(v.y) * v.y;
      ss += static_cast<double>(v.z) * v.z;
      ss += static_cast<double>(v.w) * v.w;
    }
  }
  if (NORM) {
    // RMSNorm as src/kernels_gpu.cu:564-591: double sum of squares,
    // scale = float(1/sqrt(mean + eps)), out = x * scale * w.
    const double tot = dev::BlockSumD(ss, red);
    const float scale = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(K) + static_cast<double>(p.eps)));
    for (int i = threadIdx.x * 4; i < K; i += kThreads * 4) {
      float4 v = *reinterpret_cast<float4*>(xs + i);
      const float4 g = *reinterpret_cast<const float4*>(p.norm_w + i);
      v.x = v.x * scale * g.x;
      v.y = v.y * scale * g.y;
      v.z = v.z * scale * g.z;
      v.w = v.w * scale * g.w;
      *reinterpret_cast<float4*>(xs + i) = v;
    }
  }
  __syncthreads();
  for (int j = warp; j < K / 32; j += kWarps) {
    const float v = dev::WarpSum(xs[32 * j + lane]);
    if (lane == 0) sx[j] = v;
  }
  __syncthreads();

  // ---- rows
  float best_v = -FLT_MAX;
  int best_i = 0;
  const int n_tasks = p.total_rows / RW;
  for (int task = blockIdx.x * kWarps + warp; task < n_tasks; task += gridDim.x * kWarps) {
    const int row0 = task * RW;
    int si = 0;
    if (p.n_seg > 1 && row0 >= p.seg[1].out_off) si = 1;
    if (p.n_seg > 2 && row0 >= p.seg[2].out_off) si = 2;
    const DevMat w = p.seg[si].w;
    const int lr0 = row0 - p.seg[si].out_off;
    float acc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) acc[r] = 0.f;
    if (w.type == 12u) {
      DotQ4K<RW>(w, lr0, xs, sx, lane, acc);
    } else {
      DotQ6K<RW>(w, lr0, xs, lane, acc);
    }
#pragma unroll
    for (int r = 0; r < RW; ++r) acc[r] = dev::WarpSum(acc[r]);
    if (lane == 0) {
      if (EPI == static_cast<int>(Epi::kStore)) {
#pragma unroll
        for (int r = 0; r < RW; ++r) p.out[row0 + r] = acc[r];
      } else if (EPI == static_cast<int>(Epi::kResid)) {
#pragma unroll
        for (int r = 0; r < RW; ++r) p.out[row0 + r] = p.resid[row0 + r] + acc[r];
      } else if (EPI == static_cast<int>(Epi::kSilu)) {
#pragma unroll
        for (int r = 0; r < RW / 2; ++r) {
          const float g = acc[2 * r], u = acc[2 * r + 1];
          // (g / (1 + exp(-g))) * u, as src/kernels_gpu.cu:863-869
          p.out[row0 / 2 + r] = (g / (1.0f + expf(-g))) * u;
        }
      } else {
#pragma unroll
        for (int r = 0; r < RW; ++r) {
          p.out[row0 + r] = acc[r];
          if (acc[r] > best_v) {
            best_v = acc[r];
            best_i = row0 + r;
          }
        }
      }
    }
  }

  if (EPI == static_cast<int>(Epi::kArgmax)) {
    // Ties go to the lowest index at every level (src/kernels_gpu.cu:827-859).
    if (lane == 0) {
      s_bv[warp] = best_v;
      s_bi[warp] = best_i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float bv = s_bv[0];
      int bi = s_bi[0];
      for (int i = 1; i < kWarps; ++i) {
        if (s_bv[i] > bv || (s_bv[i] == bv && s_bi[i] < bi)) {
          bv = s_bv[i];
          bi = s_bi[i];
        }
      }
      p.part_val[blockIdx.x] = bv;
      p.part_idx[blockIdx.x] = bi;
      __threadfence();
      const unsigned t = atomicAdd(p.ticket, 1u);
      s_last = (t == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      float bv = -FLT_MAX;
      int bi = 0x7FFFFFFF;
      for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += kThreads) {
        const float v = __ldcg(p.part_val + i);
        const int ix = __ldcg(p.part_idx + i);
        if (v > bv || (v == bv && ix < bi)) {
          bv = v;
          bi = ix;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        s_bv[warp] = bv;
        s_bi[warp] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        bv = s_bv[0];
        bi = s_bi[0];
        for (int i = 1; i < kWarps; ++i) {
          if (s_bv[i] > bv || (s_bv[i] == bv && s_bi[i] < bi)) {
            bv = s_bv[i];
            bi = s_bi[i];
          }
        }
        *p.tok_out = bi;
        if (p.pos != nullptr) *p.pos += p.pos_bump;
        *p.ticket = 0u;
      }
    }
  }
}

__global__ void EmbedKernel(const DevMat e, const int32_t* __restrict__ tok, float* __restrict__ x,
                            const int64_t* __restrict__ pos, int32_t* __restrict__ out_ids) {
  const int t = blockIdx.y;
  int32_t id = tok[t];
  if (out_ids != nullptr && blockIdx.x == 0 && threadIdx.x == 0) out_ids[*pos + t] = id;
  if (id < 0 || id >= e.rows) id = 0;  // host validates ids; device-sampled ids are in range
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < e.cols; c += gridDim.x * blockDim.x) {
    x[static_cast<int64_t>(t) * e.cols + c] = dev::DeqElem(e, id, c);
  }
}

__global__ void DequantRowsKernel(const DevMat w, int64_t row0, float* __restrict__ dst) {
  const int64_t r = row0 + blockIdx.y;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < w.cols; c += gridDim.x * blockDim.x) {
    dst[static_cast<int64_t>(blockIdx.y) * w.cols + c] = dev::DeqElem(w, r, c);
  }
}

using MvFn = void (*)(const MvParams);

template <int RW, bool NORM>
MvFn PickEpi(Epi epi) {
  switch (epi) {
    case Epi::kStore: return MatvecKernel<RW, NORM, 0>;
    case Epi::kResid: return MatvecKernel<RW, NORM, 1>;
    case Epi::kSilu:
      if constexpr (RW % 2 == 0) return MatvecKernel<RW, NORM, 2>;
      Throw("kSilu needs an even rows_per_warp");
    case Epi::kArgmax: return MatvecKernel<RW, NORM, 3>;
  }
  Throw("bad epilogue");
}

template <int RW>
MvFn PickNorm(bool norm, Epi epi) {
  return norm ? PickEpi<RW, true>(epi) : PickEpi<RW, false>(epi);
}

}  // namespace

void PrepareMatvecKernels() {
  const Epi epis[4] = {Epi::kStore, Epi::kResid, Epi::kSilu, Epi::kArgmax};
  for (int norm = 0; norm < 2; ++norm) {
    for (Epi e : epis) {
      MvFn fns[3] = {e == Epi::kSilu ? nullptr : PickNorm<1>(norm != 0, e), PickNorm<2>(norm != 0, e),
                     PickNorm<4>(norm != 0, e)};
      for (MvFn f : fns) {
        if (f != nullptr) {
          RPGB_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kMaxMatvecSmem)));
        }
      }
    }
  }
}

int MatvecGrid(int total_rows, int rw, int num_sms) {
  const int tasks = total_rows / rw;
  const int need = (tasks + kWarps - 1) / kWarps;
  return std::max(1, std::min(need, num_sms * 2));
}

void LaunchMatvec(const MvParams& p, Epi epi, int rw, int num_sms, cudaStream_t s) {
  const int K = p.seg[0].w.cols;
  RPGB_CHECK(p.n_seg >= 1 && p.n_seg <= 3, "matvec: 1..3 segments");
  RPGB_CHECK(K % 256 == 0 && K > 0, "matvec: width %d is not a multiple of 256", K);
  int rows = 0;
  for (int i = 0; i < p.n_seg; ++i) {
    RPGB_CHECK(p.seg[i].w.cols == K, "matvec: segments differ in width");
    RPGB_CHECK(p.seg[i].out_off == rows, "matvec: segments must be contiguous");
    RPGB_CHECK(p.seg[i].w.rows % (rw * (epi == Epi::kSilu ? 1 : 1)) == 0, "matvec: rows %% rows_per_warp != 0");
    RPGB_CHECK(p.seg[i].w.type == kGgmlQ4_K || p.seg[i].w.type == kGgmlQ6_K, "matvec: unsupported type");
    rows += p.seg[i].w.rows;
  }
  RPGB_CHECK(rows == p.total_rows, "matvec: total_rows mismatch");
  MvFn fn = nullptr;
  switch (rw) {
    case 1: fn = PickNorm<1>(p.norm_w != nullptr, epi); break;
    case 2: fn = PickNorm<2>(p.norm_w != nullptr, epi); break;
    case 4: fn = PickNorm<4>(p.norm_w != nullptr, epi); break;
    default: Throw("rows_per_warp must be 1, 2 or 4");
  }
  const size_t smem = static_cast<size_t>(K + K / 32) * sizeof(float);
  RPGB_CHECK(smem <= kMaxMatvecSmem, "matvec: width %d needs %zu bytes of shared memory (limit %zu)", K, smem,
             kMaxMatvecSmem);
  const int grid = MatvecGrid(p.total_rows, rw, num_sms);
  fn<<<grid, kThreads, smem, s>>>(p);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

void LaunchEmbed(const DevMat& embd, const int32_t* tok, int n_tok, float* x, const int64_t* pos,
                 int32_t* out_ids, cudaStream_t s) {
  RPGB_CHECK(n_tok > 0 && n_tok < 65536, "embed: bad token count %d", n_tok);
  const dim3 grid((embd.cols + 255) / 256, n_tok);
  EmbedKernel<<<grid, 256, 0, s>>>(embd, tok, x, pos, out_ids);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

void LaunchDequantRows(const DevMat& w, int64_t row0, int64_t n_rows, float* dst, cudaStream_t s) {
  RPGB_CHECK(row0 >= 0 && n_rows > 0 && row0 + n_rows <= w.rows && n_rows < 65536, "dequant: bad row range");
  const dim3 grid((w.cols + 255) / 256, static_cast<unsigned>(n_rows));
  DequantRowsKernel<<<grid, 256, 0, s>>>(w, row0, dst);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

}  // namespace rpgb
