// k_matvec.cu -- decode (n = 1) dequant-fused matvec for Q4_K / Q6_K.
//
// Replaces MatMulQ4KKernel / MatMulQ6KKernel with TILE = 1 (src/kernels_gpu.cu:
// 325-494) and the surrounding RmsNorm / VecAdd / SiluMul / ArgMax launches of
// GpuForwardLayer (src/qwen3_gpu.cu:47-109): one launch computes
// prologue(x) -> W x -> epilogue.
//
// Structure (one persistent block per SM, 8 warps):
//  * the block owns a contiguous range of 32-row groups; its weights stream
//    through a ring of shared-memory slots filled by 1-D TMA bulk copies
//    (cp.async.bulk + mbarrier), one slot = (group, up to `kb` blocks);
//  * the first ring slots are requested BEFORE griddepcontrol.wait: with
//    programmatic dependent launch the weights of this kernel stream in while
//    the previous kernel of the decode step is still computing;
//  * lane r of every warp owns row r of the group (row-interleaved layout, see
//    kernels.cuh), the 8 warps split the block units of a slot, x is read from
//    shared memory as broadcast float4 loads, and the 8 partial sums of a row
//    are combined once per group -- no per-row shuffles;
//  * Q4_K regroups (d*sc)*sum(q*x) - (dmin*m)*sum(x) per 32-element sub-block,
//    Q6_K (d*sc)*sum((q-32)*x) per 16-element sub-block; the 4- and 6-bit
//    values become floats exactly via the 2^23 mantissa trick (PRMT + FADD).
#include <algorithm>
#include <cfloat>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "launch.h"

namespace rpgb {
namespace {

using dev::kGroupRows;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxSlots = 8;
// Dynamic shared memory budget per block: leaves room for the next kernel's
// block on the same SM (programmatic launch overlap needs co-residency).
constexpr size_t kSmemBudget = 110 * 1024;
constexpr size_t kSmemLimit = kSmemBudget + 8192;

struct Layout {
  size_t ring, xs, sx, red, bars, total;
};

__host__ __device__ inline Layout SmemLayout(int K, int slots, int slot_bytes) {
  Layout l;
  l.ring = 0;
  l.xs = static_cast<size_t>(slots) * slot_bytes;
  l.sx = l.xs + static_cast<size_t>(K) * 4;
  l.red = l.sx + static_cast<size_t>(K / 32) * 4;
  l.bars = l.red + kWarps * 32 * 4;
  l.total = l.bars + kMaxSlots * 8;
  return l;
}

__device__ __forceinline__ int SegOf(const MvParams& p, int row) {
  int si = 0;
  if (p.n_seg > 1 && row >= p.seg[1].out_off) si = 1;
  if (p.n_seg > 2 && row >= p.seg[2].out_off) si = 2;
  return si;
}

// Issues the bulk copies of stage `st` (group gb + st / n_chunks, chunk st % n_chunks).
__device__ __forceinline__ void IssueStage(const MvParams& p, int st, int gb, uint8_t* ring, uint64_t* bars) {
  const int g = gb + st / p.n_chunks, c = st % p.n_chunks;
  const int si = SegOf(p, g * kGroupRows);
  const DevMat& w = p.seg[si].w;
  const int lg = g - p.seg[si].out_off / kGroupRows;
  const int nb = w.nb, b0 = c * p.kb, kbn = min(p.kb, nb - b0);
  const int nc = dev::QChunks(w.type);
  const uint32_t qb = static_cast<uint32_t>(kbn * nc * 512), sb = static_cast<uint32_t>(kbn * 512);
  const uint32_t db = w.type == 14u ? static_cast<uint32_t>(kbn * 64) : 0u;
  const int slot = st % p.slots;
  uint8_t* dst = ring + static_cast<size_t>(slot) * p.slot_bytes;
  uint64_t* bar = bars + slot;
  const int64_t gblk = static_cast<int64_t>(lg) * nb + b0;
  dev::MbarExpectTx(bar, qb + sb + db);
  dev::BulkG2S(dst, w.q + gblk * nc * 512, qb, bar);
  dev::BulkG2S(dst + p.kb * nc * 512, w.s + gblk * 512, sb, bar);
  if (db) dev::BulkG2S(dst + p.kb * nc * 512 + p.kb * 512, w.d + gblk * 32, db, bar);
}

// One 64-weight Q4_K unit (block bl of the slot, qs bytes [32j, 32j+32)) for the lane's row.
__device__ __forceinline__ float UnitQ4K(const uint8_t* slot, int kb, int bl, int j, int lane,
                                         const float* __restrict__ xs, const float* __restrict__ sx, int b) {
  const uint4 q0 = *reinterpret_cast<const uint4*>(slot + (bl * 8 + 2 * j) * 512 + lane * 16);
  const uint4 q1 = *reinterpret_cast<const uint4*>(slot + (bl * 8 + 2 * j + 1) * 512 + lane * 16);
  const uint4 hd = *reinterpret_cast<const uint4*>(slot + kb * 8 * 512 + bl * 512 + lane * 16);
  const float4* xp = reinterpret_cast<const float4*>(xs + b * 256 + 64 * j);
  const uint32_t wd[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  float sa = 0.f, sb = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t lo = wd[k] & 0x0F0F0F0Fu;
    const uint32_t hi = (wd[k] >> 4) & 0x0F0F0F0Fu;
    const float4 a = xp[k], c = xp[8 + k];
    sa = fmaf(dev::ByteBiased<0>(lo) - 8388608.f, a.x, sa);
    sb = fmaf(dev::ByteBiased<0>(hi) - 8388608.f, c.x, sb);
    sa = fmaf(dev::ByteBiased<1>(lo) - 8388608.f, a.y, sa);
    sb = fmaf(dev::ByteBiased<1>(hi) - 8388608.f, c.y, sb);
    sa = fmaf(dev::ByteBiased<2>(lo) - 8388608.f, a.z, sa);
    sb = fmaf(dev::ByteBiased<2>(hi) - 8388608.f, c.z, sb);
    sa = fmaf(dev::ByteBiased<3>(lo) - 8388608.f, a.w, sa);
    sb = fmaf(dev::ByteBiased<3>(hi) - 8388608.f, c.w, sb);
  }
  int sca, ma, scb, mb;
  dev::Q4kScaleMin(hd.y, hd.z, hd.w, 2 * j, &sca, &ma);
  dev::Q4kScaleMin(hd.y, hd.z, hd.w, 2 * j + 1, &scb, &mb);
  const float d = dev::Half(hd.x & 0xFFFFu), dmin = dev::Half(hd.x >> 16);
  const float da = d * static_cast<float>(sca), db = d * static_cast<float>(scb);
  const float ma_f = dmin * static_cast<float>(ma), mb_f = dmin * static_cast<float>(mb);
  return da * sa + db * sb - (ma_f * sx[b * 8 + 2 * j] + mb_f * sx[b * 8 + 2 * j + 1]);
}

// One 64-weight Q6_K unit (block bl, half hh, 16-run bb) for the lane's row.
__device__ __forceinline__ float UnitQ6K(const uint8_t* slot, int kb, int bl, int hh, int bb, int lane,
                                         const float* __restrict__ xs, int b) {
  const uint8_t* qp = slot + bl * 12 * 512 + lane * 16;
  const uint4 A = *reinterpret_cast<const uint4*>(qp + (4 * hh + bb) * 512);
  const uint4 B = *reinterpret_cast<const uint4*>(qp + (4 * hh + 2 + bb) * 512);
  const uint4 H = *reinterpret_cast<const uint4*>(qp + (8 + 2 * hh + bb) * 512);
  const uint4 S = *reinterpret_cast<const uint4*>(slot + kb * 12 * 512 + bl * 512 + lane * 16);
  const uint16_t dh = *reinterpret_cast<const uint16_t*>(slot + kb * 12 * 512 + kb * 512 + bl * 64 + lane * 2);
  const float* xb = xs + b * 256 + 128 * hh + 16 * bb;
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
    const float4 x0 = reinterpret_cast<const float4*>(xb)[k];
    const float4 x1 = reinterpret_cast<const float4*>(xb + 32)[k];
    const float4 x2 = reinterpret_cast<const float4*>(xb + 64)[k];
    const float4 x3 = reinterpret_cast<const float4*>(xb + 96)[k];
    // 8388640 = 2^23 + 32 turns the 6-bit value into (q - 32).
    t0 = fmaf(dev::ByteBiased<0>(u0) - 8388640.f, x0.x, t0);
    t1 = fmaf(dev::ByteBiased<0>(u1) - 8388640.f, x1.x, t1);
    t2 = fmaf(dev::ByteBiased<0>(u2) - 8388640.f, x2.x, t2);
    t3 = fmaf(dev::ByteBiased<0>(u3) - 8388640.f, x3.x, t3);
    t0 = fmaf(dev::ByteBiased<1>(u0) - 8388640.f, x0.y, t0);
    t1 = fmaf(dev::ByteBiased<1>(u1) - 8388640.f, x1.y, t1);
    t2 = fmaf(dev::ByteBiased<1>(u2) - 8388640.f, x2.y, t2);
    t3 = fmaf(dev::ByteBiased<1>(u3) - 8388640.f, x3.y, t3);
    t0 = fmaf(dev::ByteBiased<2>(u0) - 8388640.f, x0.z, t0);
    t1 = fmaf(dev::ByteBiased<2>(u1) - 8388640.f, x1.z, t1);
    t2 = fmaf(dev::ByteBiased<2>(u2) - 8388640.f, x2.z, t2);
    t3 = fmaf(dev::ByteBiased<2>(u3) - 8388640.f, x3.z, t3);
    t0 = fmaf(dev::ByteBiased<3>(u0) - 8388640.f, x0.w, t0);
    t1 = fmaf(dev::ByteBiased<3>(u1) - 8388640.f, x1.w, t1);
    t2 = fmaf(dev::ByteBiased<3>(u2) - 8388640.f, x2.w, t2);
    t3 = fmaf(dev::ByteBiased<3>(u3) - 8388640.f, x3.w, t3);
  }
  const float d = dev::Half(dh);
  const int si = 8 * hh + bb;
  return (d * static_cast<float>(dev::Q6kScale(S, si))) * t0 + (d * static_cast<float>(dev::Q6kScale(S, si + 2))) * t1 +
         (d * static_cast<float>(dev::Q6kScale(S, si + 4))) * t2 +
         (d * static_cast<float>(dev::Q6kScale(S, si + 6))) * t3;
}

template <bool NORM, int EPI>
__global__ void __launch_bounds__(kThreads, 1) MatvecKernel(const MvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ double dred[32];
  __shared__ float s_bv[kWarps];
  __shared__ int s_bi[kWarps];
  __shared__ int s_last;

  const int K = p.seg[0].w.cols;
  const Layout L = SmemLayout(K, p.slots, p.slot_bytes);
  uint8_t* ring = smem + L.ring;
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  float* sx = reinterpret_cast<float*>(smem + L.sx);
  float* red = reinterpret_cast<float*>(smem + L.red);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int G = p.n_groups;
  const int gb = static_cast<int>((static_cast<int64_t>(blockIdx.x) * G) / gridDim.x);
  const int ge = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * G) / gridDim.x);
  const int n_stages = (ge - gb) * p.n_chunks;

  // ---- weights first: they do not depend on the previous kernel
  if (tid == 0) {
    for (int s = 0; s < p.slots; ++s) dev::MbarInit(bars + s, 1);
    dev::MbarInitFence();
  }
  __syncthreads();
  if (tid == 0) {
    const int pre = n_stages < p.slots ? n_stages : p.slots;
    for (int st = 0; st < pre; ++st) IssueStage(p, st, gb, ring, bars);
  }
  dev::GridLaunchDependents();
  dev::GridWait();

  // ---- prologue: x (optionally RMSNorm'ed) and 32-element sums
  double ss = 0.0;
  for (int i = tid * 4; i < K; i += kThreads * 4) {
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
    const double tot = dev::BlockSumD(ss, dred);
    const float scale = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(K) + static_cast<double>(p.eps)));
    for (int i = tid * 4; i < K; i += kThreads * 4) {
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

  // ---- stream the stages
  float acc = 0.f;
  float best_v = -FLT_MAX;
  int best_i = 0;
  bool timed_out = false;
  for (int st = 0; st < n_stages; ++st) {
    const int slot = st % p.slots;
    if (!timed_out && !dev::MbarWait(bars + slot, static_cast<uint32_t>((st / p.slots) & 1))) timed_out = true;
    const int g = gb + st / p.n_chunks, c = st % p.n_chunks;
    const int si = SegOf(p, g * kGroupRows);
    const uint32_t type = p.seg[si].w.type;
    const int nb = p.seg[si].w.nb;
    const int b0 = c * p.kb, kbn = min(p.kb, nb - b0);
    const uint8_t* sl = ring + static_cast<size_t>(slot) * p.slot_bytes;
    if (!timed_out) {
      if (type == 12u) {
        for (int u = warp; u < kbn * 4; u += kWarps) {
          acc += UnitQ4K(sl, p.kb, u >> 2, u & 3, lane, xs, sx, b0 + (u >> 2));
        }
      } else {
        for (int u = warp; u < kbn * 4; u += kWarps) {
          acc += UnitQ6K(sl, p.kb, u >> 2, (u >> 1) & 1, u & 1, lane, xs, b0 + (u >> 2));
        }
      }
    }
    const bool last = c == p.n_chunks - 1;
    if (last) {
      red[warp * 32 + lane] = acc;
      acc = 0.f;
    }
    __syncthreads();
    if (tid == 0 && !timed_out && st + p.slots < n_stages) {
      dev::FenceProxyAsync();
      IssueStage(p, st + p.slots, gb, ring, bars);
    }
    if (last && warp == 0) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += red[w * 32 + lane];
      const int row = g * kGroupRows + lane;
      if (EPI == static_cast<int>(Epi::kStore)) {
        p.out[row] = v;
      } else if (EPI == static_cast<int>(Epi::kResid)) {
        p.out[row] = p.resid[row] + v;
      } else if (EPI == static_cast<int>(Epi::kSilu)) {
        // rows 2i (gate) and 2i+1 (up) sit on adjacent lanes
        const float up = __shfl_down_sync(0xFFFFFFFFu, v, 1);
        // (g / (1 + exp(-g))) * u, as src/kernels_gpu.cu:863-869
        if ((lane & 1) == 0) p.out[row >> 1] = (v / (1.0f + expf(-v))) * up;
      } else {
        p.out[row] = v;
        if (v > best_v) {  // a lane's rows increase: strict > keeps the lowest index
          best_v = v;
          best_i = row;
        }
      }
    }
  }
  if (timed_out && p.err != nullptr) atomicOr(p.err, 1);

  if (EPI == static_cast<int>(Epi::kArgmax)) {
    // Ties go to the lowest index at every level (src/kernels_gpu.cu:827-859).
    if (warp == 0) {
      if (n_stages == 0) best_i = 0x7FFFFFFF;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best_v, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, best_i, o);
        if (ov > best_v || (ov == best_v && oi < best_i)) {
          best_v = ov;
          best_i = oi;
        }
      }
      if (lane == 0) {
        p.part_val[blockIdx.x] = best_v;
        p.part_idx[blockIdx.x] = best_i;
        __threadfence();
        const unsigned t = atomicAdd(p.ticket, 1u);
        s_last = (t == gridDim.x - 1) ? 1 : 0;
      }
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      float bv = -FLT_MAX;
      int bi = 0x7FFFFFFF;
      for (int i = tid; i < static_cast<int>(gridDim.x); i += kThreads) {
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
      if (tid == 0) {
        bv = s_bv[0];
        bi = s_bi[0];
        for (int i = 1; i < kWarps; ++i) {
          if (s_bv[i] > bv || (s_bv[i] == bv && s_bi[i] < bi)) {
            bv = s_bv[i];
            bi = s_bi[i];
          }
        }
        *p.tok_out = bi == 0x7FFFFFFF ? 0 : bi;
        if (p.pos != nullptr) *p.pos += p.pos_bump;
        *p.ticket = 0u;
      }
    }
  }
}

__global__ void EmbedKernel(const DevMat e, const int32_t* __restrict__ tok, float* __restrict__ x,
                            const int64_t* __restrict__ pos, int32_t* __restrict__ out_ids) {
  dev::GridLaunchDependents();
  dev::GridWait();
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

template <bool NORM>
MvFn PickEpi(Epi epi) {
  switch (epi) {
    case Epi::kStore: return MatvecKernel<NORM, 0>;
    case Epi::kResid: return MatvecKernel<NORM, 1>;
    case Epi::kSilu: return MatvecKernel<NORM, 2>;
    case Epi::kArgmax: return MatvecKernel<NORM, 3>;
  }
  Throw("bad epilogue");
}

}  // namespace

void PrepareMatvecKernels() {
  const Epi epis[4] = {Epi::kStore, Epi::kResid, Epi::kSilu, Epi::kArgmax};
  for (int norm = 0; norm < 2; ++norm) {
    for (Epi e : epis) {
      MvFn f = norm ? PickEpi<true>(e) : PickEpi<false>(e);
      RPGB_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)));
    }
  }
}

int MatvecGrid(int total_rows, int /*rows_per_warp*/, int num_sms) {
  const int groups = total_rows / kGroupRows;
  return std::max(1, std::min(groups, num_sms));
}

void LaunchMatvec(const MvParams& in, Epi epi, int /*rows_per_warp*/, int num_sms, cudaStream_t s, bool pdl) {
  MvParams p = in;
  const int K = p.seg[0].w.cols;
  RPGB_CHECK(p.n_seg >= 1 && p.n_seg <= 3, "matvec: 1..3 segments");
  RPGB_CHECK(K % 256 == 0 && K > 0 && K <= 16384, "matvec: width %d must be a multiple of 256 up to 16384", K);
  int rows = 0;
  size_t per_block = 0;
  for (int i = 0; i < p.n_seg; ++i) {
    const DevMat& w = p.seg[i].w;
    RPGB_CHECK(w.cols == K, "matvec: segments differ in width");
    RPGB_CHECK(p.seg[i].out_off == rows, "matvec: segments must be contiguous");
    RPGB_CHECK(w.rows % kGroupRows == 0, "matvec: rows %d not a multiple of %d", w.rows, kGroupRows);
    RPGB_CHECK(w.type == kGgmlQ4_K || w.type == kGgmlQ6_K, "matvec: unsupported type");
    const size_t pb = w.type == kGgmlQ4_K ? (8 * 512 + 512) : (12 * 512 + 512 + 64);
    per_block = std::max(per_block, pb);
    rows += w.rows;
  }
  RPGB_CHECK(rows == p.total_rows, "matvec: total_rows mismatch");
  const int nb = K / 256;
  p.kb = std::min(nb, 4);
  p.n_chunks = (nb + p.kb - 1) / p.kb;
  p.slot_bytes = static_cast<int32_t>(per_block * p.kb);
  const size_t xbytes = static_cast<size_t>(K) * 4 + static_cast<size_t>(K / 32) * 4;
  const int slots = static_cast<int>((kSmemBudget > xbytes ? kSmemBudget - xbytes : 0) / p.slot_bytes);
  p.slots = std::max(2, std::min(kMaxSlots, slots));
  p.n_groups = rows / kGroupRows;
  const Layout L = SmemLayout(K, p.slots, p.slot_bytes);
  RPGB_CHECK(L.total <= kSmemLimit, "matvec: shared memory plan %zu exceeds the limit", L.total);
  MvFn fn = p.norm_w != nullptr ? PickEpi<true>(epi) : PickEpi<false>(epi);
  const int grid = MatvecGrid(rows, 1, num_sms);
  LaunchKernelArgs(reinterpret_cast<const void*>(fn), dim3(grid), dim3(kThreads), L.total, s, pdl, p);
  CountLaunches(1);
}

void LaunchEmbed(const DevMat& embd, const int32_t* tok, int n_tok, float* x, const int64_t* pos,
                 int32_t* out_ids, cudaStream_t s, bool pdl) {
  RPGB_CHECK(n_tok > 0 && n_tok < 65536, "embed: bad token count %d", n_tok);
  const dim3 grid((embd.cols + 255) / 256, n_tok);
  LaunchKernelArgs(reinterpret_cast<const void*>(EmbedKernel), grid, dim3(256), 0, s, pdl, embd, tok, x, pos,
                   out_ids);
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
