// k_matvec.cu -- decode (n = 1) dequant-fused matvec for Q4_K / Q6_K.
//
// Replaces MatMulQ4KKernel / MatMulQ6KKernel with TILE = 1 (src/kernels_gpu.cu:
// 325-494) and the surrounding RmsNorm / VecAdd / SiluMul / ArgMax launches of
// GpuForwardLayer (src/qwen3_gpu.cu:47-109): one launch computes
// prologue(x) -> W x -> epilogue.
//
// Arithmetic.  A decode matvec streams 4.5-6.6 bits per weight, so at HBM
// speed an SM has a budget of well under one instruction per weight.  The
// products therefore run on the integer tensor cores (mma.sync m16n8k32,
// u8 x s8 -> s32) and stay exact:
//  * the A operand is the quantised weight itself (Q4_K nibble, or 16x the
//    nibble for the high half; Q6_K 6-bit value, or 4x it), unpacked from the
//    block group with one or two logical ops per 4 weights;
//  * x is split per 256-column super-block into four signed 8-bit digits,
//    x = s * (x0 + x1/64 + x2/8192 + x3/2^20), s a power of two with
//    |x / s| < 64, exact to 2^-26 of the super-block's largest |x|.  The digits are the
//    columns of the B operand: columns 0-3 carry the digits of the first 16
//    positions of an MMA, columns 4-7 those of the next sub-block half, so one
//    MMA yields two sub-block partial sums;
//  * integer partial sums are scaled by the 6-bit (Q4_K) or 8-bit (Q6_K)
//    sub-block scale with IMAD; Q6_K's "-32" offset is a second MMA with a
//    constant A; d, dmin and the Q4_K min term (dmin*m*sum(x), sums of x per
//    32 columns precomputed) are applied in FP32 once per super-block.
// Results differ from the reference's per-element FP32 dequant + FMA only by
// rounding (relative 1e-7 level); DeqQ4K / DeqQ6K stay the bit-exact path.
//
// Data movement (one persistent block of 8 warps per SM):
//  * the block owns a contiguous range of 16-row tiles; its (tile, super-block)
//    units are split into 8 contiguous per-warp ranges;
//  * every warp streams its units through its own ring of shared-memory slots
//    with 1-D TMA bulk copies (cp.async.bulk + mbarrier, bounded waits);
//  * the first slots are requested BEFORE griddepcontrol.wait, so with
//    programmatic dependent launch the weights of this kernel stream in while
//    the previous kernel of the decode step still runs;
//  * partial row sums of a warp are combined per tile in shared memory in a
//    fixed order (results are deterministic), then the epilogue runs.
#include <algorithm>
#include <cfloat>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "launch.h"
#include "mv_dev.cuh"

namespace rpgb {
namespace {

using namespace mv;
constexpr int kMaxRing = 6;
constexpr int kBatch = 3;  // prologue super-blocks whose loads a warp issues together
// Dynamic shared memory budget per block: leaves room for the next kernel's
// block on the same SM (programmatic launch overlap needs co-residency).
constexpr size_t kSmemBudget = 108 * 1024;
constexpr size_t kSmemBudgetWide = 190 * 1024;
constexpr size_t kSmemLimit = 200 * 1024;

struct Layout {
  size_t ring, bfrag, sx, sscale, red, sq, bars, total;
};

__host__ __device__ inline Layout SmemLayout(int nb, int ring, int slot_bytes, int max_tiles, int nw) {
  Layout l;
  l.ring = 0;
  l.bfrag = static_cast<size_t>(nw) * ring * slot_bytes;
  l.sx = l.bfrag + static_cast<size_t>(nb) * 1024;
  l.sscale = l.sx + static_cast<size_t>(nb) * 32;
  l.red = l.sscale + static_cast<size_t>(nb) * 4;
  l.sq = l.red + static_cast<size_t>(max_tiles + nw) * kTile * 4;
  l.sq = (l.sq + 7) & ~static_cast<size_t>(7);
  l.bars = l.sq + nw * 8;
  l.total = l.bars + static_cast<size_t>(nw) * ring * 8;
  return l;
}

__device__ __forceinline__ int SegOfTile(const MvParams& p, int tile) {
  const int row = tile * kTile;
  int si = 0;
  if (p.n_seg > 1 && row >= p.seg[1].out_off) si = 1;
  if (p.n_seg > 2 && row >= p.seg[2].out_off) si = 2;
  return si;
}

// Source of the units a warp requests, advanced one unit at a time.
struct IssueCursor {
  const uint8_t* src;
  uint32_t bytes;
  int tile, b, seg_end_tile;
};

__device__ __forceinline__ void CursorSeek(const MvParams& p, int tile, int b, int nb, IssueCursor& c) {
  const int si = SegOfTile(p, tile);
  const DevMat& w = p.seg[si].w;
  const int t0 = p.seg[si].out_off / kTile;
  c.bytes = static_cast<uint32_t>(dev::GroupBytesOf(w.type));
  c.src = w.q + (static_cast<int64_t>(tile - t0) * nb + b) * c.bytes;
  c.tile = tile;
  c.b = b;
  c.seg_end_tile = t0 + w.rows / kTile;
}

__device__ __forceinline__ void IssueNext(const MvParams& p, int nb, IssueCursor& c, uint8_t* dst, uint64_t* bar) {
  dev::MbarExpectTx(bar, c.bytes);
  dev::BulkG2S(dst, c.src, c.bytes, bar);
  // block groups of one segment are contiguous in tile-major order
  c.src += c.bytes;
  if (++c.b == nb) {
    c.b = 0;
    if (++c.tile == c.seg_end_tile) CursorSeek(p, c.tile, 0, nb, c);
  }
}

template <bool NORM, int EPI, int NW>
__global__ void __launch_bounds__(32 * NW, NW == 8 ? 2 : 1) MatvecKernel(const MvParams p) {
  constexpr int kWarps = NW;
  constexpr int kThreads = 32 * NW;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_bv[kWarps];
  __shared__ int s_bi[kWarps];
  __shared__ int s_last;
  dev::TraceScope trace(p.trace);

  const int K = p.seg[0].w.cols, nb = K >> 8;
  const Layout L = SmemLayout(nb, p.ring, p.slot_bytes, p.max_tiles, NW);
  uint8_t* bfrag = smem + L.bfrag;
  float* sx = reinterpret_cast<float*>(smem + L.sx);
  float* sscale = reinterpret_cast<float*>(smem + L.sscale);
  float* red = reinterpret_cast<float*>(smem + L.red);
  double* sq = reinterpret_cast<double*>(smem + L.sq);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int T = p.n_tiles;
  const int t0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * T) / gridDim.x);
  const int t1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * T) / gridDim.x);
  const int U = (t1 - t0) * nb;
  const int u0 = warp * U / kWarps, u1 = (warp + 1) * U / kWarps;
  const int n_units = u1 - u0;
  const int R = p.ring;
  uint8_t* ring = smem + L.ring + static_cast<size_t>(warp) * R * p.slot_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * R;

  // ---- weights first: they do not depend on the previous kernel
  IssueCursor cur;
  int issued = 0;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) dev::MbarInit(bars + s, 1);
    dev::MbarInitFence();
    if (n_units > 0) {
      CursorSeek(p, t0 + u0 / nb, u0 % nb, nb, cur);
      const int pre = n_units < R ? n_units : R;
      for (; issued < pre; ++issued) IssueNext(p, nb, cur, ring + issued * p.slot_bytes, bars + issued);
    }
  }
  __syncwarp();
  // norm weights of the first prologue batch: constant, so loaded before the wait
  float wpre[kBatch][8];
  if (NORM) {
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int b = warp + q * kWarps;
      if (b < nb) {
        const float4 wa = *reinterpret_cast<const float4*>(p.norm_w + b * 256 + 8 * lane);
        const float4 wb = *reinterpret_cast<const float4*>(p.norm_w + b * 256 + 8 * lane + 4);
        wpre[q][0] = wa.x; wpre[q][1] = wa.y; wpre[q][2] = wa.z; wpre[q][3] = wa.w;
        wpre[q][4] = wb.x; wpre[q][5] = wb.y; wpre[q][6] = wb.z; wpre[q][7] = wb.w;
      }
    }
  }
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();
  // residual of this thread's first epilogue row, fetched with the prologue loads
  float resid0 = 0.f;
  if (EPI == static_cast<int>(Epi::kResid) && tid < (t1 - t0) * kTile) resid0 = p.resid[t0 * kTile + tid];

  // ---- prologue: x (times the RMSNorm weight) as 4 signed 8-bit digits per
  // super-block, laid out as B fragments; 32-column sums for the Q4_K min term.
  // A warp handles super-blocks warp, warp + 8, ...; the loads of up to
  // kBatch of them are issued together, and the norm weights of the first
  // batch were loaded before the dependency wait (they are constant).
  double ssq = 0.0;
  for (int bb = 0; bb < nb; bb += kBatch * kWarps) {
    float xv[kBatch][8], wv[kBatch][8];
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int b = bb + warp + q * kWarps;
      if (b < nb) {
        const float4 xa = *reinterpret_cast<const float4*>(p.x + b * 256 + 8 * lane);
        const float4 xb = *reinterpret_cast<const float4*>(p.x + b * 256 + 8 * lane + 4);
        xv[q][0] = xa.x; xv[q][1] = xa.y; xv[q][2] = xa.z; xv[q][3] = xa.w;
        xv[q][4] = xb.x; xv[q][5] = xb.y; xv[q][6] = xb.z; xv[q][7] = xb.w;
        if (NORM) {
          if (bb == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) wv[q][i] = wpre[q][i];
          } else {
            const float4 wa = *reinterpret_cast<const float4*>(p.norm_w + b * 256 + 8 * lane);
            const float4 wb = *reinterpret_cast<const float4*>(p.norm_w + b * 256 + 8 * lane + 4);
            wv[q][0] = wa.x; wv[q][1] = wa.y; wv[q][2] = wa.z; wv[q][3] = wa.w;
            wv[q][4] = wb.x; wv[q][5] = wb.y; wv[q][6] = wb.z; wv[q][7] = wb.w;
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kBatch; ++q) {
      const int b = bb + warp + q * kWarps;
      if (b >= nb) break;
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = xv[q][i];
      if (NORM) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ssq += static_cast<double>(v[i]) * v[i];
          v[i] *= wv[q][i];
        }
      }
      PutDigits(v, b, lane, bfrag, sx, sscale);
    }
  }
  if (NORM) {
    ssq = dev::WarpSumD(ssq);
    if (lane == 0) sq[warp] = ssq;
  }
  __syncthreads();
  trace.Mark(1);  // prologue done

  // ---- stream the units
  const LaneK lk = MakeLane(lane);
  uint32_t bA[8], bB[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) bA[i] = bB[i] = 0u;
  const uint32_t lo_half = lk.g < 4 ? 1u : 0u;
  float rg = 0.f, rg8 = 0.f;
  bool timed_out = false;
  int stalled = 0;  // first unit whose copy did not arrive
  int tl = n_units > 0 ? u0 / nb : 0, b = n_units > 0 ? u0 % nb : 0;
  uint32_t type = n_units > 0 ? p.seg[SegOfTile(p, t0 + tl)].w.type : 12u;
  for (int i = 0; i < n_units; ++i) {
    const int slot = i % R;
    if (!timed_out) {
      const bool ok = dev::MbarWait(bars + slot, static_cast<uint32_t>((i / R) & 1));
      timed_out = !__all_sync(0xFFFFFFFFu, ok);
      if (timed_out) stalled = i;
    }
    if (!timed_out) {
      const uint8_t* grp = ring + static_cast<size_t>(slot) * p.slot_bytes;
      LoadB(bfrag, b, lane, lo_half, bA, bB);
      const float s = sscale[b];
      UnitOf(type, grp, bA, bB, sx + b * 8, s, lk, lane, rg, rg8);
      __syncwarp();
      if (lane == 0 && issued < n_units) {
        dev::FenceProxyAsync();
        IssueNext(p, nb, cur, ring + static_cast<size_t>(issued % R) * p.slot_bytes, bars + (issued % R));
        ++issued;
      }
    }
    if (++b == nb || i + 1 == n_units) {
      FlushPiece(red, tl + warp, lk, rg, rg8);
      if (b == nb) {
        b = 0;
        ++tl;
        if (i + 1 < n_units) type = p.seg[SegOfTile(p, t0 + tl)].w.type;
      }
    }
  }
  if (timed_out) {
    // drain copies still in flight into this warp's ring (bounded) before the
    // shared memory can be handed to another block
    if (lane == 0) {
      for (int j = stalled; j < issued; ++j) dev::MbarWait(bars + (j % R), static_cast<uint32_t>((j / R) & 1));
      if (p.err != nullptr) atomicOr(p.err, 1u);
    }
  }
  __syncthreads();
  trace.Mark(2);  // all units done

  // ---- epilogue: combine the per-warp pieces of every row in warp order
  float scale = 1.f;
  if (NORM) {
    double tot = 0.0;
    for (int w = 0; w < kWarps; ++w) tot += sq[w];
    // RMSNorm as src/kernels_gpu.cu:564-591: double sum of squares,
    // scale = float(1/sqrt(mean + eps)); applied to W (x * w) here.
    scale = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(K) + static_cast<double>(p.eps)));
  }
  const int n_rows = (t1 - t0) * kTile;
  float best_v = -FLT_MAX;
  int best_i = 0x7FFFFFFF;
  const int step = EPI == static_cast<int>(Epi::kSilu) ? 2 : 1;
  for (int lr = tid * step; lr < n_rows; lr += kThreads * step) {
    const int ti = lr / kTile, r = lr - ti * kTile;
    float v = 0.f, v2 = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int a = w * U / kWarps, e = (w + 1) * U / kWarps;
      if (a < e && a < (ti + 1) * nb && e > ti * nb) {
        v += red[(ti + w) * kTile + r];
        if (EPI == static_cast<int>(Epi::kSilu)) v2 += red[(ti + w) * kTile + r + 1];
      }
    }
    if (NORM) {
      v *= scale;
      v2 *= scale;
    }
    const int row = t0 * kTile + lr;
    if (EPI == static_cast<int>(Epi::kStore)) {
      p.out[row] = v;
    } else if (EPI == static_cast<int>(Epi::kResid)) {
      p.out[row] = (lr == tid ? resid0 : p.resid[row]) + v;
    } else if (EPI == static_cast<int>(Epi::kSilu)) {
      // rows 2i (gate) and 2i+1 (up): (g / (1 + exp(-g))) * u, as src/kernels_gpu.cu:863-869
      p.out[row >> 1] = (v / (1.0f + expf(-v))) * v2;
    } else {
      p.out[row] = v;
      if (v > best_v) {  // a thread's rows increase: strict > keeps the lowest index
        best_v = v;
        best_i = row;
      }
    }
  }

  if (EPI == static_cast<int>(Epi::kArgmax)) {
    // Ties go to the lowest index at every level (src/kernels_gpu.cu:827-859).
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
      s_bv[warp] = best_v;
      s_bi[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
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
      __syncthreads();
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
                            const int64_t* __restrict__ pos, int32_t* __restrict__ out_ids, const Trace tr) {
  dev::TraceScope trace(tr);
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();
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

template <bool NORM, int NW>
MvFn PickEpi(Epi epi) {
  switch (epi) {
    case Epi::kStore: return MatvecKernel<NORM, 0, NW>;
    case Epi::kResid: return MatvecKernel<NORM, 1, NW>;
    case Epi::kSilu: return MatvecKernel<NORM, 2, NW>;
    case Epi::kArgmax: return MatvecKernel<NORM, 3, NW>;
  }
  Throw("bad epilogue");
}

MvFn Pick(bool norm, int nw, Epi epi) {
  if (nw == 16) return norm ? PickEpi<true, 16>(epi) : PickEpi<false, 16>(epi);
  return norm ? PickEpi<true, 8>(epi) : PickEpi<false, 8>(epi);
}

}  // namespace

void PrepareMatvecKernels() {
  const Epi epis[4] = {Epi::kStore, Epi::kResid, Epi::kSilu, Epi::kArgmax};
  for (int norm = 0; norm < 2; ++norm) {
    for (int nw : {8, 16}) {
      for (Epi e : epis) {
        RPGB_CUDA(cudaFuncSetAttribute(Pick(norm != 0, nw, e), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kSmemLimit)));
      }
    }
  }
}

int MatvecGrid(int total_rows, int /*rows_per_warp*/, int num_sms) {
  const int tiles = total_rows / kTile;
  return std::max(1, std::min(tiles, num_sms));
}

void LaunchMatvec(const MvParams& in, Epi epi, int /*rows_per_warp*/, int num_sms, cudaStream_t s, bool pdl) {
  MvParams p = in;
  const int K = p.seg[0].w.cols;
  RPGB_CHECK(p.n_seg >= 1 && p.n_seg <= 3, "matvec: 1..3 segments");
  RPGB_CHECK(K % 256 == 0 && K > 0 && K <= 16384, "matvec: width %d must be a multiple of 256 up to 16384", K);
  int rows = 0, slot = 0;
  for (int i = 0; i < p.n_seg; ++i) {
    const DevMat& w = p.seg[i].w;
    RPGB_CHECK(w.cols == K, "matvec: segments differ in width");
    RPGB_CHECK(p.seg[i].out_off == rows, "matvec: segments must be contiguous");
    RPGB_CHECK(w.rows % kTile == 0, "matvec: rows %d not a multiple of %d", w.rows, kTile);
    RPGB_CHECK(MatrixTypeSupported(w.type), "matvec: unsupported type");
    slot = std::max(slot, GroupBytes(w.type));
    rows += w.rows;
  }
  RPGB_CHECK(rows == p.total_rows, "matvec: total_rows mismatch");
  if (epi == Epi::kSilu) RPGB_CHECK(rows % 2 == 0, "matvec: gate/up rows must pair up");
  const int nb = K / 256;
  p.n_tiles = rows / kTile;
  const int grid = MatvecGrid(rows, 1, num_sms);
  p.max_tiles = (p.n_tiles + grid - 1) / grid;
  p.slot_bytes = slot;
  // Long streams per block (the lm_head: ~64 tiles) are compute-bound with 8
  // warps: they get 16 warps and a deeper ring (one block per SM; the kernels
  // after the lm_head are small, so co-residency buys nothing there).
  const int nw = p.max_tiles >= 24 ? 16 : 8;
  const size_t budget = nw == 16 ? kSmemBudgetWide : kSmemBudget;
  const Layout L0 = SmemLayout(nb, 0, slot, p.max_tiles, nw);
  const size_t per_ring = static_cast<size_t>(nw) * (slot + 8);
  const int ring = static_cast<int>((budget > L0.total ? budget - L0.total : 0) / per_ring);
  p.ring = std::max(2, std::min(kMaxRing, ring));
  const Layout L = SmemLayout(nb, p.ring, slot, p.max_tiles, nw);
  RPGB_CHECK(L.total <= kSmemLimit, "matvec: shared memory plan %zu exceeds the limit", L.total);
  MvFn fn = Pick(p.norm_w != nullptr, nw, epi);
  LaunchKernelArgs(reinterpret_cast<const void*>(fn), dim3(grid), dim3(32 * nw), L.total, s, pdl, p);
  CountLaunches(1);
}

void LaunchEmbed(const DevMat& embd, const int32_t* tok, int n_tok, float* x, const int64_t* pos,
                 int32_t* out_ids, cudaStream_t s, bool pdl, const Trace& trace) {
  RPGB_CHECK(n_tok > 0 && n_tok < 65536, "embed: bad token count %d", n_tok);
  const dim3 grid((embd.cols + 255) / 256, n_tok);
  LaunchKernelArgs(reinterpret_cast<const void*>(EmbedKernel), grid, dim3(256), 0, s, pdl, embd, tok, x, pos,
                   out_ids, trace);
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
