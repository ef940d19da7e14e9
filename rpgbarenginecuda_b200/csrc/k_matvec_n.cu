// k_matvec_n.cu -- Q4_K / Q6_K matmul for a few tokens (2 .. 15 activation
// rows) on the integer tensor-core unit of the decode matvec.
//
// Replaces the reference's PickShape tiles for small n (MatMulQ4KKernel /
// MatMulQ6KKernel with TILE = 2..8, src/kernels_gpu.cu:101-106, 325-494):
// OUT[t, r] = sum_c W[r, c] X[t, c].
//
// The weights stream once per pass from HBM exactly as in the decode matvec
// (persistent block per SM, per-warp rings of 1-D TMA copies, one (16-row
// tile, super-block) unit per slot); every unit that lands in shared memory
// is applied to every token of the pass: each token's x is split into four
// 8-bit digits per super-block (the B fragments of mma.sync.m16n8k32) in the
// prologue, and UnitQ4K / UnitQ6K run once per token on the same slot.  A
// pass takes as many tokens as the shared memory holds (their digits: 1 KiB
// per super-block per token); longer inputs take several passes over the
// weights.  Per-warp row pieces are combined in a fixed order (deterministic).
#include <algorithm>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "launch.h"
#include "mv_dev.cuh"

namespace rpgb {
namespace {

using namespace mv;

constexpr int kPassMax = 4;  // tokens per pass (registers: two partial sums per token)
constexpr int kMaxRingN = 6;
constexpr size_t kSmemLimitN = 200 * 1024;

struct NLayout {
  size_t ring, bfrag, sx, sscale, red, bars, total;
};

// per token: digits (1 KiB per super-block), 32-column sums, scale, row pieces
__host__ __device__ inline NLayout NSmem(int nb, int ring, int slot, int max_tiles, int nw, int tp) {
  NLayout l;
  l.ring = 0;
  l.bfrag = static_cast<size_t>(nw) * ring * slot;
  l.sx = l.bfrag + static_cast<size_t>(tp) * nb * 1024;
  l.sscale = l.sx + static_cast<size_t>(tp) * nb * 32;
  l.red = l.sscale + static_cast<size_t>(tp) * nb * 4;
  l.bars = l.red + static_cast<size_t>(tp) * (max_tiles + nw) * kTile * 4;
  l.bars = (l.bars + 7) & ~static_cast<size_t>(7);
  l.total = l.bars + static_cast<size_t>(nw) * ring * 8;
  return l;
}

template <int NW>
__global__ void __launch_bounds__(32 * NW, 1) MatvecTokensKernel(const MvnParams p) {
  constexpr int kThreads = 32 * NW;
  extern __shared__ __align__(128) uint8_t smem[];
  const int K = p.w.cols, nb = K >> 8;
  const NLayout L = NSmem(nb, p.ring, p.slot_bytes, p.max_tiles, NW, p.tp);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int T = p.w.rows / kTile;
  const int t0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * T) / gridDim.x);
  const int t1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * T) / gridDim.x);
  const int U = (t1 - t0) * nb;
  const int u0 = warp * U / NW, u1 = (warp + 1) * U / NW;
  const int n_units = u1 - u0;
  const int n_pass = (p.n_tok + p.tp - 1) / p.tp;
  const int total = n_units * n_pass;  // the warp's units over all passes
  const int R = p.ring;
  const uint32_t gbytes = static_cast<uint32_t>(dev::GroupBytesOf(p.w.type));
  uint8_t* ring = smem + L.ring + static_cast<size_t>(warp) * R * p.slot_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars) + warp * R;
  // block groups of the matrix are contiguous in tile-major order: the
  // warp's units are one contiguous byte range, re-read by every pass
  const uint8_t* src0 = p.w.q + (static_cast<int64_t>(t0) * nb + u0) * gbytes;

  // ---- weights first: they do not depend on the previous kernel
  int issued = 0;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) dev::MbarInit(bars + s, 1);
    dev::MbarInitFence();
    const int pre = total < R ? total : R;
    for (; issued < pre; ++issued) {
      dev::MbarExpectTx(bars + issued, gbytes);
      dev::BulkG2S(ring + issued * p.slot_bytes, src0 + static_cast<int64_t>(issued % n_units) * gbytes, gbytes,
                   bars + issued);
    }
  }
  __syncwarp();
  dev::GridLaunchDependents();
  dev::GridWait();

  const LaneK lk = MakeLane(lane);
  const uint32_t lo_half = lk.g < 4 ? 1u : 0u;
  bool timed_out = false;
  int stalled = 0;
  for (int pass = 0; pass < n_pass; ++pass) {
    const int tok0 = pass * p.tp;
    const int nt = p.n_tok - tok0 < p.tp ? p.n_tok - tok0 : p.tp;
    // ---- prologue: digits of this pass's tokens
    for (int j = warp; j < nt * nb; j += NW) {
      const int t = j / nb, b = j - t * nb;
      const float* xr = p.x + static_cast<int64_t>(tok0 + t) * p.ldx + b * 256 + 8 * lane;
      const float4 xa = *reinterpret_cast<const float4*>(xr);
      const float4 xb = *reinterpret_cast<const float4*>(xr + 4);
      const float v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
      PutDigits(v, b, lane, smem + L.bfrag + static_cast<size_t>(t) * nb * 1024,
                reinterpret_cast<float*>(smem + L.sx) + t * nb * 8, reinterpret_cast<float*>(smem + L.sscale) + t * nb);
    }
    __syncthreads();

    // ---- units: each landed slot serves every token of the pass
    float rg[kPassMax], rg8[kPassMax];
#pragma unroll
    for (int t = 0; t < kPassMax; ++t) rg[t] = rg8[t] = 0.f;
    int tl = n_units > 0 ? u0 / nb : 0, b = n_units > 0 ? u0 % nb : 0;
    for (int j = 0; j < n_units; ++j) {
      const int i = pass * n_units + j;
      const int slot = i % R;
      if (!timed_out) {
        const bool ok = dev::MbarWait(bars + slot, static_cast<uint32_t>((i / R) & 1));
        timed_out = !__all_sync(0xFFFFFFFFu, ok);
        if (timed_out) stalled = i;
      }
      if (!timed_out) {
        const uint8_t* grp = ring + static_cast<size_t>(slot) * p.slot_bytes;
#pragma unroll
        for (int t = 0; t < kPassMax; ++t) {
          if (t < nt) {
            uint32_t bA[8], bB[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) bA[q] = bB[q] = 0u;
            LoadB(smem + L.bfrag + static_cast<size_t>(t) * nb * 1024, b, lane, lo_half, bA, bB);
            const float s = reinterpret_cast<const float*>(smem + L.sscale)[t * nb + b];
            UnitOf(p.w.type, grp, bA, bB, reinterpret_cast<const float*>(smem + L.sx) + (t * nb + b) * 8, s, lk,
                   lane, rg[t], rg8[t]);
          }
        }
        __syncwarp();
        if (lane == 0 && issued < total) {
          dev::FenceProxyAsync();
          const int s2 = issued % R;
          dev::MbarExpectTx(bars + s2, gbytes);
          dev::BulkG2S(ring + s2 * p.slot_bytes, src0 + static_cast<int64_t>(issued % n_units) * gbytes, gbytes,
                       bars + s2);
          ++issued;
        }
      }
      if (++b == nb || j + 1 == n_units) {
#pragma unroll
        for (int t = 0; t < kPassMax; ++t) {
          if (t < nt) {
            float* red = reinterpret_cast<float*>(smem + L.red) + static_cast<size_t>(t) * (p.max_tiles + NW) * kTile;
            FlushPiece(red, tl + warp, lk, rg[t], rg8[t]);
          }
        }
        if (b == nb) {
          b = 0;
          ++tl;
        }
      }
    }
    __syncthreads();

    // ---- epilogue: per token, the warps' pieces of every row in warp order
    const int n_rows = (t1 - t0) * kTile;
    const int step = p.epi == Epi::kSilu ? 2 : 1;  // gate/up: one thread per row pair
    const int n_items = n_rows / step;
    for (int k = tid; k < nt * n_items; k += kThreads) {
      const int t = k / n_items, lr = (k - t * n_items) * step;
      const int ti = lr / kTile, r = lr - ti * kTile;
      const float* red = reinterpret_cast<const float*>(smem + L.red) + static_cast<size_t>(t) * (p.max_tiles + NW) * kTile;
      float v = 0.f, v2 = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const int a = w * U / NW, e = (w + 1) * U / NW;
        if (a < e && a < (ti + 1) * nb && e > ti * nb) {
          v += red[(ti + w) * kTile + r];
          if (step == 2) v2 += red[(ti + w) * kTile + r + 1];
        }
      }
      const int row = t0 * kTile + lr;
      float* o = p.out + static_cast<int64_t>(tok0 + t) * p.ldo;
      if (p.epi == Epi::kStore) {
        o[p.out_off + row] = v;
      } else if (p.epi == Epi::kResid) {
        o[row] += v;
      } else {
        // rows 2i (gate) and 2i+1 (up): (g / (1 + exp(-g))) * u, as src/kernels_gpu.cu:863-869
        o[row >> 1] = (v / (1.0f + expf(-v))) * v2;
      }
    }
    __syncthreads();  // the next pass reuses the digits and the pieces
  }
  if (timed_out && lane == 0) {
    // copies still in flight into this warp's ring land (bounded) before exit
    for (int j = stalled; j < issued; ++j) dev::MbarWait(bars + (j % R), static_cast<uint32_t>((j / R) & 1));
    if (p.err != nullptr) atomicOr(p.err, 1u);
  }
}

using MvnFn = void (*)(const MvnParams);

}  // namespace

void PrepareMatvecTokensKernels() {
  for (MvnFn f : {MatvecTokensKernel<8>, MatvecTokensKernel<16>}) {
    RPGB_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimitN)));
  }
}

void LaunchMatvecTokens(const MvnParams& in, int num_sms, cudaStream_t s, bool pdl) {
  MvnParams p = in;
  const DevMat& w = p.w;
  RPGB_CHECK(MatrixTypeSupported(w.type), "matvec: unsupported type");
  RPGB_CHECK(w.cols % 256 == 0 && w.cols > 0 && w.cols <= 16384, "matvec: width %d must be a multiple of 256",
             w.cols);
  RPGB_CHECK(w.rows % kTile == 0, "matvec: rows %d not a multiple of %d", w.rows, kTile);
  RPGB_CHECK(p.epi == Epi::kStore || p.epi == Epi::kResid || p.epi == Epi::kSilu, "matvec: unsupported epilogue");
  const int out_cols = p.epi == Epi::kSilu ? w.rows / 2 : p.out_off + w.rows;
  RPGB_CHECK(p.n_tok >= 1 && p.ldx >= w.cols && p.ldo >= out_cols, "matvec: bad token rows");
  RPGB_CHECK(p.ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0, "matvec: x rows must be 16-byte aligned");
  const int nb = w.cols / 256;
  const int tiles = w.rows / kTile;
  const int grid = std::max(1, std::min(tiles, num_sms));
  p.max_tiles = (tiles + grid - 1) / grid;
  p.slot_bytes = GroupBytes(w.type);
  const int nw = p.max_tiles >= 24 ? 16 : 8;
  // tokens per pass: as many as the shared memory holds (at least one), with
  // a ring of at least three slots per warp
  const size_t ring_min = static_cast<size_t>(nw) * 3 * (p.slot_bytes + 8);
  int tp = std::min(kPassMax, p.n_tok);
  while (tp > 1 && NSmem(nb, 3, p.slot_bytes, p.max_tiles, nw, tp).total > kSmemLimitN) --tp;
  const size_t fixed = NSmem(nb, 0, p.slot_bytes, p.max_tiles, nw, tp).total;
  RPGB_CHECK(fixed + ring_min <= kSmemLimitN, "matvec: shared memory plan does not fit");
  const int ring = static_cast<int>((kSmemLimitN - fixed) / (static_cast<size_t>(nw) * (p.slot_bytes + 8)));
  p.ring = std::max(3, std::min(kMaxRingN, ring));
  p.tp = tp;
  const NLayout L = NSmem(nb, p.ring, p.slot_bytes, p.max_tiles, nw, tp);
  const MvnFn fn = nw == 16 ? MatvecTokensKernel<16> : MatvecTokensKernel<8>;
  LaunchKernelArgs(reinterpret_cast<const void*>(fn), dim3(grid), dim3(32 * nw), L.total, s, pdl, p);
  CountLaunches(1);
}

}  // namespace rpgb
