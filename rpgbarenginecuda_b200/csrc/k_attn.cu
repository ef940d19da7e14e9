// k_attn.cu -- GQA attention over the fp16 KV cache, plus the prefill helpers.
//
// Replaces AttentionFromCacheKernel (src/kernels_gpu.cu:737-823), KvWriteKernel
// (708-727), RopeKernel (598-621) and the per-head RmsNorm launches of
// GpuForwardLayer (src/qwen3_gpu.cu:74-94).
//
// One block owns (position split s, KV head h, query t) and all G query heads
// of that group, so each K/V row is read once per group instead of once per
// query head.  Positions are processed 128 at a time with an online softmax;
// with n_splits > 1 (decode) every split writes (m, l, acc) and the last block
// of a head to finish merges them (ticket counter, no spin-wait).
//
// Cache layout is the reference's: [layer][kv_head][max_seq][128] fp16, RNE
// rounding (__float2half_rn, src/kernels_gpu.cu:725).
#include <cfloat>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "launch.h"

namespace rpgb {
namespace {

constexpr int D = 128;

template <int G>
__device__ __forceinline__ void BlockMaxG(float (&v)[G], float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    v[g] = dev::WarpMax(v[g]);
    if (lane == 0) sh[warp * G + g] = v[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) v[g] = fmaxf(fmaxf(sh[g], sh[G + g]), fmaxf(sh[2 * G + g], sh[3 * G + g]));
}

template <int G>
__device__ __forceinline__ void BlockSumG(double (&v)[G], double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    v[g] = dev::WarpSumD(v[g]);
    if (lane == 0) sh[warp * G + g] = v[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) v[g] = ((sh[g] + sh[G + g]) + sh[2 * G + g]) + sh[3 * G + g];
}

// In-place per-head RMSNorm + rotate-half RoPE of N vectors held one element
// per thread (thread = dimension); vector i is scaled by weight row w[i].
template <int N>
__device__ __forceinline__ void NormRopeW(float (&v)[N], const float* const (&w)[N], float eps,
                                          const float* __restrict__ rope_row, float (*buf)[D], double* dsh) {
  const int tid = threadIdx.x;
  double ss[N];
#pragma unroll
  for (int g = 0; g < N; ++g) ss[g] = static_cast<double>(v[g]) * v[g];
  BlockSumG<N>(ss, dsh);
#pragma unroll
  for (int g = 0; g < N; ++g) {
    const float scale = static_cast<float>(1.0 / sqrt(ss[g] / static_cast<double>(D) + static_cast<double>(eps)));
    buf[g][tid] = v[g] * scale * w[g][tid];
  }
  __syncthreads();
  if (tid < D / 2) {
    const float c = rope_row[tid], sn = rope_row[D / 2 + tid];
#pragma unroll
    for (int g = 0; g < N; ++g) {
      const float a = buf[g][tid], b = buf[g][tid + D / 2];
      buf[g][tid] = a * c - b * sn;
      buf[g][tid + D / 2] = b * c + a * sn;
    }
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < N; ++g) v[g] = buf[g][tid];
}

template <int G>
__device__ __forceinline__ void NormRope(float (&v)[G], const float* __restrict__ w, float eps,
                                         const float* __restrict__ rope_row, float (*buf)[D], double* dsh) {
  const float* ws[G];
#pragma unroll
  for (int g = 0; g < G; ++g) ws[g] = w;
  NormRopeW<G>(v, ws, eps, rope_row, buf, dsh);
}

// Positions per split at least this many: short contexts run one split per
// KV head and skip the merge.
constexpr int64_t kMinSplit = 256;
constexpr int kMaxSplits = 64;

// Positions of the split starting at p0: min(128, L - p0).
__device__ __forceinline__ int64_t p1_of(int64_t p0, int64_t L) {
  return L - p0 < kAttnSplitPositions ? L - p0 : kAttnSplitPositions;
}

template <int G>
__global__ void __launch_bounds__(128) AttnKernel(const AttnParams p) {
  __shared__ __align__(16) float qs[G + 1][D];  // G query vectors (+ the new key while fusing)
  __shared__ float sc[G][128];
  __shared__ __align__(16) float vred[4][G][D];
  __shared__ double dsh[4 * (G + 1)];
  __shared__ float fsh[4 * G];
  __shared__ float s_wm[kMaxSplits][G];
  __shared__ double s_wl[kMaxSplits][G];
  __shared__ int s_last;

  dev::TraceScope trace(p.trace);
  const int s = blockIdx.x, h = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // The position counter of this step was written before the step started
  // (previous graph launch / host copy), so it may be read before the wait.
  const int64_t pos = *p.pos + t;
  const int64_t L = pos + 1;
  int64_t chunk = (L + p.n_splits - 1) / p.n_splits;
  if (chunk < kMinSplit) chunk = kMinSplit;
  const int active = static_cast<int>((L + chunk - 1) / chunk);
  if (s >= active) return;  // nothing to do at this length (no memory touched)
  const int64_t p0 = static_cast<int64_t>(s) * chunk;
  const int64_t p1 = p0 + chunk < L ? p0 + chunk : L;
  const int q_dim = p.n_heads * D;
  __half* kbase = p.kc + static_cast<int64_t>(h) * p.max_seq * D;
  __half* vbase = p.vc + static_cast<int64_t>(h) * p.max_seq * D;

  // Rows before `pos` were written by earlier steps: pull them toward L2 while
  // the previous kernel (the q/k/v projection) is still running.
  if (p.fused && tid == 0) {
    const int64_t pe = p1 < pos ? p1 : pos;
    if (pe > p0) {
      const uint32_t bytes = static_cast<uint32_t>((pe - p0) * D * 2);
      dev::PrefetchL2(kbase + p0 * D, bytes);
      dev::PrefetchL2(vbase + p0 * D, bytes);
    }
  }
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();

  // ---- the G query vectors of this group
  {
    float v[G];
#pragma unroll
    for (int g = 0; g < G; ++g) v[g] = p.q[static_cast<int64_t>(t) * p.q_stride + (h * G + g) * D + tid];
    if (p.fused) {
      // q heads and the new key normalised and rotated together (one block sum)
      float vk[G + 1];
      const float* ws[G + 1];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        vk[g] = v[g];
        ws[g] = p.q_norm;
      }
      vk[G] = p.k_raw[h * D + tid];
      ws[G] = p.k_norm;
      NormRopeW<G + 1>(vk, ws, p.eps, p.rope + pos * D, qs, dsh);
      if (p0 <= pos && pos < p1) {
        // This split owns the new position: write its K/V (fp16, RNE) first.
        kbase[pos * D + tid] = __float2half_rn(vk[G]);
        vbase[pos * D + tid] = __float2half_rn(p.v_raw[h * D + tid]);
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) qs[g][tid] = v[g];
    }
  }
  __syncthreads();

  float m[G];
  double l[G];
  float acc[G][4];  // dims 4*lane .. 4*lane+3, positions of this warp
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  }

  for (int64_t c0 = p0; c0 < p1; c0 += 128) {
    const int64_t pp = c0 + tid;
    float sg[G];
    if (pp < p1) {
      // one position per thread: 256 B of K, dot in ascending d (src/kernels_gpu.cu:772-777)
      const uint4* kr = reinterpret_cast<const uint4*>(kbase + pp * D);
      float dot[G];
#pragma unroll
      for (int g = 0; g < G; ++g) dot[g] = 0.f;
#pragma unroll 4
      for (int i = 0; i < D / 8; ++i) {
        const uint4 kw = kr[i];
        const __half2* h2 = reinterpret_cast<const __half2*>(&kw);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(h2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int e = 0; e < 8; ++e) dot[g] = fmaf(qs[g][i * 8 + e], kf[e], dot[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) sg[g] = dot[g] * p.scale;
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) sg[g] = -INFINITY;
    }
    float cm[G];
#pragma unroll
    for (int g = 0; g < G; ++g) cm[g] = sg[g];
    BlockMaxG<G>(cm, fsh);
    double cs[G];
    float alpha[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float nm = fmaxf(m[g], cm[g]);
      const float e = pp < p1 ? expf(sg[g] - nm) : 0.f;
      sc[g][tid] = e;
      cs[g] = static_cast<double>(e);
      alpha[g] = m[g] == -INFINITY ? 0.f : expf(m[g] - nm);
      m[g] = nm;
    }
    BlockSumG<G>(cs, dsh);  // its barriers also publish sc[] to all warps
    const int nv = static_cast<int>(p1 - c0 < 128 ? p1 - c0 : 128);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      l[g] = l[g] * static_cast<double>(alpha[g]) + cs[g];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] *= alpha[g];
    }
    // V: warp w takes positions w, w+4, ...; lane holds 4 consecutive dims (8 B loads)
    const __half* vr = vbase + c0 * D + 4 * lane;
#pragma unroll 4
    for (int j = warp; j < nv; j += 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(vr + static_cast<int64_t>(j) * D);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float e = sc[g][j];
        acc[g][0] = fmaf(e, a.x, acc[g][0]);
        acc[g][1] = fmaf(e, a.y, acc[g][1]);
        acc[g][2] = fmaf(e, b.x, acc[g][2]);
        acc[g][3] = fmaf(e, b.y, acc[g][3]);
      }
    }
    __syncthreads();
  }

  // combine the 4 warps' partial V sums: thread tid ends up with dim tid
#pragma unroll
  for (int g = 0; g < G; ++g) {
    *reinterpret_cast<float4*>(&vred[warp][g][4 * lane]) = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  }
  __syncthreads();
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = ((vred[0][g][tid] + vred[1][g][tid]) + vred[2][g][tid]) + vred[3][g][tid];

  if (active == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      p.out[static_cast<int64_t>(t) * q_dim + (h * G + g) * D + tid] = o[g] * static_cast<float>(1.0 / l[g]);
    }
    return;
  }

  // ---- split-K: publish (m, l, acc) and let the last block of this head merge
  constexpr int kRec = D + 2;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* rec = p.part + (static_cast<int64_t>(h * p.n_splits + s) * G + g) * kRec;
    if (tid == 0) {
      rec[0] = m[g];
      rec[1] = static_cast<float>(l[g]);
    }
    rec[2 + tid] = o[g];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned tk = atomicAdd(p.ticket + h, 1u);
    s_last = tk == static_cast<unsigned>(active - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // split maxima and masses, one thread per split (loads in parallel)
  if (tid < active) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float* rec = p.part + (static_cast<int64_t>(h * p.n_splits + tid) * G + g) * kRec;
      s_wm[tid][g] = __ldcg(rec);
      s_wl[tid][g] = static_cast<double>(__ldcg(rec + 1));
    }
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
    for (int sp = 0; sp < active; ++sp) M = fmaxf(M, s_wm[sp][g]);
    double den = 0.0;
    float num = 0.f;
#pragma unroll 4
    for (int sp = 0; sp < active; ++sp) {
      const float ms = s_wm[sp][g];
      const float w = ms == -INFINITY ? 0.f : expf(ms - M);
      den += static_cast<double>(w) * s_wl[sp][g];
      num = fmaf(w, __ldcg(p.part + (static_cast<int64_t>(h * p.n_splits + sp) * G + g) * kRec + 2 + tid), num);
    }
    p.out[(h * G + g) * D + tid] = num * static_cast<float>(1.0 / den);
  }
  if (tid == 0) p.ticket[h] = 0u;
}

}  // namespace

namespace {

// ---- decode attention with the split's K/V staged in shared memory
//
// Block (split s, KV head h): positions [128 s, min(128 s + 128, L)).  Rows
// below the current position were written by earlier steps, so thread 0
// requests them with two 1-D TMA bulk copies before griddepcontrol.wait; the
// current row is normalised, rotated and written by this kernel itself.
// Scores: thread = position, the 16-byte chunks of the key row visited in a
// per-thread rotated order (conflict-free shared loads).  V: thread = dimension.
constexpr int kSP = kAttnSplitPositions;
constexpr size_t kAttnDynSmem = 2 * static_cast<size_t>(kSP) * D * sizeof(__half) + 16;

template <int G>
__global__ void __launch_bounds__(128) AttnDecodeKernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __half* Ks = reinterpret_cast<__half*>(dsm);
  __half* Vs = Ks + kSP * D;
  uint64_t* bar = reinterpret_cast<uint64_t*>(Vs + kSP * D);
  __shared__ __align__(16) float qs[G + 1][D];
  __shared__ float sc[G][kSP];
  __shared__ double dsh[4 * (G + 1)];
  __shared__ float fsh[4 * G];
  __shared__ float s_wm[kMaxSplits][G];
  __shared__ double s_wl[kMaxSplits][G];
  __shared__ int s_last;

  dev::TraceScope trace(p.trace);
  const int s = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x;
  // The position counter of this step was written before the step started
  // (previous graph launch / host copy), so it may be read before the wait.
  const int64_t pos = *p.pos;
  const int64_t L = pos + 1;
  const int active = static_cast<int>((L + kSP - 1) / kSP);
  if (s >= active) return;  // nothing to do at this length (no memory touched)
  const int64_t p0 = static_cast<int64_t>(s) * kSP;
  const int n = static_cast<int>(p1_of(p0, L));
  const int q_dim = p.n_heads * D;
  __half* kbase = p.kc + static_cast<int64_t>(h) * p.max_seq * D;
  __half* vbase = p.vc + static_cast<int64_t>(h) * p.max_seq * D;
  const int n_old = static_cast<int>(pos - p0 < n ? pos - p0 : n);  // rows already in the cache

  if (tid == 0) {
    dev::MbarInit(bar, 1);
    dev::MbarInitFence();
    if (n_old > 0) {
      const uint32_t bytes = static_cast<uint32_t>(n_old) * D * 2;
      dev::MbarExpectTx(bar, 2 * bytes);
      dev::BulkG2S(Ks, kbase + p0 * D, bytes, bar);
      dev::BulkG2S(Vs, vbase + p0 * D, bytes, bar);
    }
  }
  __syncthreads();
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();

  // ---- q heads and the new key: RMSNorm + RoPE in one pass
  {
    float vk[G + 1];
    const float* ws[G + 1];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      vk[g] = p.q[(h * G + g) * D + tid];
      ws[g] = p.q_norm;
    }
    vk[G] = p.k_raw[h * D + tid];
    ws[G] = p.k_norm;
    const float vv = p.v_raw[h * D + tid];
    NormRopeW<G + 1>(vk, ws, p.eps, p.rope + pos * D, qs, dsh);
    if (n_old < n) {  // this split owns the new position (fp16, RNE)
      const __half kh = __float2half_rn(vk[G]), vh = __float2half_rn(vv);
      kbase[pos * D + tid] = kh;
      vbase[pos * D + tid] = vh;
      Ks[n_old * D + tid] = kh;
      Vs[n_old * D + tid] = vh;
    }
  }
  if (n_old > 0) {
    bool ok = dev::MbarWait(bar, 0);
    if (!ok) {
      if (tid == 0 && p.err != nullptr) atomicOr(p.err, 2u);
      dev::MbarWait(bar, 0);  // give the copy one more bounded chance before the buffer is read
    }
  }
  __syncthreads();

  // ---- scores: thread = position
  float sg[G];
  if (tid < n) {
    float dot[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dot[g] = 0.f;
    const uint4* kr = reinterpret_cast<const uint4*>(Ks + tid * D);
#pragma unroll 4
    for (int i = 0; i < D / 8; ++i) {
      const int c = (i + tid) & (D / 8 - 1);
      const uint4 kw = kr[c];
      const __half2* h2 = reinterpret_cast<const __half2*>(&kw);
      float kf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(h2[e]);
        kf[2 * e] = f.x;
        kf[2 * e + 1] = f.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 qa = *reinterpret_cast<const float4*>(&qs[g][c * 8]);
        const float4 qb = *reinterpret_cast<const float4*>(&qs[g][c * 8 + 4]);
        dot[g] = fmaf(qa.x, kf[0], dot[g]);
        dot[g] = fmaf(qa.y, kf[1], dot[g]);
        dot[g] = fmaf(qa.z, kf[2], dot[g]);
        dot[g] = fmaf(qa.w, kf[3], dot[g]);
        dot[g] = fmaf(qb.x, kf[4], dot[g]);
        dot[g] = fmaf(qb.y, kf[5], dot[g]);
        dot[g] = fmaf(qb.z, kf[6], dot[g]);
        dot[g] = fmaf(qb.w, kf[7], dot[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sg[g] = dot[g] * p.scale;
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) sg[g] = -INFINITY;
  }
  float m[G];
#pragma unroll
  for (int g = 0; g < G; ++g) m[g] = sg[g];
  BlockMaxG<G>(m, fsh);
  double l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float e = tid < n ? expf(sg[g] - m[g]) : 0.f;
    sc[g][tid] = e;
    l[g] = static_cast<double>(e);
  }
  BlockSumG<G>(l, dsh);  // its barriers also publish sc[] to all threads

  // ---- V: thread = dimension, two accumulators per head
  float o[G];
  {
    float a0[G], a1[G];
#pragma unroll
    for (int g = 0; g < G; ++g) a0[g] = a1[g] = 0.f;
    int j = 0;
    for (; j + 1 < n; j += 2) {
      const float v0 = __half2float(Vs[j * D + tid]), v1 = __half2float(Vs[(j + 1) * D + tid]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        a0[g] = fmaf(sc[g][j], v0, a0[g]);
        a1[g] = fmaf(sc[g][j + 1], v1, a1[g]);
      }
    }
    if (j < n) {
      const float v0 = __half2float(Vs[j * D + tid]);
#pragma unroll
      for (int g = 0; g < G; ++g) a0[g] = fmaf(sc[g][j], v0, a0[g]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] = a0[g] + a1[g];
  }

  if (active == 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) p.out[(h * G + g) * D + tid] = o[g] * static_cast<float>(1.0 / l[g]);
    return;
  }

  // ---- split-K: publish (m, l, acc) and let the last block of this head merge
  constexpr int kRec = D + 2;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* rec = p.part + (static_cast<int64_t>(h * p.n_splits + s) * G + g) * kRec;
    if (tid == 0) {
      rec[0] = m[g];
      rec[1] = static_cast<float>(l[g]);
    }
    rec[2 + tid] = o[g];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned tk = atomicAdd(p.ticket + h, 1u);
    s_last = tk == static_cast<unsigned>(active - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < active) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float* rec = p.part + (static_cast<int64_t>(h * p.n_splits + tid) * G + g) * kRec;
      s_wm[tid][g] = __ldcg(rec);
      s_wl[tid][g] = static_cast<double>(__ldcg(rec + 1));
    }
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = -INFINITY;
    for (int sp = 0; sp < active; ++sp) M = fmaxf(M, s_wm[sp][g]);
    double den = 0.0;
    float num = 0.f;
#pragma unroll 4
    for (int sp = 0; sp < active; ++sp) {
      const float ms = s_wm[sp][g];
      const float w = ms == -INFINITY ? 0.f : expf(ms - M);
      den += static_cast<double>(w) * s_wl[sp][g];
      num = fmaf(w, __ldcg(p.part + (static_cast<int64_t>(h * p.n_splits + sp) * G + g) * kRec + 2 + tid), num);
    }
    p.out[(h * G + g) * D + tid] = num * static_cast<float>(1.0 / den);
  }
  if (tid == 0) p.ticket[h] = 0u;
}

// Prefill: per token, q heads -> q_out (normalised + rotated), k heads -> cache
// (normalised + rotated, fp16), v heads -> cache (fp16).
__global__ void __launch_bounds__(128) QkRopeKvKernel(const float* __restrict__ qkv, int q_dim, int kv_dim,
                                                      const float* __restrict__ q_norm,
                                                      const float* __restrict__ k_norm,
                                                      const float* __restrict__ rope, float eps,
                                                      const int64_t* __restrict__ pos0, __half* kc, __half* vc,
                                                      int32_t max_seq, int n_heads, int n_kv,
                                                      float* __restrict__ q_out) {
  __shared__ __align__(16) float buf[1][D];
  __shared__ double dsh[4];
  const int t = blockIdx.x, tid = threadIdx.x;
  const int64_t pos = *pos0 + t;
  const float* row = qkv + static_cast<int64_t>(t) * (q_dim + 2 * kv_dim);
  const float* rr = rope + pos * D;
  for (int hq = 0; hq < n_heads; ++hq) {
    float v[1] = {row[hq * D + tid]};
    NormRope<1>(v, q_norm, eps, rr, buf, dsh);
    q_out[static_cast<int64_t>(t) * q_dim + hq * D + tid] = v[0];
  }
  for (int hk = 0; hk < n_kv; ++hk) {
    float v[1] = {row[q_dim + hk * D + tid]};
    NormRope<1>(v, k_norm, eps, rr, buf, dsh);
    const int64_t off = (static_cast<int64_t>(hk) * max_seq + pos) * D + tid;
    kc[off] = __float2half_rn(v[0]);
    vc[off] = __float2half_rn(row[q_dim + kv_dim + hk * D + tid]);
  }
}

__global__ void __launch_bounds__(256) RmsNormRowsKernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         int n, float eps, float* __restrict__ out) {
  __shared__ double dsh[32];
  const float* xr = x + static_cast<int64_t>(blockIdx.x) * n;
  float* orow = out + static_cast<int64_t>(blockIdx.x) * n;
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double v = static_cast<double>(xr[i]);
    ss += v * v;
  }
  const double tot = dev::BlockSumD(ss, dsh);
  const float scale = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(n) + static_cast<double>(eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) orow[i] = xr[i] * scale * w[i];
}

}  // namespace

size_t AttentionPartialFloats(int n_kv, int group, int n_splits) {
  return static_cast<size_t>(n_kv) * n_splits * group * (D + 2);
}

void PrepareAttentionKernels() {
  const void* fns[4] = {reinterpret_cast<const void*>(AttnDecodeKernel<1>),
                        reinterpret_cast<const void*>(AttnDecodeKernel<2>),
                        reinterpret_cast<const void*>(AttnDecodeKernel<4>),
                        reinterpret_cast<const void*>(AttnDecodeKernel<8>)};
  for (const void* f : fns) {
    RPGB_CUDA(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kAttnDynSmem)));
  }
}

void LaunchAttention(const AttnParams& p, int n_queries, cudaStream_t s, bool pdl) {
  RPGB_CHECK(n_queries >= 1 && n_queries < 65536, "attention: bad query count %d", n_queries);
  RPGB_CHECK(p.n_splits >= 1 && (p.n_splits == 1 || n_queries == 1), "attention: split-K is decode only");
  RPGB_CHECK(p.n_heads % p.n_kv == 0, "attention: bad head counts");
  RPGB_CHECK(p.n_splits <= kMaxSplits, "attention: %d splits exceed %d", p.n_splits, kMaxSplits);
  const int G = p.n_heads / p.n_kv;
  const void* fn = nullptr;
  if (p.fused) {
    RPGB_CHECK(n_queries == 1, "attention: the fused decode kernel takes one query");
    RPGB_CHECK(static_cast<int64_t>(p.n_splits) * kSP >= p.max_seq, "attention: %d splits cannot cover %d positions",
               p.n_splits, p.max_seq);
    switch (G) {
      case 1: fn = reinterpret_cast<const void*>(AttnDecodeKernel<1>); break;
      case 2: fn = reinterpret_cast<const void*>(AttnDecodeKernel<2>); break;
      case 4: fn = reinterpret_cast<const void*>(AttnDecodeKernel<4>); break;
      case 8: fn = reinterpret_cast<const void*>(AttnDecodeKernel<8>); break;
      default: Throw("attention: GQA group %d is not supported (1, 2, 4, 8)", G);
    }
    LaunchKernelArgs(fn, dim3(p.n_splits, p.n_kv), dim3(128), kAttnDynSmem, s, pdl, p);
    CountLaunches(1);
    return;
  }
  const dim3 grid(p.n_splits, p.n_kv, n_queries);
  switch (G) {
    case 1: fn = reinterpret_cast<const void*>(AttnKernel<1>); break;
    case 2: fn = reinterpret_cast<const void*>(AttnKernel<2>); break;
    case 4: fn = reinterpret_cast<const void*>(AttnKernel<4>); break;
    case 8: fn = reinterpret_cast<const void*>(AttnKernel<8>); break;
    default: Throw("attention: GQA group %d is not supported (1, 2, 4, 8)", G);
  }
  LaunchKernelArgs(fn, grid, dim3(128), 0, s, pdl, p);
  CountLaunches(1);
}

void LaunchQkRopeKv(const float* qkv, int n_tok, int q_dim, int kv_dim, const float* q_norm, const float* k_norm,
                    const float* rope, float eps, const int64_t* pos0, __half* kc, __half* vc, int32_t max_seq,
                    int n_heads, int n_kv, float* q_out, cudaStream_t s) {
  RPGB_CHECK(n_tok > 0, "qk_rope: empty");
  QkRopeKvKernel<<<n_tok, 128, 0, s>>>(qkv, q_dim, kv_dim, q_norm, k_norm, rope, eps, pos0, kc, vc, max_seq,
                                       n_heads, n_kv, q_out);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

void LaunchRmsNormRows(const float* x, const float* w, int n_rows, int n, float eps, float* out, cudaStream_t s) {
  RPGB_CHECK(n_rows > 0 && n > 0, "rmsnorm: empty");
  RmsNormRowsKernel<<<n_rows, 256, 0, s>>>(x, w, n, eps, out);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

}  // namespace rpgb
