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
constexpr int kMaxSplits = kMaxAttnSplits;


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

// ---- decode attention: one thread-block cluster per KV head
//
// The splits of KV head h are the blocks of one cluster (at most 8, one
// block per split), each owning a run of 128-position stages; long contexts
// give each block several stages.  K and V of a stage arrive by two 1-D TMA
// bulk copies into single K / V buffers: the first stage is requested before
// griddepcontrol.wait (rows below the current position were written by
// earlier steps), the next stage's K as soon as the scores of the current
// stage are done, its V after the V pass.  The current position's row is
// normalised, rotated and written by the block that owns it.
//
// Inside a block (8 warps) every warp keeps its own online softmax over its
// positions w, w + 8, ...: scores use 8 lanes per position (4 positions per
// pass, 3-step shuffle reductions), the V pass one lane per 4 dimensions.
// The warps are combined once per block, and the blocks of the cluster once,
// through distributed shared memory: no partials in global memory, no
// tickets, no fences.
constexpr int kSP = kAttnSplitPositions;
constexpr int kMaxCluster = kMaxAttnCluster;
// Threads of the decode attention block: 8 warps at <= 128 registers, so a
// block shares its SM with a matvec block (programmatic launch overlap).
__host__ __device__ constexpr int AttnThreads(int /*G*/) { return 256; }

__host__ __device__ constexpr size_t AttnDynSmem(int /*G*/) {
  return 2 * static_cast<size_t>(kSP) * D * sizeof(__half) + 16;
}

template <int N, int NW>
__device__ __forceinline__ void BlockSumW(double (&v)[N], double* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < N; ++g) {
    v[g] = dev::WarpSumD(v[g]);
    if (lane == 0) sh[warp * N + g] = v[g];
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < N; ++g) {
    double t = sh[g];
#pragma unroll
    for (int w = 1; w < NW; ++w) t += sh[w * N + g];
    v[g] = t;
  }
}

__device__ __forceinline__ uint32_t ClusterRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void ClusterSync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `p` (this block's shared memory) in block `rank` of the cluster.
__device__ __forceinline__ uint32_t MapRank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(dev::SmemAddr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float LdCluster(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ double LdClusterD(uint32_t addr) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
  return v;
}

template <int G>
__global__ void __launch_bounds__(AttnThreads(G), 2) AttnDecodeKernel(const AttnParams p) {
  constexpr int kAT = AttnThreads(G);
  constexpr int kAW = kAT / 32;
  static_assert(static_cast<size_t>(kAW) * G * D * sizeof(float) <= 2 * kSP * D * sizeof(__half),
                "the warp partials must fit in the K/V buffers");
  extern __shared__ __align__(128) uint8_t dsm[];
  __half* Ks = reinterpret_cast<__half*>(dsm);
  __half* Vs = Ks + kSP * D;
  float* vred = reinterpret_cast<float*>(dsm);  // [kAW][G][D], reuses Ks/Vs after the last stage
  uint64_t* bars = reinterpret_cast<uint64_t*>(Vs + kSP * D);  // [0] K, [1] V
  __shared__ __align__(16) float qs[G + 1][D];
  __shared__ float sc[G][kSP];
  __shared__ double dsh[kAW * (G + 1)];
  __shared__ float fsh[kAW * G];
  // this block's result, read by the cluster's rank 0
  __shared__ float rec_m[G];
  __shared__ double rec_l[G];
  __shared__ __align__(16) float rec_o[G][D];

  dev::TraceScope trace(p.trace);
  const int h = blockIdx.y;
  const int s = static_cast<int>(ClusterRank());  // == blockIdx.x (one cluster spans the splits)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // The position counter of this step was written before the step started
  // (previous graph launch / host copy), so it may be read before the wait.
  const int64_t pos = *p.pos;
  const int64_t L = pos + 1;
  const int stages = static_cast<int>((L + kSP - 1) / kSP);
  const int per = (stages + p.n_splits - 1) / p.n_splits;  // stages per split
  const int st0 = s * per < stages ? s * per : stages;
  const int st1 = st0 + per < stages ? st0 + per : stages;  // st0 == st1: idle block (still merges)
  __half* kbase = p.kc + static_cast<int64_t>(h) * p.max_seq * D;
  __half* vbase = p.vc + static_cast<int64_t>(h) * p.max_seq * D;
  auto old_rows = [&](int st) -> int {  // rows of stage st already in the cache
    const int64_t r = pos - static_cast<int64_t>(st) * kSP;
    return static_cast<int>(r < kSP ? r : kSP);
  };
  auto issue = [&](int which, int st) {  // thread 0 only
    const int n_old = old_rows(st);
    if (n_old <= 0) return;
    const uint32_t bytes = static_cast<uint32_t>(n_old) * D * 2;
    __half* src = (which == 0 ? kbase : vbase) + static_cast<int64_t>(st) * kSP * D;
    dev::MbarExpectTx(bars + which, bytes);
    dev::BulkG2S(which == 0 ? Ks : Vs, src, bytes, bars + which);
  };

  if (tid == 0) {
    dev::MbarInit(bars + 0, 1);
    dev::MbarInit(bars + 1, 1);
    dev::MbarInitFence();
    if (st0 < st1) {
      issue(0, st0);
      issue(1, st0);
    }
  }
  // constants of this step (norm weights, the RoPE row of pos): before the wait
  const bool dimt = tid < D;
  const float wq = dimt ? p.q_norm[tid] : 0.f, wk = dimt ? p.k_norm[tid] : 0.f;
  const float rc = tid < D / 2 ? p.rope[pos * D + tid] : 0.f, rs = tid < D / 2 ? p.rope[pos * D + D / 2 + tid] : 0.f;
  __syncthreads();
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();

  // ---- q heads and the new key: RMSNorm + RoPE (threads 0..127 = dimensions)
  __half kh = __float2half_rn(0.f), vh = kh;
  {
    float vk[G + 1];
#pragma unroll
    for (int g = 0; g < G; ++g) vk[g] = dimt ? p.q[(h * G + g) * D + tid] : 0.f;
    vk[G] = dimt ? p.k_raw[h * D + tid] : 0.f;
    const float vv = dimt ? p.v_raw[h * D + tid] : 0.f;
    double ss[G + 1];
#pragma unroll
    for (int g = 0; g <= G; ++g) ss[g] = static_cast<double>(vk[g]) * vk[g];
    BlockSumW<G + 1, kAW>(ss, dsh);
    if (dimt) {
#pragma unroll
      for (int g = 0; g <= G; ++g) {
        const float scale = static_cast<float>(1.0 / sqrt(ss[g] / static_cast<double>(D) + static_cast<double>(p.eps)));
        qs[g][tid] = vk[g] * scale * (g < G ? wq : wk);
      }
    }
    __syncthreads();
    if (tid < D / 2) {
#pragma unroll
      for (int g = 0; g <= G; ++g) {
        const float a = qs[g][tid], b = qs[g][tid + D / 2];
        qs[g][tid] = a * rc - b * rs;
        qs[g][tid + D / 2] = b * rc + a * rs;
      }
    }
    __syncthreads();
    if (dimt) {
      kh = __float2half_rn(qs[G][tid]);
      vh = __float2half_rn(vv);
      if (st0 < st1 && pos < static_cast<int64_t>(st1) * kSP) {  // this block owns the new position
        kbase[pos * D + tid] = kh;
        vbase[pos * D + tid] = vh;
      }
    }
  }
  trace.Mark(1);  // q/k normalised and rotated

  // scores: 8 lanes per position; lane sub holds dimensions 8 sub .. +7 and
  // 64 + 8 sub .. +7 of every query head (scaled by 1/sqrt(128))
  const int sub = lane & 7, pp = lane >> 3;
  float qv[G][16];
#pragma unroll
  for (int g = 0; g < G; ++g) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const float4 qa = *reinterpret_cast<const float4*>(&qs[g][64 * hf + 8 * sub]);
      const float4 qb = *reinterpret_cast<const float4*>(&qs[g][64 * hf + 8 * sub + 4]);
      qv[g][8 * hf + 0] = qa.x * p.scale;
      qv[g][8 * hf + 1] = qa.y * p.scale;
      qv[g][8 * hf + 2] = qa.z * p.scale;
      qv[g][8 * hf + 3] = qa.w * p.scale;
      qv[g][8 * hf + 4] = qb.x * p.scale;
      qv[g][8 * hf + 5] = qb.y * p.scale;
      qv[g][8 * hf + 6] = qb.z * p.scale;
      qv[g][8 * hf + 7] = qb.w * p.scale;
    }
  }
  constexpr int kPasses = kSP / (4 * kAW);  // score passes per stage
  constexpr int kPerWarp = kSP / kAW;       // positions per warp per stage
  float m[G], acc[G][4];
  double l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  }
  for (int st = st0; st < st1; ++st) {
    const uint32_t par = static_cast<uint32_t>((st - st0) & 1);
    const int n_old = old_rows(st);
    const int64_t rem = L - static_cast<int64_t>(st) * kSP;
    const int n = static_cast<int>(rem < kSP ? rem : kSP);
    if (n_old > 0 && !dev::MbarWait(bars + 0, par)) {
      if (tid == 0 && p.err != nullptr) atomicOr(p.err, 2u);
    }
    if (n_old < n) {  // the stage holding the current position: publish its row
      if (dimt) {
        Ks[n_old * D + tid] = kh;
        Vs[n_old * D + tid] = vh;
      }
      __syncthreads();
    }
    // ---- scores of this warp's positions w + kAW (4 t + pp)
    float sv[G][kPasses];
#pragma unroll
    for (int t = 0; t < kPasses; ++t) {
      const int j = warp + kAW * (4 * t + pp);
      float d[G];
#pragma unroll
      for (int g = 0; g < G; ++g) d[g] = 0.f;
      if (j < n) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint4 raw = *reinterpret_cast<const uint4*>(Ks + j * D + 64 * hf + 8 * sub);
          const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(h2[e]);
#pragma unroll
            for (int g = 0; g < G; ++g) {
              d[g] = fmaf(qv[g][8 * hf + 2 * e], f.x, d[g]);
              d[g] = fmaf(qv[g][8 * hf + 2 * e + 1], f.y, d[g]);
            }
          }
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) d[g] += __shfl_xor_sync(0xFFFFFFFFu, d[g], o);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) sv[g][t] = j < n ? d[g] : -INFINITY;
    }
    if (st + 1 < st1) {
      __syncthreads();  // all reads of Ks done
      if (tid == 0) {
        dev::FenceProxyAsync();
        issue(0, st + 1);
      }
    }
    // ---- this warp's online softmax
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = sv[g][0];
#pragma unroll
      for (int t = 1; t < kPasses; ++t) mx = fmaxf(mx, sv[g][t]);
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
      const float nm = fmaxf(m[g], mx);
      const float alpha = m[g] == -INFINITY ? 0.f : expf(m[g] - nm);
      m[g] = nm;
      double ps = 0.0;
#pragma unroll
      for (int t = 0; t < kPasses; ++t) {
        const float e = sv[g][t] == -INFINITY ? 0.f : expf(sv[g][t] - nm);
        if (sub == 0) {
          sc[g][warp + kAW * (4 * t + pp)] = e;
          ps += static_cast<double>(e);
        }
      }
      ps = dev::WarpSumD(ps);
      l[g] = l[g] * static_cast<double>(alpha) + ps;
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[g][e] *= alpha;
    }
    if (n_old > 0 && !dev::MbarWait(bars + 1, par)) {
      if (tid == 0 && p.err != nullptr) atomicOr(p.err, 2u);
    }
    __syncwarp();  // this warp's weights are visible to its lanes
    // ---- V: the warp's positions; lane holds 4 dimensions
#pragma unroll
    for (int k = 0; k < kPerWarp; ++k) {
      const int j = warp + kAW * k;
      if (j < n) {
        const uint2 raw = *reinterpret_cast<const uint2*>(Vs + j * D + 4 * lane);
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
    }
    __syncwarp();
    if (st + 1 < st1) {
      __syncthreads();  // all reads of Vs done
      if (tid == 0) {
        dev::FenceProxyAsync();
        issue(1, st + 1);
      }
    }
  }
  // ---- combine this block's warps (Ks / Vs are free now: vred reuses them)
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      fsh[warp * G + g] = m[g];
      dsh[warp * G + g] = l[g];
    }
  }
  __syncthreads();
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = fsh[g];
#pragma unroll
    for (int w = 1; w < kAW; ++w) M = fmaxf(M, fsh[w * G + g]);
    const float sw = m[g] == -INFINITY ? 0.f : expf(m[g] - M);
    *reinterpret_cast<float4*>(vred + (warp * G + g) * D + 4 * lane) =
        make_float4(acc[g][0] * sw, acc[g][1] * sw, acc[g][2] * sw, acc[g][3] * sw);
    if (tid == 0) {
      double Lg = 0.0;
#pragma unroll
      for (int w = 0; w < kAW; ++w) {
        const float mw = fsh[w * G + g];
        Lg += mw == -INFINITY ? 0.0 : static_cast<double>(expf(mw - M)) * dsh[w * G + g];
      }
      rec_m[g] = M;
      rec_l[g] = Lg;
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kAT) {
    const int g = i / D, d = i - g * D;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kAW; ++w) t += vred[(w * G + g) * D + d];
    rec_o[g][d] = t;
  }
  trace.Mark(2);  // this block's part done
  // ---- combine the cluster's blocks in rank 0 through distributed shared memory
  ClusterSync();
  if (s == 0) {
    const int nb = static_cast<int>(gridDim.x);
    for (int i = tid; i < G * D; i += kAT) {
      const int g = i / D, d = i - g * D;
      float M = -INFINITY;
      for (int r = 0; r < nb; ++r) M = fmaxf(M, LdCluster(MapRank(&rec_m[g], r)));
      double den = 0.0;
      float num = 0.f;
      for (int r = 0; r < nb; ++r) {
        const float mr = LdCluster(MapRank(&rec_m[g], r));
        if (mr == -INFINITY) continue;
        const float w = expf(mr - M);
        den += static_cast<double>(w) * LdClusterD(MapRank(&rec_l[g], r));
        num = fmaf(w, LdCluster(MapRank(&rec_o[g][d], r)), num);
      }
      p.out[(h * G + g) * D + d] = num * static_cast<float>(1.0 / den);
    }
  }
  ClusterSync();  // no block leaves while rank 0 still reads its shared memory
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
  // block (t, head): head < n_heads is q head `head`, the others KV head
  // head - n_heads (its k row normalised and rotated, its v row copied)
  __shared__ __align__(16) float buf[1][D];
  __shared__ double dsh[4];
  const int t = blockIdx.x, head = blockIdx.y, tid = threadIdx.x;
  const int64_t pos = *pos0 + t;
  const float* row = qkv + static_cast<int64_t>(t) * (q_dim + 2 * kv_dim);
  const float* rr = rope + pos * D;
  if (head < n_heads) {
    float v[1] = {row[head * D + tid]};
    NormRope<1>(v, q_norm, eps, rr, buf, dsh);
    q_out[static_cast<int64_t>(t) * q_dim + head * D + tid] = v[0];
  } else {
    const int hk = head - n_heads;
    float v[1] = {row[q_dim + hk * D + tid]};
    NormRope<1>(v, k_norm, eps, rr, buf, dsh);
    const int64_t off = (static_cast<int64_t>(hk) * max_seq + pos) * D + tid;
    kc[off] = __float2half_rn(v[0]);
    vc[off] = __float2half_rn(row[q_dim + kv_dim + hk * D + tid]);
  }
}

// out (when given) gets the normalised row in FP32; hi / lo (when given) get
// it as the two fp16 terms of the tensor-core GEMM's activation operand
// (hi = fp16(v), lo = fp16(v - hi), the values SplitKernel would write).
__global__ void __launch_bounds__(256) RmsNormRowsKernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         int n, float eps, float* __restrict__ out,
                                                         __half* __restrict__ hi, __half* __restrict__ lo) {
  __shared__ double dsh[32];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * n;
  const float* xr = x + r0;
  double ss = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const double v = static_cast<double>(xr[i]);
    ss += v * v;
  }
  const double tot = dev::BlockSumD(ss, dsh);
  const float scale = static_cast<float>(1.0 / sqrt(tot / static_cast<double>(n) + static_cast<double>(eps)));
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = xr[i] * scale * w[i];
    if (out != nullptr) out[r0 + i] = v;
    if (hi != nullptr) {
      const __half h = __float2half_rn(v);
      hi[r0 + i] = h;
      lo[r0 + i] = __float2half_rn(v - __half2float(h));
    }
  }
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
  const int gs[4] = {1, 2, 4, 8};
  for (int i = 0; i < 4; ++i) {
    RPGB_CUDA(cudaFuncSetAttribute(fns[i], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   static_cast<int>(AttnDynSmem(gs[i]))));
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
    switch (G) {
      case 1: fn = reinterpret_cast<const void*>(AttnDecodeKernel<1>); break;
      case 2: fn = reinterpret_cast<const void*>(AttnDecodeKernel<2>); break;
      case 4: fn = reinterpret_cast<const void*>(AttnDecodeKernel<4>); break;
      case 8: fn = reinterpret_cast<const void*>(AttnDecodeKernel<8>); break;
      default: Throw("attention: GQA group %d is not supported (1, 2, 4, 8)", G);
    }
    RPGB_CHECK(p.n_splits <= kMaxCluster, "attention: %d splits exceed the cluster limit %d", p.n_splits,
               kMaxCluster);
    LaunchKernelClusterArgs(fn, dim3(p.n_splits, p.n_kv), dim3(AttnThreads(G)), AttnDynSmem(G), s, pdl,
                            static_cast<unsigned>(p.n_splits), p);
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
  RPGB_CHECK(n_heads + n_kv < 65536, "qk_rope: too many heads");
  QkRopeKvKernel<<<dim3(n_tok, n_heads + n_kv), 128, 0, s>>>(qkv, q_dim, kv_dim, q_norm, k_norm, rope, eps, pos0, kc,
                                                            vc, max_seq, n_heads, n_kv, q_out);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

void LaunchRmsNormRows(const float* x, const float* w, int n_rows, int n, float eps, float* out, cudaStream_t s,
                       __half* hi, __half* lo) {
  RPGB_CHECK(n_rows > 0 && n > 0, "rmsnorm: empty");
  RPGB_CHECK((hi == nullptr) == (lo == nullptr) && (out != nullptr || hi != nullptr), "rmsnorm: bad outputs");
  RmsNormRowsKernel<<<n_rows, 256, 0, s>>>(x, w, n, eps, out, hi, lo);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

}  // namespace rpgb
