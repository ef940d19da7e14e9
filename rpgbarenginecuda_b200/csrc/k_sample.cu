// k_sample.cu -- on-device temperature / top-k / top-p sampling.
//
// Semantics are the reference's (src/sampler.h:35-44, src/sampler_gpu.cu:161-348):
//   T <= 0      argmax, ties -> lowest index, no random number consumed
//   v = logit * (1/T)                        (only when T != 1)
//   top_k       active iff 1 < k < n; threshold = k-th largest value, v < thr dropped
//   softmax     e = expf(v - max), sum in double, p = e * float(1/sum)
//   top_p       active iff 0 < p < 1: cut = largest key t with sum{p_i : key_i <= t}
//               <= 1 - top_p; p <= cut dropped; keep >= 1 (argmax -> 1.0); renormalise
//   draw        u = SplitMix64 counter uniform; first i with serial double cumsum > u
//
// The reference finds both thresholds by 32-step bisection over the uint32 key
// space (64 full passes) and draws with a single-thread scan.  Here:
//  * general kernel (one 1024-thread block): exact radix selects (4 passes for
//    top-k with integer counts, 4 for top-p with 2^-60 fixed-point masses), a
//    blocked prefix scan for the draw that falls back to the exact serial scan
//    whenever u lies within 1e-9 of a prefix boundary;
//  * fast path (T > 0, 1 < top_k <= 64): every block of a 148-block grid keeps
//    its slice's top-k candidates (a superset of the global top-k survivors);
//    one small block then does the whole pipeline on the survivors only.  With
//    the tail at zero probability, the serial cumsum over survivors in index
//    order is bit-identical to the reference's full serial cumsum.
#include <cfloat>
#include <climits>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "launch.h"
#include "sample_dev.cuh"

namespace rpgb {
namespace {

using namespace smp;

constexpr int kGenThreads = 1024;
constexpr int kCandThreads = 256;
constexpr int kSliceMax = 2048;
constexpr int kSmallThreads = 512;
constexpr int kMaxCand = kCandBlocks * kFastTopK;

__device__ __forceinline__ int64_t Counter(const SampleParams& p) {
  if (p.counter_override != nullptr) return *p.counter_override;
  return *p.pos + p.pos_bump;
}

__device__ __forceinline__ void Finish(const SampleParams& p, int32_t tok) {
  *p.tok_out = tok;
  if (p.pos != nullptr) *p.pos += p.pos_bump;
}

__global__ void __launch_bounds__(kGenThreads) SampleGeneralKernel(const SampleParams p, int skip_if_flag) {
  dev::TraceScope trace(p.trace);
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();
  if (skip_if_flag && p.flag != nullptr && *p.flag == 1) return;
  const int tok = GeneralSample<kGenThreads>(p.logits, p.n, p.temperature, p.top_k, p.top_p, p.seed, Counter(p),
                                             p.probs);
  if (threadIdx.x == 0) Finish(p, tok);
}

// Per-slice top-k candidates on raw logits (temperature scaling is monotone).
__global__ void __launch_bounds__(kCandThreads) CandKernel(const SampleParams p) {
  __shared__ float vals[kSliceMax];
  __shared__ unsigned hist[2048];
  __shared__ uint32_t s_sel[3];
  __shared__ int s_cnt;
  dev::TraceScope trace(p.trace);
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();
  const int n = p.n;
  const int per = (n + kCandBlocks - 1) / kCandBlocks;
  const int a = blockIdx.x * per;
  const int len = a < n ? min(per, n - a) : 0;
  {
    constexpr int kR = kSliceMax / kCandThreads;
    float lv[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int i = threadIdx.x + r * kCandThreads;
      lv[r] = i < len ? p.logits[a + i] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int i = threadIdx.x + r * kCandThreads;
      if (i < len) vals[i] = lv[r];
    }
  }
  SliceCandidates(vals, len, a, p.top_k, hist, s_sel, &s_cnt, p.cand_val + blockIdx.x * kFastTopK,
                  p.cand_idx + blockIdx.x * kFastTopK, p.cand_cnt + blockIdx.x);
}

__global__ void __launch_bounds__(kSmallThreads) SampleSmallKernel(const SampleParams p) {
  extern __shared__ __align__(16) unsigned char sm[];
  dev::TraceScope trace(p.trace);
  dev::GridLaunchDependents();
  dev::GridWait();
  trace.Ready();
  const int tok = SmallSample<kSmallThreads>(p.cand_val, p.cand_idx, p.cand_cnt, kCandBlocks, p.temperature,
                                             p.top_k, p.top_p, p.seed, Counter(p), sm, kMaxCand);
  if (threadIdx.x == 0) {
    if (tok < 0) {
      *p.flag = 0;  // the general kernel runs
    } else {
      *p.flag = 1;
      Finish(p, tok);
    }
  }
}

}  // namespace

void PrepareSampleKernels() {
  RPGB_CUDA(cudaFuncSetAttribute(SampleSmallKernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(static_cast<size_t>(kMaxCand) * 16)));
}

void LaunchSample(const SampleParams& p, bool want_probs, cudaStream_t s, bool pdl) {
  RPGB_CHECK(p.n > 0, "sample: empty vocabulary");
  RPGB_CHECK(p.tok_out != nullptr && p.probs != nullptr, "sample: null buffers");
  const bool fast = !want_probs && p.temperature > 0.0f && p.top_k > 1 && p.top_k <= kFastTopK &&
                    p.top_k < p.n && p.n <= kCandBlocks * kSliceMax && p.cand_val != nullptr &&
                    p.flag != nullptr;
  if (fast) {
    SampleParams q = p;
    LaunchKernelArgs(reinterpret_cast<const void*>(CandKernel), dim3(kCandBlocks), dim3(kCandThreads), 0, s, pdl, q);
    const size_t smem = static_cast<size_t>(kMaxCand) * 16;
    if (q.trace.rec != nullptr) ++q.trace.id;
    LaunchKernelArgs(reinterpret_cast<const void*>(SampleSmallKernel), dim3(1), dim3(kSmallThreads), smem, s, pdl, q);
    if (q.trace.rec != nullptr) ++q.trace.id;
    LaunchKernelArgs(reinterpret_cast<const void*>(SampleGeneralKernel), dim3(1), dim3(kGenThreads), 0, s, pdl, q, 1);
    CountLaunches(3);
  } else {
    LaunchKernelArgs(reinterpret_cast<const void*>(SampleGeneralKernel), dim3(1), dim3(kGenThreads), 0, s, pdl, p, 0);
    CountLaunches(1);
  }
}

}  // namespace rpgb
