// sample_dev.cuh -- device pieces of the token sampler, shared by the
// standalone sampler kernels (k_sample.cu) and the decode loop kernel
// (k_step.cu).  Semantics: see k_sample.cu.
#pragma once

#include <cfloat>
#include <climits>

#include "kernels.cuh"
#include "kernels.h"

namespace rpgb {
namespace smp {

constexpr double kFix = 1152921504606846976.0;  // 2^60

// Block argmax over a global array, ties -> lowest index.  All threads return it.
__device__ inline int BlockArgmax(const float* x, int n, float* fsh, int* ish) {
  float bv = -FLT_MAX;
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
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
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) {
    fsh[warp] = bv;
    ish[warp] = bi;
  }
  __syncthreads();
  bv = fsh[0];
  bi = ish[0];
  for (int w = 1; w < nw; ++w) {
    if (fsh[w] > bv || (fsh[w] == bv && ish[w] < bi)) {
      bv = fsh[w];
      bi = ish[w];
    }
  }
  __syncthreads();
  return bi == INT_MAX ? 0 : bi;
}

// Warp 0 finds the digit d of the k-th largest key among the histogram's 256
// bins (bins taken from the top): s_sel = {d, rank of the k-th inside bin d}.
// Lane L owns bins 8L .. 8L+7; a suffix scan over the lanes replaces a serial
// 256-step walk.
__device__ __forceinline__ void SelectBin(const unsigned* hist, int rem, uint32_t* s_sel) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  unsigned h[8];
  unsigned sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    h[j] = hist[8 * lane + j];
    sum += h[j];
  }
  unsigned incl = sum;  // count of bins >= 8 lane
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_down_sync(0xFFFFFFFFu, incl, o);
    if (lane + o < 32) incl += v;
  }
  const unsigned excl = incl - sum;  // count of bins >= 8 (lane + 1)
  const unsigned r = static_cast<unsigned>(rem);
  if (excl < r && r <= incl) {
    unsigned cum = excl;
    int d = 8 * lane;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (cum + h[j] >= r) {
        d = 8 * lane + j;
        break;
      }
      cum += h[j];
    }
    s_sel[0] = static_cast<uint32_t>(d);
    s_sel[1] = r - cum;
  }
}

// As SelectBin for NB (a multiple of 32) bins: s_sel = {d, rank inside bin d,
// count of elements in the bins above d}.
template <int NB>
__device__ __forceinline__ void SelectBinN(const unsigned* hist, int rem, uint32_t* s_sel) {
  if (threadIdx.x >= 32) return;
  constexpr int PER = NB / 32;
  const int lane = threadIdx.x;
  unsigned sum = 0;
#pragma unroll 16
  for (int j = 0; j < PER; ++j) sum += hist[PER * lane + j];
  unsigned incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned v = __shfl_down_sync(0xFFFFFFFFu, incl, o);
    if (lane + o < 32) incl += v;
  }
  const unsigned excl = incl - sum;
  const unsigned r = static_cast<unsigned>(rem);
  if (excl < r && r <= incl) {
    unsigned cum = excl;
    int d = PER * lane;
    for (int j = PER - 1; j >= 0; --j) {
      const unsigned h = hist[PER * lane + j];
      if (cum + h >= r) {
        d = PER * lane + j;
        break;
      }
      cum += h;
    }
    s_sel[0] = static_cast<uint32_t>(d);
    s_sel[1] = r - cum;
    s_sel[2] = cum;
  }
}

// A radix-bin lower edge t with k <= #{OrderKey(x) >= t} <= kFastTopK (1 <= k
// <= n), found with 11-, 11- and 10-bit passes that stop as soon as the bin
// holding the k-th largest leaves few enough elements at or above it; *cnt
// receives #{key >= t} (more than kFastTopK only when ties at one exact key
// make the bound impossible).  hist holds 2048 bins.
__device__ inline uint32_t SliceBound(const float* x, int n, int k, unsigned* hist, uint32_t* s_sel, int* cnt) {
  uint32_t prefix = 0, mask = 0;
  int rem = k, above = 0;
  const int n_up = (n + 31) & ~31;
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const uint32_t nbm = pass == 2 ? 1023u : 2047u;
    for (int i = threadIdx.x; i <= static_cast<int>(nbm); i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n_up; i += blockDim.x) {
      uint32_t bin = 0xFFFFFFFFu;
      if (i < n) {
        const uint32_t key = dev::OrderKey(x[i]);
        if ((key & mask) == prefix) bin = (key >> shift) & nbm;
      }
      const unsigned same = __match_any_sync(0xFFFFFFFFu, bin);
      if (bin != 0xFFFFFFFFu && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
    }
    __syncthreads();
    if (pass < 2) {
      SelectBinN<2048>(hist, rem, s_sel);
    } else {
      SelectBinN<1024>(hist, rem, s_sel);
    }
    __syncthreads();
    const uint32_t d = s_sel[0];
    const int ge = above + static_cast<int>(s_sel[2]) + static_cast<int>(hist[d]);
    const uint32_t t = prefix | (d << shift);
    if (ge <= kFastTopK || pass == 2) {
      *cnt = ge;
      __syncthreads();
      return t;
    }
    prefix = t;
    mask |= nbm << shift;
    above += static_cast<int>(s_sel[2]);
    rem = static_cast<int>(s_sel[1]);
    __syncthreads();
  }
  return prefix;  // not reached
}

// Key of the k-th largest element of x[0..n) (multiplicity counted), 1 <= k <= n.
__device__ inline uint32_t RadixKth(const float* x, int n, int k, unsigned* hist, uint32_t* s_sel) {
  uint32_t prefix = 0, mask = 0;
  int rem = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    // Keys near the k-th share their leading bytes, so most increments hit the
    // same bin: lanes with equal bins are combined first (one atomic per group).
    const int n_up = (n + 31) & ~31;
    for (int i = threadIdx.x; i < n_up; i += blockDim.x) {
      uint32_t bin = 0xFFFFFFFFu;
      if (i < n) {
        const uint32_t key = dev::OrderKey(x[i]);
        if ((key & mask) == prefix) bin = (key >> shift) & 255u;
      }
      const unsigned same = __match_any_sync(0xFFFFFFFFu, bin);
      if (bin != 0xFFFFFFFFu && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&hist[bin], __popc(same));
    }
    __syncthreads();
    SelectBin(hist, rem, s_sel);
    __syncthreads();
    prefix |= s_sel[0] << shift;
    mask |= 255u << shift;
    rem = static_cast<int>(s_sel[1]);
    __syncthreads();
  }
  return prefix;
}

// Top-k candidates of one slice of the raw logits (temperature scaling is
// monotone): vals[0..len) in shared memory hold vocabulary ids base ..
// base + len - 1.  Writes up to kFastTopK (value, id) pairs and their count,
// or -1 when ties at one exact key make the bound impossible.  hist: 2048 bins.
__device__ __forceinline__ void SliceCandidates(const float* vals, int len, int base, int k, unsigned* hist,
                                                uint32_t* s_sel, int* s_cnt, float* cv, int32_t* ci,
                                                int32_t* cnt_out) {
  if (threadIdx.x == 0) *s_cnt = 0;
  __syncthreads();
  uint32_t thr = 0u;  // keep everything when the slice is not larger than k
  int ge = len;
  if (len > k) thr = SliceBound(vals, len, k, hist, s_sel, &ge);
  if (ge > kFastTopK) {
    if (threadIdx.x == 0) *cnt_out = -1;
    return;
  }
  for (int i = threadIdx.x; i < len; i += blockDim.x) {
    if (dev::OrderKey(vals[i]) >= thr) {
      const int slot = atomicAdd(s_cnt, 1);
      if (slot < kFastTopK) {
        cv[slot] = vals[i];
        ci[slot] = base + i;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *cnt_out = *s_cnt <= kFastTopK ? *s_cnt : -1;
}

// The general sampler: one block of NT threads over the whole vocabulary.
// Returns the token in every thread; probs[0..n) is scratch and is left
// holding the filtered, renormalised distribution.
template <int NT>
__device__ int GeneralSample(const float* logits, int n, float temperature, int top_k, float top_p, uint64_t seed,
                             int64_t counter, float* probs) {
  __shared__ double dsh[32];
  __shared__ float fsh[32];
  __shared__ int ish[32];
  __shared__ unsigned hist[256];
  __shared__ unsigned long long mhist[256];
  __shared__ uint32_t s_sel[3];
  __shared__ unsigned long long s_below;
  __shared__ double wsc[32];
  __shared__ int s_idx, s_amb, s_tok;
  const int tid = threadIdx.x;

  if (!(temperature > 0.0f)) {
    const int best = BlockArgmax(logits, n, fsh, ish);
    for (int i = tid; i < n; i += NT) probs[i] = i == best ? 1.0f : 0.0f;
    return best;
  }
  const float inv_t = 1.0f / temperature;
  for (int i = tid; i < n; i += NT) {
    float v = logits[i];
    if (temperature != 1.0f) v *= inv_t;
    probs[i] = v;
  }
  __syncthreads();

  if (top_k > 1 && top_k < n) {
    const float kth = dev::FromOrderKey(RadixKth(probs, n, top_k, hist, s_sel));
    for (int i = tid; i < n; i += NT) {
      if (probs[i] < kth) probs[i] = -INFINITY;
    }
    __syncthreads();
  }

  float lmax = -INFINITY;
  for (int i = tid; i < n; i += NT) lmax = fmaxf(lmax, probs[i]);
  const float mx = dev::BlockMax(lmax, fsh);
  double ls = 0.0;
  for (int i = tid; i < n; i += NT) {
    const float e = expf(probs[i] - mx);
    probs[i] = e;
    ls += static_cast<double>(e);
  }
  const double sum = dev::BlockSumD(ls, dsh);
  const float inv = static_cast<float>(1.0 / sum);
  for (int i = tid; i < n; i += NT) probs[i] *= inv;
  __syncthreads();

  if (top_p > 0.0f && top_p < 1.0f) {
    const double theta = 1.0 - static_cast<double>(top_p);
    const unsigned long long theta_fx = static_cast<unsigned long long>(theta * kFix);
    uint32_t prefix = 0, mask = 0;
    bool none = false;
    if (tid == 0) s_below = 0ull;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += NT) mhist[i] = 0ull;
      __syncthreads();
      for (int i = tid; i < n; i += NT) {
        const float v = probs[i];
        const uint32_t key = dev::OrderKey(v);
        if ((key & mask) == prefix) {
          atomicAdd(&mhist[(key >> shift) & 255u], static_cast<unsigned long long>(static_cast<double>(v) * kFix));
        }
      }
      __syncthreads();
      if (tid == 0) {
        unsigned long long cum = s_below;
        int d = 0;
        for (d = 0; d < 256; ++d) {
          if (cum + mhist[d] > theta_fx) break;
          cum += mhist[d];
        }
        s_sel[0] = static_cast<uint32_t>(d);
        s_below = cum;
      }
      __syncthreads();
      if (s_sel[0] >= 256u) {
        none = true;  // the whole distribution fits under 1 - top_p: nothing is cut
        break;
      }
      prefix |= s_sel[0] << shift;
      mask |= 255u << shift;
      __syncthreads();
    }
    const float cut = none ? dev::FromOrderKey(0xFFFFFFFFu) : dev::FromOrderKey(prefix - 1u);
    for (int i = tid; i < n; i += NT) {
      if (probs[i] <= cut) probs[i] = 0.0f;
    }
    __syncthreads();
    const int best = BlockArgmax(probs, n, fsh, ish);
    if (tid == 0 && probs[best] == 0.0f) probs[best] = 1.0f;
    __syncthreads();
    double l2 = 0.0;
    for (int i = tid; i < n; i += NT) l2 += static_cast<double>(probs[i]);
    const double sum2 = dev::BlockSumD(l2, dsh);
    if (sum2 > 0.0) {
      const float inv2 = static_cast<float>(1.0 / sum2);
      for (int i = tid; i < n; i += NT) probs[i] *= inv2;
    }
    __syncthreads();
  }

  // ---- draw: blocked prefix sums, exact serial fallback near a boundary
  const double u = static_cast<double>(dev::CounterUniform(seed, static_cast<uint64_t>(counter)));
  const int per = (n + NT - 1) / NT;
  const int a = tid * per, b = a + per < n ? a + per : n;
  double local = 0.0;
  for (int i = a; i < b; ++i) local += static_cast<double>(probs[i]);
  // exclusive scan over threads in index order
  const int lane = tid & 31, warp = tid >> 5;
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += y;
  }
  if (tid == 0) {
    s_idx = INT_MAX;
    s_amb = 0;
  }
  if (lane == 31) wsc[warp] = incl;
  __syncthreads();
  double wbase = 0.0;
  for (int w = 0; w < warp; ++w) wbase += wsc[w];
  const double prefix0 = wbase + incl - local;
  const double kMargin = 1e-9;
  if (a < b && prefix0 <= u + kMargin && prefix0 + local > u - kMargin) {
    double cum = prefix0;
    for (int i = a; i < b; ++i) {
      const double before = cum;
      cum += static_cast<double>(probs[i]);
      if (cum > u) {
        if (fabs(cum - u) < kMargin || fabs(before - u) < kMargin) atomicExch(&s_amb, 1);
        atomicMin(&s_idx, i);
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int tok = s_idx;
    if (s_amb) {
      // exact reference order: one serial double cumsum
      tok = INT_MAX;
      double cum = 0.0;
      for (int i = 0; i < n; ++i) {
        cum += static_cast<double>(probs[i]);
        if (cum > u) {
          tok = i;
          break;
        }
      }
    }
    if (tok == INT_MAX) {
      float bv = probs[0];
      tok = 0;
      for (int i = 1; i < n; ++i) {
        if (probs[i] > bv) {
          bv = probs[i];
          tok = i;
        }
      }
    }
    s_tok = tok;
  }
  __syncthreads();
  return s_tok;
}

// The fast path's second half: the whole pipeline on the candidates of
// n_slices slices (slice s: src.Count(s) candidates, loaded by src.Load).
// SmallSurvivors keeps the candidates at or above the k-th largest
// temperature-scaled value, ordered by vocabulary index, in scratch (values
// at cv, ids at ci) and returns their count -- or -1 when a slice
// overflowed or more than `cap` candidates lie above the lower bound (the
// caller then runs GeneralSample).  SmallDraw turns survivors into the
// token (softmax, top_p, the inverse draw); SmallSample is both.  scratch:
// 16 * cap bytes of shared memory.  mark(k) is called by every thread after
// stage k (1: bound and compaction, 2: k-th value, 3: softmax, 4: top_p),
// for timelines.
struct NoMark {
  __device__ void operator()(int) const {}
};
// Candidates in global memory (the lm_head slices of this GPU).
struct GlobalCands {
  const float* val;
  const int32_t* idx;
  const int32_t* cnt;
  __device__ __forceinline__ int Count(int s) const { return __ldcg(cnt + s); }
  // candidate j when `use` (else v = +inf, i = -1)
  __device__ __forceinline__ void Load(bool use, int j, float& v, int& i) const {
    v = use ? __ldcg(val + j) : INFINITY;
    i = use ? __ldcg(idx + j) : -1;
  }
};
template <int NT, class Src, class Mark = NoMark>
__device__ int SmallSurvivors(const Src src, int n_slices, float temperature, int top_k, unsigned char* scratch,
                              int cap, Mark mark = Mark()) {
  float* cv = reinterpret_cast<float*>(scratch);  // [cap]
  int* ci = reinterpret_cast<int*>(cv + cap);     // [cap]
  float* kv = reinterpret_cast<float*>(ci + cap);  // kept values / probs [cap]
  int* kix = reinterpret_cast<int*>(kv + cap);     // kept indices
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_sel[2];
  __shared__ int s_bad, s_m, s_c;
  const int tid = threadIdx.x;
  // slice counts; an overflowed slice sends this draw to the general kernel
  __shared__ int s_cnt[kCandBlocks];
  __shared__ float s_hmin[(kCandBlocks * kFastTopK + 31) / 32];
  __shared__ float s_t0, s_t1;
  if (tid < n_slices) s_cnt[tid] = src.Count(tid);
  if (tid == 0) {
    s_bad = 0;
    s_m = 0;
  }
  __syncthreads();
  if (tid < n_slices && s_cnt[tid] < 0) s_bad = 1;
  __syncthreads();
  if (s_bad) return -1;
  // Two lower bounds of the k-th largest logit; candidates under the larger
  // cannot survive top_k and are dropped here.  (1) Every slice with at least
  // k candidates holds k values >= its smallest candidate: the largest such
  // minimum.  (2) The k slices with the largest maxima hold k distinct values
  // >= the k-th largest slice maximum.  With the top values spread over many
  // slices (2) is far tighter: a few dozen candidates stay above it instead of
  // thousands.  Every value at or above the k-th largest is a candidate of
  // its slice (a slice's candidates are all its values above a bound that is
  // at most its own k-th largest), so nothing the filter keeps is lost.
  constexpr int kRounds = (kCandBlocks * kFastTopK + NT - 1) / NT;
  const int total = n_slices * kFastTopK;
  float rv[kRounds];
  int ri[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int j = tid + r * NT;
    const int b = j / kFastTopK, i = j - b * kFastTopK;
    src.Load(j < total && i < s_cnt[b], j, rv[r], ri[r]);
  }
  float* hmax = kv;        // half-slice maxima (kv is free until the survivors)
  float* smax = kv + 320;  // slice maxima, -inf for an empty slice
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int j = tid + r * NT;
    float mn = rv[r], mx = ri[r] >= 0 ? rv[r] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    }
    if ((tid & 31) == 0 && j < total) {  // one half slice per warp
      s_hmin[j >> 5] = mn;
      hmax[j >> 5] = mx;
    }
  }
  if (tid == 0) s_t1 = -INFINITY;
  __syncthreads();
  if (tid < n_slices) smax[tid] = fmaxf(hmax[2 * tid], hmax[2 * tid + 1]);
  if (tid < 32) {
    float t0 = -INFINITY;
    for (int b = tid; b < n_slices; b += 32) {
      if (s_cnt[b] >= top_k) t0 = fmaxf(t0, fminf(s_hmin[2 * b], s_hmin[2 * b + 1]));
    }
    t0 = dev::WarpMax(t0);
    if (tid == 0) s_t0 = t0;
  }
  __syncthreads();
  if (tid < n_slices && n_slices >= top_k) {  // the k-th largest slice maximum, by counting
    const float me = smax[tid];
    int gt = 0, ge = 0;
    for (int c = 0; c < n_slices; ++c) {
      gt += smax[c] > me;
      ge += smax[c] >= me;
    }
    if (gt < top_k && top_k <= ge && me > -INFINITY) s_t1 = me;
  }
  __syncthreads();
  const float t0 = fmaxf(s_t0, s_t1);
  const float inv_t = 1.0f / temperature;
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    if (ri[r] >= 0 && rv[r] >= t0) {
      float v = rv[r];
      if (temperature != 1.0f) v *= inv_t;
      const int slot = atomicAdd(&s_m, 1);
      if (slot < cap) {
        cv[slot] = v;
        ci[slot] = ri[r];
      }
    }
  }
  __syncthreads();
  const int m = s_m;
  if (m > cap) return -1;  // too many near-threshold candidates for the scratch
  mark(1);
  const float kth = dev::FromOrderKey(RadixKth(cv, m, top_k, hist, s_sel));
  mark(2);
  // survivors, ordered by vocabulary index
  if (tid == 0) s_c = 0;
  __syncthreads();
  for (int i = tid; i < m; i += NT) {
    if (cv[i] >= kth) {
      const int slot = atomicAdd(&s_c, 1);
      kv[slot] = cv[i];
      kix[slot] = ci[i];
    }
  }
  __syncthreads();
  const int c = s_c;
  // rank sort by index (c is small: k plus ties)
  for (int i = tid; i < c; i += NT) {
    int rank = 0;
    for (int j = 0; j < c; ++j) rank += kix[j] < kix[i];
    cv[rank] = kv[i];
    ci[rank] = kix[i];
  }
  __syncthreads();
  return c;
}

template <int NT, class Mark = NoMark>
__device__ __forceinline__ int SmallDraw(int c, float top_p, uint64_t seed, int64_t counter, unsigned char* scratch, int cap,
                         Mark mark = Mark()) {
  float* cv = reinterpret_cast<float*>(scratch);  // [cap]
  int* ci = reinterpret_cast<int*>(cv + cap);     // [cap]
  float* kv = reinterpret_cast<float*>(ci + cap);  // [cap]
  const int tid = threadIdx.x;
  __shared__ int s_tok;
  // ---- softmax over the survivors (serial, index order; c is k plus ties)
  float* v = cv;  // probabilities, index-ordered
  const int* ix = ci;
  __shared__ int s_forced;
  __shared__ float s_mx;
  __shared__ double s_sum;
  if (tid < 32) {
    float mx = -INFINITY;
    for (int i = tid; i < c; i += 32) mx = fmaxf(mx, v[i]);
    mx = dev::WarpMax(mx);
    if (tid == 0) s_mx = mx;
  }
  __syncthreads();
  for (int i = tid; i < c; i += NT) v[i] = expf(v[i] - s_mx);
  __syncthreads();
  if (tid == 0) {  // double sum in index order, as the serial reference loop
    double sum = 0.0;
    for (int i = 0; i < c; ++i) sum += static_cast<double>(v[i]);
    s_sum = sum;
    s_forced = 0;
  }
  __syncthreads();
  {
    const float inv = static_cast<float>(1.0 / s_sum);
    for (int i = tid; i < c; i += NT) v[i] *= inv;
  }
  __syncthreads();
  mark(3);
  if (top_p > 0.0f && top_p < 1.0f) {
    // ascending (key, index) order of the survivors' probabilities
    for (int i = tid; i < c; i += NT) {
      const uint32_t ki = dev::OrderKey(v[i]);
      int rank = 0;
      for (int j = 0; j < c; ++j) {
        const uint32_t kj = dev::OrderKey(v[j]);
        rank += (kj < ki) || (kj == ki && j < i);
      }
      kv[rank] = v[i];
    }
    __syncthreads();
    if (tid == 0) {
      // smallest key K* whose cumulative mass S(K*) exceeds 1 - top_p; everything
      // at or below the float just under K* is cut (reference: largest t with
      // S(t) <= 1 - top_p, drop p <= FromOrderKey(t)).
      const double theta = 1.0 - static_cast<double>(top_p);
      double cum = 0.0;
      bool found = false;
      uint32_t kstar = 0u;
      int i = 0;
      while (i < c) {
        const uint32_t key = dev::OrderKey(kv[i]);
        double grp = 0.0;
        int j = i;
        while (j < c && dev::OrderKey(kv[j]) == key) grp += static_cast<double>(kv[j++]);
        if (cum + grp > theta) {
          kstar = key;
          found = true;
          break;
        }
        cum += grp;
        i = j;
      }
      const float cut = found ? dev::FromOrderKey(kstar - 1u) : dev::FromOrderKey(0xFFFFFFFFu);
      bool any = false;
      for (int q = 0; q < c; ++q) {
        if (v[q] <= cut) v[q] = 0.0f;
        any = any || v[q] > 0.0f;
      }
      if (!any) s_forced = 1;  // every survivor cut: the reference then samples index 0
      double s2 = 0.0;
      for (int q = 0; q < c; ++q) s2 += static_cast<double>(v[q]);
      if (s2 > 0.0) {
        const float inv2 = static_cast<float>(1.0 / s2);
        for (int q = 0; q < c; ++q) v[q] *= inv2;
      }
    }
    __syncthreads();
  }
  mark(4);
  if (tid == 0) {
    int tok;
    if (s_forced) {
      tok = 0;
    } else {
      const double u = static_cast<double>(dev::CounterUniform(seed, static_cast<uint64_t>(counter)));
      tok = -1;
      double cum = 0.0;
      for (int i = 0; i < c; ++i) {
        cum += static_cast<double>(v[i]);
        if (cum > u) {
          tok = ix[i];
          break;
        }
      }
      if (tok < 0) {
        float bv = -1.0f;
        for (int i = 0; i < c; ++i) {
          if (v[i] > bv) {
            bv = v[i];
            tok = ix[i];
          }
        }
      }
    }
    s_tok = tok;
  }
  __syncthreads();
  return s_tok;
}

template <int NT, class Mark = NoMark>
__device__ int SmallSample(const float* cand_val, const int32_t* cand_idx, const int32_t* cand_cnt, int n_slices,
                           float temperature, int top_k, float top_p, uint64_t seed, int64_t counter,
                           unsigned char* scratch, int cap, Mark mark = Mark()) {
  const int c = SmallSurvivors<NT>(GlobalCands{cand_val, cand_idx, cand_cnt}, n_slices, temperature, top_k, scratch,
                                   cap, mark);
  if (c < 0) return -1;
  return SmallDraw<NT>(c, top_p, seed, counter, scratch, cap, mark);
}

}  // namespace smp
}  // namespace rpgb
