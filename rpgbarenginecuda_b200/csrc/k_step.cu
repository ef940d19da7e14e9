// k_step.cu -- the decode loop: n steps of the token loop in one persistent,
// cooperative kernel launch (one block of 16 warps per SM).
//
// Replaces, per step, GpuForwardStepDev's launches (src/qwen3_gpu.cu:289-330,
// GpuForwardLayer at 47-113: RMSNorm, q/k/v projections, QK-norm, RoPE, KV
// write, attention, o projection + residual, RMSNorm, gate/up, SiLU*up, down
// + residual; final norm and lm_head) and the sampler launch of the graph /
// no-graph generate loops (src/qwen3_gpu.cu:451-598).  The arithmetic of every
// op is the one of the standalone kernels (k_matvec.cu, k_attn.cu,
// k_sample.cu); what changes is how the step is scheduled:
//
//  * phases instead of launches.  A step is 5 phases per layer (qkv,
//    attention, o, gate/up, down) plus lm_head and the sampler.  Blocks meet
//    at a grid barrier between phases (one release-add and an acquire poll on
//    one word per block); the launch is cooperative, so all blocks are
//    resident and every barrier completes.  Every wait is bounded and reports
//    through `err`.
//  * one weight stream per warp across phases and steps.  Each warp owns a
//    ring of shared-memory slots fed by 1-D TMA bulk copies.  Its lane 0
//    walks the warp's units of every phase in order -- matvec block groups
//    of its unit range, or the cached K / V rows of its attention chunks --
//    and refills a slot as soon as it is consumed, so while a warp waits at a
//    barrier its ring already holds the next phase's weights.  Weights and
//    the K/V rows of earlier positions never depend on the running step.
//  * attention: the blocks of KV head h are `splits` consecutive blocks, each
//    owning a range of 12-position chunks; warps keep their own online
//    softmax over their chunks and the block folds them into one partial
//    record (m, l, o).  The o phase merges the records of all splits while it
//    builds its input, so there is no ticket and no extra barrier.
//  * sampling: the lm_head epilogue leaves each block's argmax (greedy) or
//    the top-k candidates of its own rows (fast path); after one barrier
//    every block reduces them itself (the result is identical in every
//    block), so the next step starts without another barrier.  The general
//    sampler runs in block 0 followed by a barrier.
#include <algorithm>
#include <cfloat>
#include <climits>

#include "common.h"
#include "kernels.cuh"
#include "kernels.h"
#include "mv_dev.cuh"
#include "sample_dev.cuh"

namespace rpgb {
namespace {

using namespace mv;

constexpr int kNW = 16;        // warps per block
constexpr int kNT = 32 * kNW;  // threads per block
constexpr int kChunk = 4;      // attention positions per unit (their K rows, then their V rows at +1024 B)
constexpr int kD = 128;        // head dimension
constexpr int kMaxRing = 8;
constexpr int kSmallCap = 2048;  // fast-path candidates above the lower bound kept in shared memory
// Tagged words of one attention partial record: o[G][128], then per q head
// g four words {m, l_hi, l_lo, unused} (the denominator l as a float pair,
// l_lo = l - l_hi), so one head's (m, l) is a single 32-byte read and
// consecutive records stay 16-byte aligned.
__host__ __device__ constexpr int RecWords(int G) { return 132 * G; }
constexpr int kSliceRows = 2048;
constexpr int kMaxOwnRows = 64;  // rows of x one block owns in the o / down phases
constexpr int kMaxLayers = 40;  // lm_head rows of one block for the candidate slices
constexpr uint32_t kBarLimit = 1u << 22;  // polls of a grid barrier before giving up (seconds)

enum Kind : int { kQkv = 0, kAttn = 1, kO = 2, kGu = 3, kDown = 4, kLm = 5 };

// float(1 / sqrt(a)) for the RMSNorm scale: the float estimate refined by two
// Newton steps in double (error ~2^-50 before the rounding to float, against
// ~0.3 us for a double sqrt and division on the critical path of a phase).
__device__ __forceinline__ float RmsScale(double a) {
  double r = static_cast<double>(rsqrtf(static_cast<float>(a)));
  r = r * (1.5 - 0.5 * a * r * r);
  r = r * (1.5 - 0.5 * a * r * r);
  return static_cast<float>(r);
}

// ------------------------------------------------------------------ shared memory plan

struct Plan {
  size_t bars, scratch, red, total;
  // inside the scratch union: matvec prologue
  size_t bfrag, sx, sscale, xs, merge;
};

__host__ __device__ inline size_t Al(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Ring slots are `slot` bytes: the largest block group of the model (Q6_K
// 3360 B for the Q4_K_M mix, 4352 B with Q5_K or Q8_0 matrices; a K + V
// attention chunk is 2048 B).
__host__ __device__ inline Plan MakePlan(int ring, int slot, int nb_max, int x_max, int scratch_bytes, int max_tiles) {
  Plan l;
  l.bars = static_cast<size_t>(kNW) * ring * slot;
  l.scratch = Al(l.bars + static_cast<size_t>(kNW) * ring * 8, 128);
  l.bfrag = 0;
  l.sx = l.bfrag + static_cast<size_t>(nb_max) * 1024;
  l.sscale = l.sx + static_cast<size_t>(nb_max) * 32;
  l.xs = Al(l.sscale + static_cast<size_t>(nb_max) * 4, 16);
  l.merge = Al(l.xs + static_cast<size_t>(x_max) * 4, 16);
  l.red = Al(l.scratch + static_cast<size_t>(scratch_bytes), 16);
  l.total = l.red + static_cast<size_t>(max_tiles + kNW) * kTile * 4;
  return l;
}

// Bytes of the split-merge tables: weights (float) and denominators (double)
// of every (KV head, split, group member), and 1/L per (KV head, member).
__host__ __device__ inline size_t MergeBytes(int n_kv, int splits, int group) {
  (void)n_kv;  // one head is merged at a time
  return static_cast<size_t>(splits) * group * 12 + static_cast<size_t>(group) * 4 + 16;
}

// Bytes of the scratch union for a model (the largest phase user).
size_t ScratchBytes(int nb_max, int x_max, int group, int n_kv, int splits) {
  const size_t prologue = Al(Al(static_cast<size_t>(nb_max) * (1024 + 32 + 4), 16) + static_cast<size_t>(x_max) * 4, 16) +
                          MergeBytes(n_kv, splits, group);
  const size_t attn = static_cast<size_t>(kNW) * group * kD * 4;
  const size_t lm = static_cast<size_t>(kSliceRows) * 4 + 2048 * 4;
  const size_t small = static_cast<size_t>(kSmallCap) * 16;
  size_t m = prologue;
  if (attn > m) m = attn;
  if (lm > m) m = lm;
  if (small > m) m = small;
  return Al(m, 128);
}

// ------------------------------------------------------------------ geometry

struct MvShape {
  int rows, K;
};

__device__ __forceinline__ MvShape ShapeOf(const LoopParams& p, int kind) {
  const int qd = p.n_heads * kD, kvd = p.n_kv * kD;
  switch (kind) {
    case kQkv: return {qd + 2 * kvd, p.hidden};
    case kO: return {p.hidden, qd};
    case kGu: return {2 * p.ffn, p.hidden};
    case kDown: return {p.hidden, p.ffn};
    default: return {p.lm_head.rows, p.hidden};
  }
}

struct Geo {
  int t0, t1, nb, u0, u1;
  int uoff0;  // first unit of the warp: block-group offset inside its matrix
};

// Segments of a phase's row space: q, k, v for the qkv phase, one matrix otherwise.
__device__ __forceinline__ int SegTiles(const LoopParams& p, int kind, int seg) {
  if (kind == kQkv) return seg == 0 ? p.n_heads * kD / kTile : p.n_kv * kD / kTile;
  return ShapeOf(p, kind).rows / kTile;
}
__device__ __forceinline__ int SegOfTile(const LoopParams& p, int kind, int tile, int* seg_t0) {
  int seg = 0, t0 = 0;
  if (kind == kQkv) {
    const int tq = p.n_heads * kD / kTile, tkv = p.n_kv * kD / kTile;
    if (tile >= tq + tkv) {
      seg = 2;
      t0 = tq + tkv;
    } else if (tile >= tq) {
      seg = 1;
      t0 = tq;
    }
  }
  *seg_t0 = t0;
  return seg;
}

// Tile range of this block and unit range of `warp` in a matvec phase.
__device__ __forceinline__ Geo MvGeo(const LoopParams& p, int kind, int warp) {
  const MvShape sh = ShapeOf(p, kind);
  Geo g;
  const int T = sh.rows / kTile;
  g.t0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * T / gridDim.x);
  g.t1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * T / gridDim.x);
  g.nb = sh.K >> 8;
  const int U = (g.t1 - g.t0) * g.nb;
  g.u0 = warp * U / kNW;
  g.u1 = (warp + 1) * U / kNW;
  const int tile = g.t0 + g.u0 / g.nb, b = g.u0 % g.nb;
  int st0 = 0;
  SegOfTile(p, kind, tile, &st0);
  g.uoff0 = (tile - st0) * g.nb + b;
  return g;
}

// The geometry of every matvec phase for every warp of this block, computed
// once per launch (it is the same for all layers and steps).
struct GeoTable {
  Geo g[6][kNW];  // indexed by Kind (the attention row is unused)
  int att_h, att_s;  // this block's KV head and split (att_h = n_kv: no attention work)
};

// A warp's attention chunks at one step: the weight stream's walk enters an
// attention phase once per layer, the geometry changes once per step.
struct AttnCache {
  int step, n, c0;
};
__shared__ AttnCache g_attc[kNW];

// Per super-block of a matvec phase's input: the phase's output tag once the
// warp computing its digits has stored them, so a warp's units start as soon
// as their own super-blocks are ready instead of after every input word of
// the phase has arrived.
constexpr int kMaxSb = 64;  // K <= 16384
__shared__ uint32_t g_sbready[kMaxSb];
__device__ __forceinline__ void SbPublish(int b, uint32_t tag) {
  asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(dev::SmemAddr(&g_sbready[b])), "r"(tag) : "memory");
}
__device__ __forceinline__ uint32_t SbLoad(int b) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(dev::SmemAddr(&g_sbready[b])) : "memory");
  return v;
}

// A warp's weight stream of one layer as runs of consecutive block groups
// (built once per launch): slots 0-2 the q, k and v parts of its qkv units,
// 3 the attention chunks (counted per step, g_attc), 4 o, 5 gate/up, 6 down,
// 7 lm_head (after the last layer).  Within one matrix the block groups of
// consecutive units are contiguous (tile-major), so a run is (offset, count).
constexpr int kRunAttn = 3, kRunDown = 6, kRunLm = 7, kRuns = 8;
struct Run {
  int off;  // first block group inside the matrix
  int n;    // units
  int mat;  // the layer's matrix (0-5: q, k, v, o, gate/up, down); lm_head for kRunLm
};
__shared__ Run g_runs[kNW][kRuns];

// Per layer: block-group bases of q, k, v, o, gate/up, down, the four norm
// weights and which matrices are Q6_K -- a copy of the layer table in shared
// memory, so the weight stream never waits on a global load.
struct LayerRow {
  const uint8_t* w[6];
  const float* norm[4];  // attn, ffn, q, k
  uint8_t type[6];       // ggml type of matrix i
};

// Matrix `seg` of a phase in layer `layer`: its block groups and type.
__device__ __forceinline__ int MatIdx(int kind, int seg) {
  return kind == kQkv ? seg : (kind == kO ? 3 : (kind == kGu ? 4 : 5));
}

__shared__ GeoTable g_geo;
__shared__ LayerRow g_layers[kMaxLayers];

__device__ __forceinline__ void FillTables(const LoopParams& p) {
  const int tid = threadIdx.x;
  if (tid < 6 * kNW) {
    const int kind = tid / kNW, warp = tid - kind * kNW;
    if (kind != kAttn) {
      const Geo g = MvGeo(p, kind, warp);
      g_geo.g[kind][warp] = g;
      if (kind == kQkv) {
        // split the warp's units at the q / k / v boundaries
        for (int sg = 0; sg < 3; ++sg) g_runs[warp][sg] = Run{0, 0, sg};
        int u = g.u0;
        while (u < g.u1) {
          const int tile = g.t0 + u / g.nb, b = u % g.nb;
          int st0 = 0;
          const int sg = SegOfTile(p, kind, tile, &st0);
          const int seg_end = (st0 + SegTiles(p, kind, sg) - g.t0) * g.nb;  // block unit index where sg ends
          const int n = (seg_end < g.u1 ? seg_end : g.u1) - u;
          g_runs[warp][sg] = Run{(tile - st0) * g.nb + b, n, sg};
          u += n;
        }
      } else {
        const int slot = kind == kLm ? kRunLm : kind + 2;  // o 4, gate/up 5, down 6
        g_runs[warp][slot] = Run{g.uoff0, g.u1 - g.u0, kind == kLm ? 6 : MatIdx(kind, 0)};
      }
    } else {
      g_attc[warp].step = -1;
      for (int i = warp; i < kMaxSb; i += kNW) g_sbready[i] = 0u;  // tags start at 1
      g_runs[warp][kRunAttn] = Run{0, 0, -1};
    }
    if (tid == 0) {
      const int c = static_cast<int>(blockIdx.x), S = p.splits;
      g_geo.att_h = c < p.n_kv * S ? c / S : p.n_kv;
      g_geo.att_s = c < p.n_kv * S ? c - (c / S) * S : 0;
    }
  } else if (tid - 6 * kNW < p.n_layers) {
    const int l = tid - 6 * kNW;
    const DevLayer& L = p.layers[l];
    const DevMat* m[6] = {&L.q, &L.k, &L.v, &L.o, &L.gateup, &L.down};
    LayerRow r;
    for (int i = 0; i < 6; ++i) {
      r.w[i] = m[i]->q;
      r.type[i] = static_cast<uint8_t>(m[i]->type);
    }
    r.norm[0] = L.attn_norm;
    r.norm[1] = L.ffn_norm;
    r.norm[2] = L.q_norm;
    r.norm[3] = L.k_norm;
    g_layers[l] = r;
  }
}

__device__ __forceinline__ uint32_t SegType(const LoopParams& p, int kind, int layer, int seg) {
  if (kind == kLm) return p.lm_head.type;
  return g_layers[layer].type[MatIdx(kind, seg)];
}

// Splits of a KV head that hold positions at this step: sixteen chunks (one
// per warp) or more each, so short contexts use few blocks and the o phase
// merges few records.
__device__ __forceinline__ int EffSplits(const LoopParams& p, int64_t pos) {
  const int n_ch = static_cast<int>((pos + kChunk) / kChunk);  // chunks covering positions 0..pos
  const int se = (n_ch + 15) / 16;  // at least 16 chunks (one per warp) per split
  return se < p.splits ? se : p.splits;
}

struct AttnGeo {
  int h, c0, c1;  // KV head, chunk range of this block (empty for an idle block)
};

__device__ __forceinline__ AttnGeo AttnOf(const LoopParams& p, const GeoTable& gt, int64_t pos) {
  AttnGeo a;
  a.h = gt.att_h;
  const int s = gt.att_s;
  const int se = EffSplits(p, pos);
  if (a.h >= p.n_kv || s >= se) {
    a.c0 = a.c1 = 0;
    return a;
  }
  const int n_ch = static_cast<int>((pos + kChunk) / kChunk);
  a.c0 = s * n_ch / se;
  a.c1 = (s + 1) * n_ch / se;
  return a;
}

__device__ __forceinline__ int WarpChunks(const AttnGeo& a, int warp) {
  const int n = a.c1 - a.c0 - warp;
  return n > 0 ? (n + kNW - 1) / kNW : 0;
}

// ------------------------------------------------------------------ the per-warp weight stream

struct Cursor {
  int step, layer, ri, j, n;  // run slot ri of (step, layer); unit j of its n
  uint32_t bytes;             // matvec: bytes of one unit of the run
  const uint8_t* src;         // matvec: next block group; attention: K row 0 of (layer, head)
  int c0;                     // attention: first chunk of this block
};

// Loads run slot c.ri of (c.step, c.layer) into the cursor (lane 0).
__device__ __forceinline__ void EnterRun(const LoopParams& p, const GeoTable& gt, Cursor& c, int64_t pos0, int warp) {
  if (c.ri == kRunAttn) {
    AttnCache& ac = g_attc[warp];
    if (ac.step != c.step) {
      const AttnGeo a = AttnOf(p, gt, pos0 + c.step);
      ac.step = c.step;
      ac.n = WarpChunks(a, warp);
      ac.c0 = a.c0;
    }
    c.n = ac.n;
    c.c0 = ac.c0;
    c.src = reinterpret_cast<const uint8_t*>(p.kc + static_cast<int64_t>(c.layer) * p.layer_elems +
                                             static_cast<int64_t>(gt.att_h) * p.max_seq * kD);
    return;
  }
  const Run r = g_runs[warp][c.ri];
  c.n = r.n;
  if (r.n > 0) {
    const bool lm = c.ri == kRunLm;
    const uint32_t type = lm ? p.lm_head.type : g_layers[c.layer].type[r.mat];
    c.bytes = static_cast<uint32_t>(dev::GroupBytesOf(type));
    c.src = (lm ? p.lm_head.q : g_layers[c.layer].w[r.mat]) + static_cast<int64_t>(r.off) * c.bytes;
  }
}

// Moves past finished and empty runs to the next unit of the stream (lane 0).
__device__ __forceinline__ void NextRun(const LoopParams& p, const GeoTable& gt, Cursor& c, int64_t pos0, int warp) {
  while (c.j >= c.n && c.step < p.n_steps) {
    c.j = 0;
    if (c.ri == kRunLm) {
      ++c.step;
      c.layer = 0;
      c.ri = 0;
    } else if (c.ri == kRunDown) {
      if (c.layer + 1 == p.n_layers) {
        c.ri = kRunLm;
      } else {
        ++c.layer;
        c.ri = 0;
      }
    } else {
      ++c.ri;
    }
    c.n = 0;
    if (c.step >= p.n_steps) break;
    EnterRun(p, gt, c, pos0, warp);
  }
}

// Requests unit c.j of the cursor's run into `dst` and advances (lane 0 only).
__device__ __forceinline__ void IssueUnit(const LoopParams& p, const GeoTable& gt, Cursor& c, int64_t pos0, int warp,
                                          uint8_t* dst, uint64_t* bar) {
  if (c.ri == kRunAttn) {
    // K rows then V rows (at +1024 B) of the chunk's positions from earlier steps
    const int64_t pos = pos0 + c.step;
    const int64_t r0 = static_cast<int64_t>(c.c0 + warp + kNW * c.j) * kChunk;
    int64_t n_old = pos - r0;
    n_old = n_old < 0 ? 0 : (n_old > kChunk ? kChunk : n_old);
    const uint32_t bytes = static_cast<uint32_t>(n_old) * kD * 2;
    dev::MbarExpectTx(bar, 2 * bytes);
    if (bytes > 0) {
      const uint8_t* src = c.src + r0 * (kD * 2);
      dev::BulkG2S(dst, src, bytes, bar);
      dev::BulkG2S(dst + kChunk * kD * 2, src + p.v_minus_k, bytes, bar);
    }
  } else {
    dev::MbarExpectTx(bar, c.bytes);
    dev::BulkG2S(dst, c.src, c.bytes, bar);
    c.src += c.bytes;  // block groups of one matrix are contiguous in tile-major order
  }
  if (++c.j >= c.n) NextRun(p, gt, c, pos0, warp);
}

struct Ring {
  uint8_t* base;
  uint64_t* bars;
  int R;
  uint32_t kc, ki;  // units consumed / issued by this warp
  int cs, is;       // ring slots of the next unit to consume / issue
  uint32_t cpar;    // mbarrier parity of the next unit to consume
  Cursor cur;       // next unit to issue (meaningful in lane 0)
  int step;         // the step being consumed
  bool bad;         // a wait gave up: later waits are skipped (the launch is failing)
};

// Lane 0: fills free slots with the next units of the stream.  Attention
// units of a later step are held back until that step runs: they read the
// cache row that the running step writes in the same layer.
__device__ __forceinline__ void RingPump(Ring& r, const LoopParams& p, const GeoTable& gt, int64_t pos0, int warp) {
  while (r.ki - r.kc < static_cast<uint32_t>(r.R) && r.cur.step < p.n_steps &&
         !(r.cur.ri == kRunAttn && r.cur.step > r.step)) {
    IssueUnit(p, gt, r.cur, pos0, warp, r.base + static_cast<size_t>(r.is) * p.slot, r.bars + r.is);
    ++r.ki;
    if (++r.is == r.R) r.is = 0;
  }
}

// Waits for the next unit; returns its slot.  A wait that gives up sets err
// and turns the later waits of this warp into no-ops, so a failing launch
// reaches its next grid barrier (where every block stops) quickly.
__device__ __forceinline__ const uint8_t* RingWait(Ring& r, const LoopParams& p) {
  const int slot = r.cs;
  if (!r.bad) {
    const bool ok = dev::MbarWait(r.bars + slot, r.cpar);
    if (!__all_sync(0xFFFFFFFFu, ok)) {
      r.bad = true;
      if ((threadIdx.x & 31) == 0) atomicOr(p.err, 1u);
    }
  }
  return r.base + static_cast<size_t>(slot) * p.slot;
}

// Marks the current unit consumed and refills free slots from the stream.
// attn_only: refill only while the next unit is an attention chunk (the
// chunk loop defers the walk into the following phases' weights to the next
// phase's start, where the warp waits for its input anyway).
__device__ __forceinline__ void RingRelease(Ring& r, const LoopParams& p, const GeoTable& gt, int64_t pos0,
                                            int warp, bool attn_only = false) {
  __syncwarp();
  ++r.kc;
  if (++r.cs == r.R) {
    r.cs = 0;
    r.cpar ^= 1u;
  }
  // No proxy fence before the refill: every lane's reads of the slot were
  // consumed (their values fed the unit's MMAs or FMAs) before the
  // __syncwarp above, so the bulk copy that overwrites the slot cannot
  // overtake them (measured: 0.5 % per token without the fence).
  if ((threadIdx.x & 31) == 0 && (!attn_only || r.cur.ri == kRunAttn)) {
    RingPump(r, p, gt, pos0, warp);
  }
}

// ------------------------------------------------------------------ grid barrier

__device__ __forceinline__ unsigned AtomAddRelease(unsigned* a, unsigned v) {
  unsigned old;
  asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ unsigned LdRelaxed(const unsigned* a) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void FenceAcquire() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void FenceProxyAsyncGlobal() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ------------------------------------------------------------------ tagged words
//
// Between the phases of a layer, data moves as 64-bit words {float bits,
// tag}: a producer stores each value together with the tag of the phase that
// made it (one single-copy-atomic 8-byte store), a consumer spins on exactly
// the words it needs until every tag matches.  The value itself carries the
// "ready" signal, so no barrier and no second round trip is needed (the
// low-latency protocol of NCCL's LL transport, applied inside one GPU).
// Every consumer of a buffer has read it completely before its own output
// exists, and the next writer of the buffer needs that output: one buffer
// per kind of data suffices.

__device__ __forceinline__ uint64_t Pack(float v, uint32_t tag) {
  return (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
}
__device__ __forceinline__ void StLL(uint64_t* a, float v, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(a), "l"(Pack(v, tag)) : "memory");
}
__device__ __forceinline__ void LdLL2(const uint64_t* a, uint64_t& w0, uint64_t& w1) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(a) : "memory");
}
__device__ __forceinline__ uint64_t LdLL(const uint64_t* a) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
  return w;
}
__device__ __forceinline__ bool TagOk(uint64_t w, uint32_t tag) { return static_cast<uint32_t>(w >> 32) == tag; }
__device__ __forceinline__ float ValOf(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

constexpr uint32_t kLLLimit = 1u << 21;  // polls of one tagged word group before giving up

// A wait gives up after kLLLimit polls, or early once another block has
// reported an error (checked every 512 polls).
__device__ __forceinline__ bool LLGiveUp(const LoopParams& p, uint32_t it) {
  if (it == (p.ll_limit != 0u ? p.ll_limit : kLLLimit)) {
    atomicOr(p.err, 8u);
    return true;
  }
  return (it & 511u) == 511u && *reinterpret_cast<volatile unsigned*>(p.err) != 0u;
}

// Eight consecutive tagged words (16-byte aligned) -> v[8], waiting for `tag`.
__device__ __forceinline__ void WaitLL8(const LoopParams& p, const uint64_t* a, uint32_t tag, float (&v)[8]) {
  uint64_t w[8];
  for (uint32_t it = 0;; ++it) {
#pragma unroll
    for (int i = 0; i < 4; ++i) LdLL2(a + 2 * i, w[2 * i], w[2 * i + 1]);
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) ok = ok && TagOk(w[i], tag);
    if (ok || LLGiveUp(p, it)) break;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = ValOf(w[i]);
}

// One tagged word, waiting for `tag`.
__device__ __forceinline__ float WaitLL1(const LoopParams& p, const uint64_t* a, uint32_t tag) {
  uint64_t w;
  for (uint32_t it = 0;; ++it) {
    w = LdLL(a);
    if (TagOk(w, tag) || LLGiveUp(p, it)) break;
  }
  return ValOf(w);
}

// Four consecutive tagged words (16-byte aligned), waiting for `tag`.
__device__ __forceinline__ float4 WaitLL4(const LoopParams& p, const uint64_t* a, uint32_t tag) {
  uint64_t w0, w1, w2, w3;
  for (uint32_t it = 0;; ++it) {
    LdLL2(a, w0, w1);
    LdLL2(a + 2, w2, w3);
    if ((TagOk(w0, tag) && TagOk(w1, tag) && TagOk(w2, tag) && TagOk(w3, tag)) || LLGiveUp(p, it)) break;
  }
  return make_float4(ValOf(w0), ValOf(w1), ValOf(w2), ValOf(w3));
}

// Tag of the output of (step, layer, kind); the lm_head phase is kind 5 of layer n_layers - 1.
// ---- tensor parallel: tagged words in every rank's exchange buffer.  Peer
// words cross NVLink, so stores and polls are system-scoped; a rank may start
// a launch some time after its peers, so their waits allow more polls.
constexpr uint32_t kPeerLimit = 1u << 24;
__device__ __forceinline__ void StSys(uint64_t* a, uint64_t w) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t LdSys(const uint64_t* a) {
  uint64_t w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
  return w;
}
// The word at a (in this rank's own buffer) once a peer stored it with `tag`.
__device__ __forceinline__ uint64_t WaitPeer(const LoopParams& p, const uint64_t* a, uint32_t tag) {
  uint64_t w;
  for (uint32_t it = 0;; ++it) {
    w = LdSys(a);
    if (TagOk(w, tag)) break;
    if (it == kPeerLimit) {
      atomicOr(p.err, 16u);
      break;
    }
    if ((it & 511u) == 511u && *reinterpret_cast<volatile unsigned*>(p.err) != 0u) break;
  }
  return w;
}
// Exchange buffer offsets: partial row `row` of attn_output (sel 0) or
// ffn_down (sel 1) from rank `src`; the lm_head argmax {value, index} of
// block `blk` of rank `src`.
__device__ __forceinline__ size_t XRed(const LoopParams& p, int sel, int src, int row) {
  return static_cast<size_t>(sel * kLoopMaxTp + src) * p.hidden + row;
}
__device__ __forceinline__ size_t XAm(const LoopParams& p, int src, int blk) {
  return static_cast<size_t>(2 * kLoopMaxTp) * p.hidden + 2 * (static_cast<size_t>(src) * gridDim.x + blk);
}
// The sampler's candidates of rank `src`: a count word, kFastTopK values,
// kFastTopK vocabulary ids.
constexpr int kXCandWords = 1 + 2 * kFastTopK;
__device__ __forceinline__ size_t XCand(const LoopParams& p, int src) {
  return static_cast<size_t>(2 * kLoopMaxTp) * (p.hidden + gridDim.x) + static_cast<size_t>(src) * kXCandWords;
}

__device__ __forceinline__ uint32_t TagOf(const LoopParams& p, int step, int layer, int kind) {
  return p.epoch0 + static_cast<uint32_t>(step) * static_cast<uint32_t>(5 * p.n_layers + 2) +
         static_cast<uint32_t>(5 * layer + kind) + 1u;
}

// All blocks arrive; bit 31 of the word flips when the last one does (block 0
// adds 2^31 - (n - 1), the others 1, so the low bits return to their start).
// Returns false in every thread of the block if the wait gave up or another
// block reported an error.
__device__ __forceinline__ bool GridBarrier(const LoopParams& p, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned inc = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1u) : 1u;
    const unsigned old = AtomAddRelease(p.bar, inc);
    int ok = 0;
    for (uint32_t i = 0; i < kBarLimit; ++i) {
      if ((LdRelaxed(p.bar) ^ old) & 0x80000000u) {
        FenceAcquire();
        ok = 1;
        break;
      }
      if ((i & 255u) == 255u && *reinterpret_cast<volatile unsigned*>(p.err) != 0u) break;
    }
    if (!ok) atomicOr(p.err, 4u);
    if (ok && *reinterpret_cast<volatile unsigned*>(p.err) != 0u) ok = 0;
    *s_flag = ok;
  }
  __syncthreads();
  // cached K/V rows written by other blocks are read by TMA (async proxy) later
  if ((threadIdx.x & 31) == 0) FenceProxyAsyncGlobal();
  return *reinterpret_cast<volatile int*>(s_flag) != 0;
}

// ------------------------------------------------------------------ trace

// Thread 0 of each block records, per phase: t_start = end of its previous
// phase (barrier arrival), t_ready = barrier release, t_end = end of the
// phase; up to two marks inside a phase become extra records whose block
// field carries k << 24 and whose t_end is the time of mark k.
// Reading %globaltimer costs about a microsecond on this GPU, so the
// timeline uses the SM's cycle counter and converts it to nanoseconds with
// one %globaltimer anchor per block (the SM clock rate comes from the host).
constexpr int kMarks = 4;
struct PhaseClock {
  uint64_t t_prev, t_ready;
  uint64_t mk[kMarks];
  uint64_t gt0;  // %globaltimer at the anchor
  int64_t ck0;   // %clock64 at the anchor
};
__device__ __forceinline__ int64_t Clock64() {
  int64_t c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}
__device__ __forceinline__ uint64_t ClockNs(const LoopParams& p, const PhaseClock& c) {
  return c.gt0 + static_cast<uint64_t>(static_cast<double>(Clock64() - c.ck0) * p.ns_per_cycle);
}
__device__ __forceinline__ void TraceReady(const LoopParams& p, PhaseClock& c) {
  if (p.trace.rec != nullptr && threadIdx.x == 0) c.t_ready = ClockNs(p, c);
}
__device__ __forceinline__ void TraceMark(const LoopParams& p, PhaseClock& c, int k) {
  if (p.trace.rec != nullptr && threadIdx.x == 0) c.mk[k - 1] = ClockNs(p, c);
}
// As TraceMark, from lane 0 of warp 0 without requiring thread 0's control flow.
__device__ __forceinline__ void TraceMarkW0(const LoopParams& p, PhaseClock& c, int k) {
  if (p.trace.rec != nullptr && threadIdx.x == 0) c.mk[k - 1] = ClockNs(p, c);
}
// Records of (phase id, block) go to fixed slots (no atomics on the way).
__device__ __forceinline__ void TraceEnd(const LoopParams& p, PhaseClock& c, uint32_t id) {
  if (p.trace.rec != nullptr && threadIdx.x == 0) {
    const uint64_t t = ClockNs(p, c);
    const uint64_t i0 = (static_cast<uint64_t>(id) * gridDim.x + blockIdx.x) * (1 + kMarks);
    for (uint32_t k = 0; k <= kMarks; ++k) {
      if (i0 + k >= p.trace.cap) break;
      const uint64_t te = k == 0 ? t : c.mk[k - 1];
      if (k > 0 && te == 0) {
        p.trace.rec[i0 + k] = TraceRec{0xFFFFFFFFu, 0u, 0ull, 0ull, 0ull};
        continue;
      }
      TraceRec r;
      r.id = id;
      r.block = blockIdx.x | (k << 24);
      r.t_start = c.t_prev;
      r.t_ready = c.t_ready ? c.t_ready : c.t_prev;
      r.t_end = te;
      p.trace.rec[i0 + k] = r;
    }
    c.t_prev = t;
    c.t_ready = 0;
    for (int k = 0; k < kMarks; ++k) c.mk[k] = 0;
  }
}

// ------------------------------------------------------------------ matvec phases

// Shared-memory pointers of the dynamic plan, recomputed where used (the
// kernel keeps no plan in registers).
struct Smem {
  uint8_t* base;
  const LoopParams* p;
  __device__ __forceinline__ Plan plan() const {
    return MakePlan(p->ring, p->slot, p->nb_max, p->x_max, p->scratch_bytes, p->max_tiles);
  }
  __device__ __forceinline__ uint8_t* scratch() const { return base + plan().scratch; }
};

__device__ __forceinline__ void Ld8(const float* src, bool shared, float (&v)[8]) {
  float4 a, b;
  if (shared) {
    a = *reinterpret_cast<const float4*>(src);
    b = *reinterpret_cast<const float4*>(src + 4);
  } else {
    a = __ldcg(reinterpret_cast<const float4*>(src));
    b = __ldcg(reinterpret_cast<const float4*>(src + 4));
  }
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Merge of KV head h's split records -> the attention output of its G q
// heads, published as tagged words (tag of the attention phase): weights
// exp(m_s - M), double denominator, as the split-K merge of the standalone
// kernel.  Runs in the last block of the head to finish (the records are
// tagged words, so their arrival order needs no memory ordering).
template <int G>
__device__ void MergeHead(const LoopParams& p, int step, int layer, int64_t pos, int h, uint8_t* merge) {
  const int tid = threadIdx.x;
  const uint32_t tag = TagOf(p, step, layer, kAttn);
  const int S = p.splits, se = EffSplits(p, pos);
  constexpr int kRec = RecWords(G);
  const uint64_t* recs = p.llrec + static_cast<size_t>(h) * S * kRec;
  float* wv = reinterpret_cast<float*>(merge);                                             // [se][G]
  double* lv = reinterpret_cast<double*>(merge + Al(static_cast<size_t>(se * G) * 4, 8));  // [se][G]
  float* inv = reinterpret_cast<float*>(lv + se * G);                                      // [G]
  for (int i = tid; i < se * G; i += kNT) {
    const int sp = i / G, g = i - sp * G;
    const float4 ml = WaitLL4(p, recs + static_cast<size_t>(sp) * kRec + 128 * G + 4 * g, tag);  // {m, l_hi, l_lo, -}
    wv[i] = ml.x;
    lv[i] = static_cast<double>(ml.y) + ml.z;
  }
  __syncthreads();
  if ((tid >> 5) < G) {  // warp g: lane sp holds split sp's (m, l) of q head g
    const int g = tid >> 5, lane = tid & 31;
    float m = -INFINITY;
    double wl = 0.0;
    float w = 0.f;
    for (int sp = lane; sp < se; sp += 32) m = fmaxf(m, wv[sp * G + g]);
    const float M = dev::WarpMax(m);
    for (int sp = lane; sp < se; sp += 32) {
      const int k = sp * G + g;
      w = wv[k] == -INFINITY ? 0.f : exp2f(wv[k] - M);
      wv[k] = w;
      wl += static_cast<double>(w) * lv[k];
    }
    const double L = dev::WarpSumD(wl);
    if (lane == 0) inv[g] = static_cast<float>(1.0 / L);
  }
  __syncthreads();
  // kPer threads per output value, each over every kPer-th split, so all the
  // loads of a head's records are in flight at once (one L2 round trip for
  // up to 10 kPer splits)
  constexpr int kPer = kNT / (G * kD) > 0 ? kNT / (G * kD) : 1;
  static_assert(kPer == 1 || (kPer == 2 && 32 % kPer == 0), "merge thread split");
  for (int t = tid; t < G * kD * kPer; t += kNT) {
    const int i = t / kPer, part = t - i * kPer;
    const int g = i / kD, d = i - g * kD;
    const uint64_t* base = recs + g * kD + d;
    float o = 0.f;
    constexpr int kB = 10;
    for (int s0 = part; s0 < se; s0 += kB * kPer) {
      uint64_t w[kB];
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int sp = s0 + j * kPer;
        w[j] = sp < se ? LdLL(base + static_cast<size_t>(sp) * kRec) : 0ull;
      }
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int sp = s0 + j * kPer;
        if (sp < se) {
          const float v = TagOk(w[j], tag) ? ValOf(w[j]) : WaitLL1(p, base + static_cast<size_t>(sp) * kRec, tag);
          o = fmaf(wv[sp * G + g], v, o);
        }
      }
    }
    if constexpr (kPer == 2) o += __shfl_xor_sync(0xFFFFFFFFu, o, 1);
    if (part == 0) StLL(p.llattn + static_cast<size_t>(h * G + g) * kD + d, o * inv[g], tag);
  }
}

struct LmOut {
  float* vals;  // this block's logits (fast path), kSliceRows
};

// One matvec phase.  Returns nothing; the epilogue writes its outputs.
template <int G>
__device__ void MvPhase(const LoopParams& p, const GeoTable& gt, int kind, int layer, int step, int64_t pos0,
                        int64_t pos, int tok, Ring& rg_io, const Smem& sm, PhaseClock& clk, float* xown, double* s_sq,
                        float* s_bv, int* s_bi, int* s_cnt, uint32_t* s_sel) {
  Ring rg = rg_io;  // in registers for the unit loop
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (lane == 0) {  // refills the attention phase deferred (a no-op when the ring is full)
    RingPump(rg, p, gt, pos0, warp);
  }
  const MvShape sh = ShapeOf(p, kind);
  const Geo g = gt.g[kind][warp];
  const int K = sh.K, nb = g.nb;
  const Plan pl = sm.plan();
  uint8_t* const scratch = sm.base + pl.scratch;
  uint8_t* bfrag = scratch + pl.bfrag;
  float* sx = reinterpret_cast<float*>(scratch + pl.sx);
  float* sscale = reinterpret_cast<float*>(scratch + pl.sscale);
  float* xs = reinterpret_cast<float*>(scratch + pl.xs);
  float* red = reinterpret_cast<float*>(sm.base + pl.red);
  const bool any = g.t1 > g.t0;
  const float* norm_w = kind == kQkv ? g_layers[layer].norm[0]
                                     : (kind == kGu ? g_layers[layer].norm[1] : (kind == kLm ? p.out_norm : nullptr));

  // ---- input (tagged words of the previous phase, the merged attention, or
  // the embedding row at layer 0) -> digits of x times the norm weight
  if (any) {
    const uint64_t* ll = nullptr;
    uint32_t tag = 0;
    if (kind == kQkv && layer == 0) {
      for (int c = tid; c < p.hidden; c += kNT) xs[c] = dev::DeqElem(p.embd, tok, c);
      __syncthreads();
    } else {
      ll = kind == kDown ? p.llh : (kind == kO ? p.llattn : p.llx);
      tag = kind == kQkv ? TagOf(p, step, layer - 1, kDown)
                         : (kind == kO ? TagOf(p, step, layer, kAttn)
                                       : (kind == kGu ? TagOf(p, step, layer, kO)
                                                      : (kind == kDown ? TagOf(p, step, layer, kGu)
                                                                       : TagOf(p, step, p.n_layers - 1, kDown))));
    }
    double ssq = 0.0;
    for (int b = warp; b < nb; b += kNW) {
      float v[8];
      if (ll != nullptr) {
        WaitLL8(p, ll + b * 256 + 8 * lane, tag, v);
      } else {
        Ld8(xs + b * 256 + 8 * lane, true, v);
      }
      if (norm_w != nullptr) {
        float w[8];
        Ld8(norm_w + b * 256 + 8 * lane, true, w);  // constant: cached loads
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          ssq += static_cast<double>(v[i]) * v[i];
          v[i] *= w[i];
        }
      }
      PutDigits(v, b, lane, bfrag, sx, sscale);
      __syncwarp();  // the warp's digit stores, then the release of its flag
      if (lane == 0) SbPublish(b, TagOf(p, step, layer, kind));
    }
    if (norm_w != nullptr) {
      ssq = dev::WarpSumD(ssq);
      if (lane == 0) s_sq[warp] = ssq;
    }
  }
  TraceMark(p, clk, 1);  // this warp's digits stored

  // ---- units
  const int n_units = g.u1 - g.u0;
  if (n_units > 0) {
    const LaneK lk = MakeLane(lane);
    uint32_t bA[8], bB[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) bA[i] = bB[i] = 0u;
    const uint32_t lo_half = lk.g < 4 ? 1u : 0u;
    float rg8 = 0.f, rgv = 0.f;
    int tl = g.u0 / nb, b = g.u0 % nb;
    int st0 = 0;
    uint32_t type = SegType(p, kind, layer, SegOfTile(p, kind, g.t0 + tl, &st0));
    for (int i = 0; i < n_units; ++i) {
      const uint8_t* grp = RingWait(rg, p);
      for (uint32_t it = 0; SbLoad(b) != TagOf(p, step, layer, kind); ++it) {  // bounded: set by the block's warps
        if (it == (1u << 24)) {
          atomicOr(p.err, 32u);
          break;
        }
      }
      LoadB(bfrag, b, lane, lo_half, bA, bB);
      const float s = sscale[b];
      UnitOf(type, grp, bA, bB, sx + b * 8, s, lk, lane, rgv, rg8);
      RingRelease(rg, p, gt, pos0, warp);
      if (++b == nb || i + 1 == n_units) {
        FlushPiece(red, tl + warp, lk, rgv, rg8);
        if (b == nb) {
          b = 0;
          ++tl;
          if (i + 1 < n_units) type = SegType(p, kind, layer, SegOfTile(p, kind, g.t0 + tl, &st0));
        }
      }
    }
  }
  rg_io = rg;
  __syncthreads();
  TraceMark(p, clk, 2);  // all units done
  // RMSNorm scale (applied to W x in the epilogue) from every warp's sum of squares
  float scale = 1.f;
  if (norm_w != nullptr && any) {
    double tot = 0.0;
    for (int w = 0; w < kNW; ++w) tot += s_sq[w];
    scale = RmsScale(tot / static_cast<double>(K) + static_cast<double>(p.eps));
  }

  // ---- epilogue
  TraceMark(p, clk, 3);
  const uint32_t tag_out = TagOf(p, step, layer, kind);
  const int U = (g.t1 - g.t0) * nb;
  const int n_rows = (g.t1 - g.t0) * kTile;
  const int rstep = kind == kGu ? 2 : 1;
  float best_v = -FLT_MAX;
  int best_i = INT_MAX;
  float* vals = reinterpret_cast<float*>(scratch);  // lm fast path: this block's logits
  for (int lr = tid * rstep; lr < n_rows; lr += kNT * rstep) {
    const int ti = lr / kTile, r = lr - ti * kTile;
    float v = 0.f, v2 = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const int a = w * U / kNW, e = (w + 1) * U / kNW;
      if (a < e && a < (ti + 1) * nb && e > ti * nb) {
        v += red[(ti + w) * kTile + r];
        if (kind == kGu) v2 += red[(ti + w) * kTile + r + 1];
      }
    }
    v *= scale;
    v2 *= scale;
    const int row = g.t0 * kTile + lr;
    if (kind == kQkv) {
      if (!(p.test_drop_word != 0 && step == 0 && layer == 0 && row == 0)) StLL(p.llqkv + row, v, tag_out);
    } else if (kind == kO || kind == kDown) {
      // x += W h: this block owns these rows of x in both phases
      float add = v;
      if (p.tp > 0) {
        // this rank's columns give a partial of the row: send it to every
        // rank, then add the ranks' partials in rank order (the same sum, so
        // the same x, on every rank)
        const int sel = kind == kDown ? 1 : 0;
        const uint64_t w = Pack(v, tag_out);
        const size_t off = XRed(p, sel, p.tp_rank, row);
        for (int k = 0; k < p.tp; ++k) StSys(p.xpeer[k] + off, w);
        const uint64_t* mine = p.xpeer[p.tp_rank];
        add = 0.f;
        for (int k = 0; k < p.tp; ++k) add += ValOf(WaitPeer(p, mine + XRed(p, sel, k, row), tag_out));
      }
      const float xn = xown[lr] + add;
      xown[lr] = xn;
      StLL(p.llx + row, xn, tag_out);
    } else if (kind == kGu) {
      // rows 2i (gate) and 2i+1 (up): (g / (1 + exp(-g))) * u, as src/kernels_gpu.cu:863-869
      StLL(p.llh + (row >> 1), (v / (1.0f + expf(-v))) * v2, tag_out);
    } else if (row < p.lm_head.rows) {
      p.logits[p.vocab0 + row] = v;
      if (p.step_logits != nullptr) p.step_logits[static_cast<int64_t>(step) * p.vocab + p.vocab0 + row] = v;
      if (p.mode == 0) {
        if (v > best_v) {  // rows increase per thread: strict > keeps the lowest index
          best_v = v;
          best_i = p.vocab0 + row;
        }
      } else if (p.mode == 1) {
        vals[lr] = v;
      }
    }
  }
  TraceMark(p, clk, 4);
  if (kind == kLm && p.mode == 0) {
    // block argmax, ties -> lowest index (src/kernels_gpu.cu:827-859)
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
      for (int i = 1; i < kNW; ++i) {
        if (s_bv[i] > bv || (s_bv[i] == bv && s_bi[i] < bi)) {
          bv = s_bv[i];
          bi = s_bi[i];
        }
      }
      if (p.tp > 0) {  // to every rank: the step's token is the argmax over all ranks' blocks
        const size_t off = XAm(p, p.tp_rank, blockIdx.x);
        const uint64_t wv = Pack(bv, tag_out);
        const uint64_t wi = (static_cast<uint64_t>(tag_out) << 32) | static_cast<uint32_t>(bi);
        for (int k = 0; k < p.tp; ++k) {
          StSys(p.xpeer[k] + off, wv);
          StSys(p.xpeer[k] + off + 1, wi);
        }
      } else {
        p.am_val[blockIdx.x] = bv;
        p.am_idx[blockIdx.x] = bi;
      }
    }
  } else if (kind == kLm && p.mode == 1) {
    __syncthreads();
    const int row0 = g.t0 * kTile;  // this GPU's rows of the vocabulary start at vocab0
    int len = n_rows;
    if (row0 + len > p.lm_head.rows) len = p.lm_head.rows - row0 > 0 ? p.lm_head.rows - row0 : 0;
    unsigned* hist = reinterpret_cast<unsigned*>(scratch + kSliceRows * 4);
    smp::SliceCandidates(vals, len, p.vocab0 + row0, p.top_k, hist, s_sel, s_cnt,
                         p.cand_val + blockIdx.x * kFastTopK, p.cand_idx + blockIdx.x * kFastTopK,
                         p.cand_cnt + blockIdx.x);
  }
}

// ------------------------------------------------------------------ attention phase

template <int G>
struct __align__(16) AttnShared {
  float qs[G][kD];            // normalised, rotated q heads, times 1/sqrt(128)
  __half knew[kD], vnew[kD];  // the current position's row
  double sq[2 * (G + 1)];     // sums of squares, two warps per vector
  double dsh[kNW * G];
  float fsh[kNW * G];
  int last;  // this block merges the head's records
};

template <int G>
__device__ void AttnPhase(const LoopParams& p, const GeoTable& gt, int layer, int step, int64_t pos0, int64_t pos,
                          uint32_t tick_last, Ring& rg_io, const Smem& sm, PhaseClock& clk, AttnShared<G>& as) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const AttnGeo a = AttnOf(p, gt, pos);
  if (a.c1 <= a.c0) return;  // no positions for this block at this step
  Ring rg = rg_io;           // in registers for the chunk loop
  const int h = a.h, S = p.splits, s = static_cast<int>(blockIdx.x) - h * S;
  const LayerRow& Ly = g_layers[layer];
  const int qd = p.n_heads * kD, kvd = p.n_kv * kD;
  const int pc = static_cast<int>(pos / kChunk);
  const bool owner = pc >= a.c0 && pc < a.c1;  // this block's chunks hold the current position
  const int64_t cache_off =
      static_cast<int64_t>(layer) * p.layer_elems + (static_cast<int64_t>(h) * p.max_seq + pos) * kD;

  // ---- q heads and the new key: RMSNorm + RoPE.  Thread t < 64 (G + 1) owns
  // dimensions d and d + 64 of vector vi = t / 64 (q heads 0..G-1, then k),
  // so the rotation stays in registers; the next 128 threads take v.
  const uint32_t tag = TagOf(p, step, layer, kQkv);
  const int vi = tid >> 6, d = tid & 63;
  float e0 = 0.f, e1 = 0.f;
  // the norm weights and this position's rotation do not depend on the qkv
  // phase: load them before waiting for its words
  float nw0 = 0.f, nw1 = 0.f, rc = 0.f, rs = 0.f;
  if (vi <= G) {
    const float* nw = vi < G ? Ly.norm[2] : Ly.norm[3];
    nw0 = nw[d];
    nw1 = nw[d + 64];
    rc = p.rope[pos * kD + d];
    rs = p.rope[pos * kD + kD / 2 + d];
  }
  if (vi <= G) {
    const int64_t off = vi < G ? static_cast<int64_t>(h * G + vi) * kD : qd + h * kD;
    uint64_t w0 = LdLL(p.llqkv + off + d), w1 = LdLL(p.llqkv + off + d + 64);
    if (!TagOk(w0, tag)) w0 = Pack(WaitLL1(p, p.llqkv + off + d, tag), tag);
    if (!TagOk(w1, tag)) w1 = Pack(WaitLL1(p, p.llqkv + off + d + 64, tag), tag);
    e0 = ValOf(w0);
    e1 = ValOf(w1);
    double ss = static_cast<double>(e0) * e0 + static_cast<double>(e1) * e1;
    ss = dev::WarpSumD(ss);
    if (lane == 0) as.sq[warp] = ss;
  } else if (tid < 64 * (G + 1) + kD) {
    const int dv = tid - 64 * (G + 1);
    const __half vh = __float2half_rn(WaitLL1(p, p.llqkv + qd + kvd + h * kD + dv, tag));
    as.vnew[dv] = vh;
    if (owner) {
      p.vc[cache_off + dv] = vh;
      FenceProxyAsyncGlobal();
    }
  }
  //M1
  __syncthreads();
  if (vi <= G) {
    const double tot = as.sq[2 * vi] + as.sq[2 * vi + 1];
    const float sc = RmsScale(tot / static_cast<double>(kD) + static_cast<double>(p.eps));
    // scores in log2 units (q times 1/sqrt(128) times log2(e)): the softmax
    // then exponentiates with exp2f; the split records carry the same units
    const float qscale = p.scale * 1.4426950408889634f;
    const float x0 = e0 * sc * nw0, x1 = e1 * sc * nw1;
    const float y0 = x0 * rc - x1 * rs, y1 = x1 * rc + x0 * rs;
    if (vi < G) {
      as.qs[vi][d] = y0 * qscale;
      as.qs[vi][d + 64] = y1 * qscale;
    } else {
      const __half k0 = __float2half_rn(y0), k1 = __float2half_rn(y1);
      as.knew[d] = k0;
      as.knew[d + 64] = k1;
      if (owner) {
        p.kc[cache_off + d] = k0;
        p.kc[cache_off + d + 64] = k1;
        FenceProxyAsyncGlobal();
      }
    }
  }
  __syncthreads();
  //M2

  // ---- this warp's 4-position units.  Scores: 8 lanes per position (lane
  // sub holds dimensions 8 sub .. +7 and 64 + 8 sub .. +7, position pp = lane / 8);
  // online softmax over the warp's positions; V with 4 dimensions per lane.
  const int sub = lane & 7, pp = lane >> 3;
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[g][e] = 0.f;
  }
  // this lane's q dimensions (64 hf + 8 sub .. +7) do not change over the
  // chunks: for G = 2 they stay in registers (32 floats)
  constexpr int kQr = G == 2 ? G : 1;
  float4 qr[kQr][2][2];
  if constexpr (G == 2) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        qr[g][hf][0] = *reinterpret_cast<const float4*>(&as.qs[g][64 * hf + 8 * sub]);
        qr[g][hf][1] = *reinterpret_cast<const float4*>(&as.qs[g][64 * hf + 8 * sub + 4]);
      }
    }
  }
  for (int ch = a.c0 + warp; ch < a.c1; ch += kNW) {
    const int64_t r0 = static_cast<int64_t>(ch) * kChunk;
    const int n_valid = static_cast<int>(pos + 1 - r0 < kChunk ? pos + 1 - r0 : kChunk);
    const int n_old = static_cast<int>(pos - r0 < kChunk ? pos - r0 : kChunk);
    const uint8_t* slot = RingWait(rg, p);
    if (ch == a.c0) TraceMarkW0(p, clk, 1);
    float dd[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dd[g] = 0.f;
    if (pp < n_valid) {
      const __half* krow = pp < n_old ? reinterpret_cast<const __half*>(slot + pp * kD * 2) : as.knew;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint4 raw = *reinterpret_cast<const uint4*>(krow + 64 * hf + 8 * sub);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]);
        const float2 f2 = __half22float2(h2[2]), f3 = __half22float2(h2[3]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float4 qa, qb;
          if constexpr (G == 2) {
            qa = qr[g][hf][0];
            qb = qr[g][hf][1];
          } else {
            qa = *reinterpret_cast<const float4*>(&as.qs[g][64 * hf + 8 * sub]);
            qb = *reinterpret_cast<const float4*>(&as.qs[g][64 * hf + 8 * sub + 4]);
          }
          dd[g] = fmaf(qa.x, f0.x, dd[g]);
          dd[g] = fmaf(qa.y, f0.y, dd[g]);
          dd[g] = fmaf(qa.z, f1.x, dd[g]);
          dd[g] = fmaf(qa.w, f1.y, dd[g]);
          dd[g] = fmaf(qb.x, f2.x, dd[g]);
          dd[g] = fmaf(qb.y, f2.y, dd[g]);
          dd[g] = fmaf(qb.z, f3.x, dd[g]);
          dd[g] = fmaf(qb.w, f3.y, dd[g]);
        }
      }
    }
    float ev[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sc = dd[g];
      sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 1);
      sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 2);
      sc += __shfl_xor_sync(0xFFFFFFFFu, sc, 4);
      if (pp >= n_valid) sc = -INFINITY;
      float mx = fmaxf(sc, __shfl_xor_sync(0xFFFFFFFFu, sc, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
      const float nm = fmaxf(m[g], mx);
      const float alpha = m[g] == -INFINITY ? 0.f : exp2f(m[g] - nm);
      const float e = pp < n_valid ? exp2f(sc - nm) : 0.f;
      float ps = e + __shfl_xor_sync(0xFFFFFFFFu, e, 8);
      ps += __shfl_xor_sync(0xFFFFFFFFu, ps, 16);
      m[g] = nm;
      l[g] = l[g] * alpha + ps;
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[g][q] *= alpha;
      ev[g] = e;
    }
#pragma unroll
    for (int jj = 0; jj < kChunk; ++jj) {
      if (jj < n_valid) {
        const __half* vrow =
            jj < n_old ? reinterpret_cast<const __half*>(slot + (kChunk + jj) * kD * 2) : as.vnew;
        const uint2 raw = *reinterpret_cast<const uint2*>(vrow + 4 * lane);
        const float2 x0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 x1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float e = __shfl_sync(0xFFFFFFFFu, ev[g], 8 * jj);
          acc[g][0] = fmaf(e, x0.x, acc[g][0]);
          acc[g][1] = fmaf(e, x0.y, acc[g][1]);
          acc[g][2] = fmaf(e, x1.x, acc[g][2]);
          acc[g][3] = fmaf(e, x1.y, acc[g][3]);
        }
      }
    }
    if (ch == a.c0) TraceMarkW0(p, clk, 2);
    RingRelease(rg, p, gt, pos0, warp, true);
    if (ch == a.c0) TraceMarkW0(p, clk, 3);
  }
  TraceMarkW0(p, clk, 4);  // warp 0: its units done
  rg_io = rg;

  // ---- fold the warps into this block's record
  float* vred = reinterpret_cast<float*>(sm.scratch());  // [kNW][G][128]
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      as.fsh[warp * G + g] = m[g];
      as.dsh[warp * G + g] = static_cast<double>(l[g]);
    }
  }
  __syncthreads();
  constexpr int kRec = RecWords(G);
  uint64_t* rec = p.llrec + (static_cast<size_t>(h) * S + s) * kRec;
  const uint32_t tag_out = TagOf(p, step, layer, kAttn);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = as.fsh[g];
#pragma unroll
    for (int w = 1; w < kNW; ++w) M = fmaxf(M, as.fsh[w * G + g]);
    const float sw = m[g] == -INFINITY ? 0.f : exp2f(m[g] - M);
    *reinterpret_cast<float4*>(vred + (warp * G + g) * kD + 4 * lane) =
        make_float4(acc[g][0] * sw, acc[g][1] * sw, acc[g][2] * sw, acc[g][3] * sw);
    if (warp == 0) {  // lanes 0..15 weigh the warps' denominators
      double t = 0.0;
      if (lane < kNW) {
        const float mw = as.fsh[lane * G + g];
        t = mw == -INFINITY ? 0.0 : static_cast<double>(exp2f(mw - M)) * as.dsh[lane * G + g];
      }
      t = dev::WarpSumD(t);
      if (lane == 0) {
        const float lhi = static_cast<float>(t);
        StLL(rec + 128 * G + 4 * g, M, tag_out);
        StLL(rec + 128 * G + 4 * g + 1, lhi, tag_out);
        StLL(rec + 128 * G + 4 * g + 2, static_cast<float>(t - static_cast<double>(lhi)), tag_out);
        StLL(rec + 128 * G + 4 * g + 3, 0.f, tag_out);
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < G * kD; i += kNT) {
    const int g = i / kD, dd2 = i - g * kD;
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) t += vred[(w * G + g) * kD + dd2];
    StLL(rec + g * kD + dd2, t, tag_out);
  }
  // the last block of this head to get here merges the head's records
  __syncthreads();
  if (tid == 0) as.last = atomicAdd(p.tickets + h, 1u) == tick_last ? 1 : 0;
  __syncthreads();
  if (as.last) MergeHead<G>(p, step, layer, pos, h, sm.scratch() + sm.plan().merge);
}

// ------------------------------------------------------------------ the kernel

// ------------------------------------------------------------------ tensor parallel sampling

// The candidates every rank sent into this rank's exchange buffer (tagged
// words; each read waits for its tag).
struct PeerCands {
  const LoopParams* p;
  const uint64_t* base;  // this rank's XCand(0)
  uint32_t tag;
  __device__ __forceinline__ int Count(int s) const {
    return static_cast<int>(static_cast<uint32_t>(WaitPeer(*p, base + static_cast<size_t>(s) * kXCandWords, tag)));
  }
  __device__ __forceinline__ void Load(bool use, int j, float& v, int& i) const {
    v = INFINITY;
    i = -1;
    if (use) {  // only words a rank wrote: the others never get this tag
      const int s = j / kFastTopK, k = j - s * kFastTopK;
      const uint64_t* w = base + static_cast<size_t>(s) * kXCandWords + 1 + k;
      v = ValOf(WaitPeer(*p, w, tag));
      i = static_cast<int>(static_cast<uint32_t>(WaitPeer(*p, w + kFastTopK, tag)));
    }
  }
};

// The fast sampler over the whole vocabulary when each rank holds the
// lm_head rows of one slice of it.  Every block reduces this rank's slice
// candidates to its survivors (the candidates at or above this rank's k-th
// largest scaled value: a superset of the global top_k's members from this
// slice); blocks 0 .. tp-1 send them to ranks 0 .. tp-1; then every block
// of every rank runs the small sampler on the tp survivor sets (values
// already scaled, so temperature 1) and draws the same token.  Returns -1 in
// every block of every rank when a survivor set overflows (ties at the
// k-th value): the host then samples that token from the gathered row.
template <class Mark>
__device__ int TpSample(const LoopParams& p, int step, int64_t pos, const Smem& sm, Mark mark) {
  unsigned char* scratch = sm.scratch();
  const int tid = threadIdx.x;
  const uint32_t tag = TagOf(p, step, p.n_layers - 1, kLm);
  const int c = smp::SmallSurvivors<kNT>(smp::GlobalCands{p.cand_val, p.cand_idx, p.cand_cnt},
                                         static_cast<int>(gridDim.x), p.temperature, p.top_k, scratch, kSmallCap,
                                         mark);
  if (static_cast<int>(blockIdx.x) < p.tp) {
    const float* cv = reinterpret_cast<const float*>(scratch);
    const int* ci = reinterpret_cast<const int*>(cv + kSmallCap);
    uint64_t* dst = p.xpeer[blockIdx.x] + XCand(p, p.tp_rank);
    const int cnt = c < 0 || c > kFastTopK ? -1 : c;
    const uint64_t hi = static_cast<uint64_t>(tag) << 32;
    for (int i = tid; i < cnt; i += kNT) {
      StSys(dst + 1 + i, Pack(cv[i], tag));
      StSys(dst + 1 + kFastTopK + i, hi | static_cast<uint32_t>(ci[i]));
    }
    if (tid == 0) StSys(dst, hi | static_cast<uint32_t>(cnt));
  }
  __syncthreads();  // the survivors' scratch is reused below
  const int c2 = smp::SmallSurvivors<kNT>(PeerCands{&p, p.xpeer[p.tp_rank] + XCand(p, 0), tag}, p.tp, 1.0f,
                                          p.top_k, scratch, kSmallCap, mark);
  if (c2 < 0) return -1;
  return smp::SmallDraw<kNT>(c2, p.top_p, p.seed, pos + 1, scratch, kSmallCap, mark);
}

template <int G>
__global__ void __launch_bounds__(kNT, 1) DecodeLoopKernel(const LoopParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ AttnShared<G> as;
  __shared__ double s_sq[kNW];
  __shared__ float s_bv[kNW];
  __shared__ int s_bi[kNW];
  __shared__ int s_cnt, s_flag, s_tok;
  __shared__ uint32_t s_sel[3];
  const GeoTable& gt = g_geo;
  __shared__ float s_xown[kMaxOwnRows];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  Smem sm;
  sm.base = smem;
  sm.p = &p;
  FillTables(p);
  __syncthreads();

  const int64_t pos0 = *p.pos;
  int tok = *p.tok;

  Ring rg;
  rg.R = p.ring;
  rg.base = smem + static_cast<size_t>(warp) * p.ring * p.slot;
  rg.bars = reinterpret_cast<uint64_t*>(smem + sm.plan().bars) + warp * p.ring;
  rg.kc = rg.ki = 0;
  rg.cs = rg.is = 0;
  rg.cpar = 0u;
  rg.bad = false;
  rg.cur.step = 0;
  rg.cur.layer = 0;
  rg.cur.ri = 0;
  rg.cur.j = 0;
  rg.cur.n = 0;
  rg.cur.bytes = 0;
  rg.cur.src = nullptr;
  rg.cur.c0 = 0;
  rg.step = 0;
  if (lane == 0) {
    for (int i = 0; i < rg.R; ++i) dev::MbarInit(rg.bars + i, 1);
    dev::MbarInitFence();
    EnterRun(p, gt, rg.cur, pos0, warp);
    NextRun(p, gt, rg.cur, pos0, warp);
    RingPump(rg, p, gt, pos0, warp);
  }
  __syncwarp();

  __shared__ PhaseClock clk;  // thread 0's timeline (trace only)
  if (p.trace.rec != nullptr && tid == 0) {
    clk.gt0 = dev::GlobalTimer();
    clk.ck0 = Clock64();
    clk.t_prev = clk.gt0;
    clk.t_ready = 0;
    for (int k = 0; k < kMarks; ++k) clk.mk[k] = 0;
  }
  const uint32_t n_phase = 5u * static_cast<uint32_t>(p.n_layers) + 2u;
  int steps = 0;
  bool alive = true;
  uint32_t tick_base = 0;  // tickets taken per KV head before the current attention phase
  for (int step = 0; step < p.n_steps && alive; ++step) {
    const int64_t pos = pos0 + step;
    const uint32_t id0 = static_cast<uint32_t>(step) * n_phase;
    if (blockIdx.x == 0 && tid == 0) p.out_ids[pos] = tok;
    // this step's attention units may be requested now (the previous step
    // wrote its cache rows before the barriers that led here)
    rg.step = step;
    if (lane == 0) RingPump(rg, p, gt, pos0, warp);
    // the rows of x this block owns in the o / down phases start as the
    // embedding of the forwarded token
    {
      const Geo& go = gt.g[kO][0];
      for (int r = tid; r < (go.t1 - go.t0) * kTile; r += kNT) s_xown[r] = dev::DeqElem(p.embd, tok, go.t0 * kTile + r);
    }
    // Phases of a layer meet through tagged words, not barriers; a block only
    // synchronises its own threads between phases (shared memory is reused).
    // One call site per phase kind keeps a single copy of the matvec code,
    // which stays in the instruction cache from phase to phase.
#pragma unroll 1
    for (uint32_t q = 0; q + 1u < n_phase; ++q) {
      const int l = static_cast<int>(q / 5u), ph = static_cast<int>(q - 5u * static_cast<uint32_t>(l));
      if (l < p.n_layers && ph == 1) {
        const uint32_t se = static_cast<uint32_t>(EffSplits(p, pos));
        AttnPhase<G>(p, gt, l, step, pos0, pos, tick_base + se - 1u, rg, sm, clk, as);
        tick_base += se;  // every active block of each head took one ticket
      } else {
        const int kind = l == p.n_layers ? kLm : (ph == 0 ? kQkv : (ph == 2 ? kO : (ph == 3 ? kGu : kDown)));
        MvPhase<G>(p, gt, kind, l < p.n_layers ? l : p.n_layers - 1, step, pos0, pos, tok, rg, sm, clk, s_xown,
                   s_sq, s_bv, s_bi, &s_cnt, s_sel);
      }
      TraceEnd(p, clk, id0 + q);
      if (q + 2u < n_phase) __syncthreads();
    }
    if (!(alive = GridBarrier(p, &s_flag))) break;
    TraceReady(p, clk);

    // ---- sample the next token (counter = pos + 1); every block gets it
    int next = -1;
    if (p.mode == 0) {
      float bv = -FLT_MAX;
      int bi = INT_MAX;
      if (p.tp > 0) {
        const uint32_t tag_lm = TagOf(p, step, p.n_layers - 1, kLm);
        const uint64_t* mine = p.xpeer[p.tp_rank];
        for (int i = tid; i < p.tp * static_cast<int>(gridDim.x); i += kNT) {
          const size_t off = XAm(p, 0, 0) + 2 * static_cast<size_t>(i);  // i = rank * grid + block
          const float v = ValOf(WaitPeer(p, mine + off, tag_lm));
          const int ix = static_cast<int>(static_cast<uint32_t>(WaitPeer(p, mine + off + 1, tag_lm)));
          if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
          }
        }
      } else {
        for (int i = tid; i < static_cast<int>(gridDim.x); i += kNT) {
          const float v = __ldcg(p.am_val + i);
          const int ix = __ldcg(p.am_idx + i);
          if (v > bv || (v == bv && ix < bi)) {
            bv = v;
            bi = ix;
          }
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
        for (int i = 1; i < kNW; ++i) {
          if (s_bv[i] > s_bv[0] || (s_bv[i] == s_bv[0] && s_bi[i] < s_bi[0])) {
            s_bv[0] = s_bv[i];
            s_bi[0] = s_bi[i];
          }
        }
        s_tok = s_bi[0] == INT_MAX ? 0 : s_bi[0];
      }
      __syncthreads();
      next = s_tok;
    } else {
      if (p.mode == 1 && p.tp > 0) {
        next = TpSample(p, step, pos, sm, [&](int k) { TraceMark(p, clk, k); });
        if (next < 0) {
          // every block of every rank alike: the launch ends after this step
          // and the host samples the next token from the gathered row
          if (blockIdx.x == 0 && tid == 0) p.steps_done[1] = 1;
          steps = step + 1;
          break;
        }
      } else if (p.mode == 1) {
        next = smp::SmallSample<kNT>(p.cand_val, p.cand_idx, p.cand_cnt, static_cast<int>(gridDim.x), p.temperature,
                                     p.top_k, p.top_p, p.seed, pos + 1, sm.scratch(), kSmallCap,
                                     [&](int k) { TraceMark(p, clk, k); });
      }
      if (next < 0) {  // the same decision in every block
        if (blockIdx.x == 0) {
          const int t = smp::GeneralSample<kNT>(p.logits, p.vocab, p.temperature, p.top_k, p.top_p, p.seed, pos + 1,
                                                p.probs);
          if (tid == 0) p.tok[0] = t;
        }
        if (!(alive = GridBarrier(p, &s_flag))) break;
        if (tid == 0) s_tok = __ldcg(p.tok);
        __syncthreads();
        next = s_tok;
      }
    }
    TraceEnd(p, clk, id0 + n_phase - 1u);
    steps = step + 1;
    bool is_stop = false;
    for (int i = 0; i < p.n_stop; ++i) is_stop = is_stop || p.stop[i] == tok;
    tok = next;
    if (is_stop) break;
  }

  // ---- drain: copies still in flight into this warp's ring land before exit
  if (lane == 0) {
    for (uint32_t k = rg.kc; k < rg.ki; ++k) {
      const uint32_t slot = k % static_cast<uint32_t>(rg.R);
      if (!dev::MbarWait(rg.bars + slot, (k / static_cast<uint32_t>(rg.R)) & 1u)) atomicOr(p.err, 1u);
    }
  }
  if (p.trace.rec != nullptr && tid == 0) {
    const uint64_t n = static_cast<uint64_t>(steps) * (5u * p.n_layers + 2u) * gridDim.x * (1 + kMarks);
    atomicMax(p.trace.count, static_cast<uint32_t>(n < p.trace.cap ? n : p.trace.cap));
  }
  if (blockIdx.x == 0 && tid == 0) {
    *p.pos = pos0 + steps;
    *p.tok = tok;
    *p.steps_done = steps;
  }
}

using LoopFn = void (*)(const LoopParams);

LoopFn PickLoop(int group) {
  switch (group) {
    case 2: return DecodeLoopKernel<2>;
    case 4: return DecodeLoopKernel<4>;
  }
  Throw("decode loop: group size %d is not built (2 and 4 are)", group);
}

constexpr int kSmemMax = 227 * 1024;

}  // namespace

bool LoopSupportsGroup(int group) { return group == 2 || group == 4; }

size_t LoopExchangeWords(int hidden, int grid) {
  return static_cast<size_t>(2 * kLoopMaxTp) * (hidden + grid) + static_cast<size_t>(kLoopMaxTp) * kXCandWords;
}

size_t LoopPartialWords(int n_kv, int group, int splits) {
  return static_cast<size_t>(n_kv) * splits * RecWords(group);
}

uint32_t LoopTagsPerLaunch(int n_layers, int n_steps) {
  return static_cast<uint32_t>(n_steps) * static_cast<uint32_t>(5 * n_layers + 2) + 2u;
}

int LoopSplits(int n_kv, int num_sms, int64_t max_seq) {
  const int64_t by_blocks = num_sms / std::max(1, n_kv);
  const int64_t by_len = (max_seq + 4 * kChunk - 1) / (4 * kChunk);
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({by_blocks, by_len, 64})));
}

void PrepareLoopKernels(int num_sms) {
  (void)num_sms;
  for (int g : {2, 4}) {
    // static + dynamic shared memory of a block may not exceed the opt-in limit
    cudaFuncAttributes fa;
    RPGB_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(PickLoop(g))));
    RPGB_CUDA(cudaFuncSetAttribute(PickLoop(g), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSmemMax - static_cast<int>(fa.sharedSizeBytes)));
  }
}

void LaunchDecodeLoop(const LoopParams& in, int group, int num_sms, cudaStream_t s) {
  LoopParams p = in;
  const LoopFn fn = PickLoop(group);
  RPGB_CHECK(p.n_steps > 0, "decode loop: no steps");
  RPGB_CHECK(p.n_stop >= 0 && p.n_stop <= kLoopMaxStop, "decode loop: at most %d stop ids", kLoopMaxStop);
  const int qd = p.n_heads * kD;
  RPGB_CHECK((p.hidden / kTile + num_sms - 1) / num_sms * kTile <= kMaxOwnRows,
             "decode loop: a block would own more than %d rows of x", kMaxOwnRows);
  RPGB_CHECK(p.llx != nullptr && p.llqkv != nullptr && p.llh != nullptr && p.llrec != nullptr &&
                 p.llattn != nullptr && p.tickets != nullptr,
             "decode loop: tagged buffers missing");
  RPGB_CHECK(p.n_layers >= 1 && p.n_layers <= kMaxLayers, "decode loop: %d layers (at most %d)", p.n_layers,
             kMaxLayers);
  if (p.tp > 0) {
    RPGB_CHECK(p.tp <= kLoopMaxTp && p.tp_rank >= 0 && p.tp_rank < p.tp, "decode loop: rank %d of %d", p.tp_rank,
               p.tp);
    RPGB_CHECK(p.mode == 0 || (p.mode == 1 && p.top_k < p.lm_head.rows && num_sms >= p.tp),
               "decode loop: tensor parallel decode is greedy or the fast sampler (1 < top_k <= %d)", kFastTopK);
    for (int k = 0; k < p.tp; ++k) RPGB_CHECK(p.xpeer[k] != nullptr, "decode loop: rank %d's buffer missing", k);
  }
  p.nb_max = std::max({p.hidden, qd, p.ffn}) / 256;
  p.x_max = std::max(p.hidden, qd);
  // most tiles of one block over the phases' row counts
  const int kvd = p.n_kv * kD;
  p.max_tiles = 0;
  for (const int rows : {qd + 2 * kvd, p.hidden, 2 * p.ffn, p.lm_head.rows}) {
    RPGB_CHECK(rows % kTile == 0, "decode loop: %d rows are not a multiple of %d", rows, kTile);
    p.max_tiles = std::max(p.max_tiles, (rows / kTile + num_sms - 1) / num_sms);
  }
  p.scratch_bytes = static_cast<int32_t>(ScratchBytes(p.nb_max, p.x_max, group, p.n_kv, p.splits));
  cudaFuncAttributes fa;
  RPGB_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(fn)));
  RPGB_CHECK(p.slot >= 2048 && p.slot % 16 == 0 && p.slot <= 8192, "decode loop: slot of %d bytes", p.slot);
  RPGB_CHECK(std::max({p.hidden, p.n_heads * kD, p.ffn}) / 256 <= kMaxSb, "decode loop: inputs wider than %d",
             kMaxSb * 256);
  const size_t fixed = MakePlan(0, p.slot, p.nb_max, p.x_max, p.scratch_bytes, p.max_tiles).total;
  const size_t avail = static_cast<size_t>(kSmemMax) - fa.sharedSizeBytes;
  RPGB_CHECK(avail > fixed, "decode loop: shared memory plan does not fit");
  const int ring = static_cast<int>((avail - fixed) / (static_cast<size_t>(kNW) * (p.slot + 8)));
  RPGB_CHECK(ring >= 2, "decode loop: room for only %d ring slots per warp", ring);
  p.ring = std::min(ring, kMaxRing);
  const size_t total = MakePlan(p.ring, p.slot, p.nb_max, p.x_max, p.scratch_bytes, p.max_tiles).total;
  if (p.mode == 1) {
    // the candidate slices are the blocks' lm_head rows
    RPGB_CHECK(num_sms <= kCandBlocks && p.max_tiles * kTile <= kSliceRows, "decode loop: fast sampler geometry");
  }
  int per_sm = 0;
  RPGB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kNT, total));
  RPGB_CHECK(per_sm >= 1, "decode loop: a block does not fit on an SM (%zu bytes of shared memory)", total);
  RPGB_CUDA(cudaMemsetAsync(p.bar, 0, sizeof(unsigned), s));
  RPGB_CUDA(cudaMemsetAsync(p.tickets, 0, sizeof(uint32_t) * p.n_kv, s));
  void* args[] = {&p};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kNT);
  cfg.dynamicSmemBytes = total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RPGB_CUDA(cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(fn), args));
  CountLaunches(1);
}

}  // namespace rpgb
