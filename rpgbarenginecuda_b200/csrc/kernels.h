// kernels.h -- host-side launchers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "model.h"

namespace rpgb {

// Process-wide count of kernel launches issued by this library (graph nodes
// count once per replay, added by the engine when it launches a graph).
void CountLaunches(int64_t n);
int64_t LaunchCount();

// Optional device-side timeline: when `rec` is set, thread 0 of every block
// appends {launch id, block, start, ready (after the programmatic-dependency
// wait), end} in %globaltimer nanoseconds.  Used by the trace entry point to
// see the real overlap of the launches inside a decode-step graph.
struct TraceRec {
  uint32_t id, block;
  uint64_t t_start, t_ready, t_end;
};
struct Trace {
  TraceRec* rec = nullptr;
  uint32_t* count = nullptr;
  uint32_t cap = 0;
  int32_t id = -1;
};

// ------------------------------------------------------------------ decode matvec (n = 1)
//
// out = W x with W one to three row segments of the same width (the q, k and v
// projections run as one launch).  Prologue: optional RMSNorm of x.  Epilogue:
//   kStore   out[r] = acc
//   kResid   out[r] = resid[r] + acc              (attn_o, ffn_down: x += W h)
//   kSilu    rows interleaved gate/up: out[i] = silu(acc[2i]) * acc[2i+1]
//   kArgmax  logits[r] = acc, plus argmax (ties -> lowest index) -> *tok_out
enum class Epi : int { kStore = 0, kResid = 1, kSilu = 2, kArgmax = 3 };

struct MvSeg {
  DevMat w;
  int32_t out_off = 0;  // first output row of the segment (a multiple of 16)
};

struct MvParams {
  MvSeg seg[3];
  int32_t n_seg = 1;
  int32_t total_rows = 0;
  const float* x = nullptr;
  const float* norm_w = nullptr;  // non-null: RMSNorm prologue
  float eps = 1e-6f;
  float* out = nullptr;
  const float* resid = nullptr;
  // kArgmax bookkeeping
  float* part_val = nullptr;
  int32_t* part_idx = nullptr;
  uint32_t* ticket = nullptr;
  int32_t* tok_out = nullptr;
  int64_t* pos = nullptr;  // incremented by pos_bump by the reducing block
  int32_t pos_bump = 0;
  unsigned* err = nullptr;  // set to nonzero if a bounded device wait gave up
  // launch geometry, filled in by LaunchMatvec
  int32_t n_tiles = 0, ring = 0, slot_bytes = 0, max_tiles = 0;
  Trace trace;
};

// Sets the dynamic shared-memory limits of every kernel instantiation on the
// current device.  Called once per device before any launch or graph capture
// (cudaFuncSetAttribute cannot be recorded into a graph).
void PrepareMatvecKernels();
void PrepareSampleKernels();

// The tile shape is fixed by the layout (16 rows per warp fragment); the
// rows_per_warp argument is kept for call-site compatibility.  `pdl`: launch
// with programmatic dependent launch (see launch.h).
void LaunchMatvec(const MvParams& p, Epi epi, int rows_per_warp, int num_sms, cudaStream_t s, bool pdl = false);
// Scratch sizes needed by kArgmax for a given launch.
int MatvecGrid(int total_rows, int rows_per_warp, int num_sms);

// out[t][r] = sum_c W[r][c] x[t][c] for a few tokens (k_matvec_n.cu): the
// decode matvec's integer tensor-core units applied to every token of a pass
// while each weight unit is in shared memory.
struct MvnParams {
  DevMat w;
  const float* x = nullptr;  // [n_tok][ldx], rows 16-byte aligned
  float* out = nullptr;      // [n_tok][ldo]
  int32_t n_tok = 0, ldx = 0, ldo = 0;
  // epilogue: kStore out[t][out_off + r] = v; kResid out[t][r] += v (the
  // residual stream in place); kSilu rows 2i / 2i+1 (gate / up) give
  // out[t][i] = silu(gate) * up
  int32_t out_off = 0;
  Epi epi = Epi::kStore;
  unsigned* err = nullptr;  // set to nonzero if a bounded device wait gave up
  // launch geometry, filled in by LaunchMatvecTokens
  int32_t ring = 0, slot_bytes = 0, max_tiles = 0, tp = 0;
};
void PrepareMatvecTokensKernels();
void LaunchMatvecTokens(const MvnParams& p, int num_sms, cudaStream_t s, bool pdl = false);

// ------------------------------------------------------------------ embedding

// x[t, :] = dequant(embd row tok[t]); if out_ids != nullptr also out_ids[*pos + t] = tok[t].
void LaunchEmbed(const DevMat& embd, const int32_t* tok, int n_tok, float* x, const int64_t* pos,
                 int32_t* out_ids, cudaStream_t s, bool pdl = false, const Trace& trace = Trace());

// dst[i] = dequant(W row `row`, element i) for a whole row (bit-exact dequant entry).
void LaunchDequantRows(const DevMat& w, int64_t row0, int64_t n_rows, float* dst, cudaStream_t s);

// ------------------------------------------------------------------ attention

struct AttnParams {
  const float* q = nullptr;  // decode: raw qkv row; prefill: normalised + rotated q [n][q_dim]
  int32_t q_stride = 0;      // floats between consecutive tokens in q
  const float* k_raw = nullptr;  // decode only: raw k / v rows of the current token
  const float* v_raw = nullptr;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  const float* rope = nullptr;
  float eps = 1e-6f;
  __half* kc = nullptr;  // layer base, [n_kv][max_seq][128]
  __half* vc = nullptr;
  int32_t max_seq = 0;
  const int64_t* pos = nullptr;  // position of query 0
  int32_t n_heads = 0, n_kv = 0;
  float scale = 0.f;
  float* out = nullptr;  // [n][q_dim]
  float* part = nullptr;
  uint32_t* ticket = nullptr;  // [n_kv]
  int32_t n_splits = 1;
  int32_t fused = 0;  // 1: decode (norm + rope + cache write of the current token inside)
  unsigned* err = nullptr;  // decode: set when a bounded wait for the staged K/V gave up
  Trace trace;
};
// Decode (fused, n_queries == 1) uses one block per (split, KV head); a split
// owns a run of 128-position stages whose cached K/V rows are staged into
// shared memory by TMA (the first before the programmatic wait).  n_splits
// bounds the block count (about one block per SM); at most kMaxAttnSplits.
constexpr int kAttnSplitPositions = 128;
constexpr int kMaxAttnSplits = 64;
constexpr int kMaxAttnCluster = 8;  // decode: the splits of one KV head form one thread-block cluster
void LaunchAttention(const AttnParams& p, int n_queries, cudaStream_t s, bool pdl = false);
void PrepareAttentionKernels();
size_t AttentionPartialFloats(int n_kv, int group, int n_splits);
// Prefill attention on the tensor cores (k_flash.cu): q = p.q (normalised,
// rotated, stride p.q_stride), queries at positions pos0 .. pos0 + n - 1 over
// the layer's cache p.kc / p.vc, out = p.out [n][q_dim]; p.err receives
// bounded-wait failures.  For head_dim 128 and group sizes 1, 2, 4, 8.
bool FlashSupports(int group, int head_dim);
// Few query tiles (an appended turn at a long context) leave most SMs idle;
// then the key range of each (query tile, KV head) is split over up to
// kMaxFlashSplits blocks whose partial outputs p.part (at least
// FlashSplitFloats floats; null = never split) are merged by a second launch.
constexpr int kMaxFlashSplits = 16;
size_t FlashSplitFloats(int n_heads, int n_kv, int num_sms);
void LaunchFlashPrefill(const AttnParams& p, int n_queries, int64_t pos0, int num_sms, cudaStream_t s);
void PrepareFlashKernels();

// Prefill helpers: per-head RMSNorm + RoPE for q and k, fp16 cache write of k and v.
void LaunchQkRopeKv(const float* qkv, int n_tok, int q_dim, int kv_dim, const float* q_norm,
                    const float* k_norm, const float* rope, float eps, const int64_t* pos0, __half* kc,
                    __half* vc, int32_t max_seq, int n_heads, int n_kv, float* q_out, cudaStream_t s);

// Row-wise RMSNorm (double sum of squares, as src/kernels_gpu.cu:564-591):
// the normalised rows in FP32 (out) and/or as the fp16 hi/lo terms of the
// tensor-core GEMM's activation operand (hi, lo: [n_rows][n] each).
void LaunchRmsNormRows(const float* x, const float* w, int n_rows, int n, float eps, float* out, cudaStream_t s,
                       __half* hi = nullptr, __half* lo = nullptr);

// ------------------------------------------------------------------ prefill GEMM
struct GemmParams {
  DevMat w;
  const float* X = nullptr;  // [n][ldx]
  int32_t n_tok = 0, ldx = 0;
  float* out = nullptr;
  int32_t ldo = 0, out_off = 0;
  const float* resid = nullptr;
  int32_t ldr = 0;
  // tensor-core path (k_tcgemm.cu): fp16 operand scratch of at least
  // TcGemmScratchHalves(rows, n_tok, cols, w.wh != nullptr) halves, and an
  // error word.  With w.wh / w.wl set the weights are read from that fp16
  // copy and w.q may be null (the fused q|k|v matrix of a layer).
  __half* tc_scratch = nullptr;
  size_t tc_scratch_halves = 0;
  unsigned* err = nullptr;
  // split-K for GEMMs with few output tiles (short prompts, appended turns):
  // a float buffer for the partial tiles (TcGemmPartFloats(num_sms) is
  // enough for any shape; null = no split) and the SM count to fill
  float* part = nullptr;
  size_t part_floats = 0;
  int32_t num_sms = 0;
  // the activations already split into fp16 terms ([n][cols] each, from
  // LaunchRmsNormRows): the tensor-core path then skips its own split
  const __half* xh = nullptr;
  const __half* xl = nullptr;
  // SiLU epilogue of the tensor-core path: write SiLU(g) * u as its fp16
  // hi/lo terms ([n][ldo] each, the values SplitKernel would make) instead
  // of FP32 out, to be the next GEMM's xh / xl
  __half* out_h = nullptr;
  __half* out_l = nullptr;
};
// Prompts of at least kTcMinTokens tokens (and weight rows a multiple of 128)
// run on the tcgen05 GEMM when scratch is given; others on the FP32 SIMT tile.
constexpr int kTcMinTokens = 16;
void LaunchGemm(const GemmParams& p, Epi epi, cudaStream_t s);
void LaunchTcGemm(const GemmParams& p, Epi epi, __half* scratch, size_t scratch_halves, cudaStream_t s);
// fp16 operand scratch of one GEMM: the activations' hi/lo terms, plus the
// weights' hi/lo expansion unless the matrix carries its own (w.wh, w.wl)
size_t TcGemmScratchHalves(int64_t rows, int64_t n_tok, int K, bool has_wh = false);
// W (repacked) -> hi, lo [rows][cols] fp16 with hi + lo the bit-exact
// dequantised value to ~22 bits (the prefill GEMM's weight operands)
void LaunchDequantSplit(const DevMat& w, __half* hi, __half* lo, cudaStream_t s);
// Splits of the K range the GEMM uses for this shape (1 = none): with fewer
// 128 x 128 output tiles than half the SMs, enough to fill the SMs with at
// least four 64-column k-slices each, bounded by the partial buffer.
int TcGemmSplits(int64_t rows, int64_t n_tok, int K, int num_sms, size_t part_floats);
size_t TcGemmPartFloats(int num_sms);
void PrepareTcGemmKernels();

// ------------------------------------------------------------------ sampler
struct SampleParams {
  const float* logits = nullptr;
  int32_t n = 0;
  float temperature = 0.f;
  int32_t top_k = 0;
  float top_p = 1.f;
  uint64_t seed = 0;
  int64_t* pos = nullptr;  // counter = *pos + pos_bump; then *pos += pos_bump
  int32_t pos_bump = 0;
  const int64_t* counter_override = nullptr;  // optional explicit counter
  float* probs = nullptr;  // [n] scratch (also the filtered distribution output)
  int32_t* tok_out = nullptr;
  uint64_t* fixed_hist = nullptr;  // scratch for the general path
  // fast path scratch
  float* cand_val = nullptr;
  int32_t* cand_idx = nullptr;
  int32_t* cand_cnt = nullptr;
  int32_t* flag = nullptr;  // fast path result flag (1 = done)
  Trace trace;  // id of the first launch; the sampler's launches use id, id + 1, ...
};
// Fast path (1 < top_k <= kFastTopK, T > 0): candidates + one small block.  Falls
// back to the general kernel on the device if a block overflowed.
constexpr int kFastTopK = 64;
constexpr int kCandBlocks = 148;
void LaunchSample(const SampleParams& p, bool want_probs, cudaStream_t s, bool pdl = false);

// ------------------------------------------------------------------ decode loop
//
// n_steps decode steps in one cooperative launch of one block per SM (see
// k_step.cu).  Step i forwards token *tok at position pos = *pos (+ i): the
// token is recorded at out_ids[pos], the step's logits land in `logits`, the
// next token is sampled with counter pos + 1.  The loop ends after n_steps
// steps or after a step that forwarded one of the n_stop stop ids; then *pos,
// *tok (the last sampled token) and *steps_done are written.
struct LoopParams {
  const DevLayer* layers = nullptr;  // device array [n_layers]
  int32_t n_layers = 0;
  DevMat embd, lm_head;
  const float* out_norm = nullptr;
  const float* rope = nullptr;
  int32_t hidden = 0, n_heads = 0, n_kv = 0, ffn = 0, vocab = 0, max_seq = 0;
  float eps = 1e-6f, scale = 0.f;
  __half* kc = nullptr;  // [layer][kv_head][max_seq][128]
  __half* vc = nullptr;
  int64_t layer_elems = 0;
  int64_t v_minus_k = 0;  // (char*)vc - (char*)kc
  // Tagged 64-bit words {float bits, tag} passed between the phases of a layer
  // (see k_step.cu): x [hidden], q|k|v [q_dim + 2 kv_dim], SiLU(g)*u [ffn],
  // attention split records [n_kv][splits][LoopRecordWords(group)].
  uint64_t *llx = nullptr, *llqkv = nullptr, *llh = nullptr, *llrec = nullptr;
  uint64_t* llattn = nullptr;     // merged attention output [q_dim]
  uint32_t* tickets = nullptr;    // [n_kv]: blocks of each head done with the attention phase
  uint32_t epoch0 = 1;  // tags of this launch start above it; strictly increasing across launches
  float *logits = nullptr, *probs = nullptr;
  // optional [n_steps][vocab]: step i's logits row is also stored at
  // step_logits + i * vocab (parity checks of multi-step launches)
  float* step_logits = nullptr;
  int64_t* pos = nullptr;
  int32_t* tok = nullptr;
  int32_t* out_ids = nullptr;
  // sampling: mode 0 argmax, 1 candidate fast path, 2 general block
  int32_t mode = 0;
  float temperature = 0.f, top_p = 1.f;
  int32_t top_k = 0;
  uint64_t seed = 0;
  float* cand_val = nullptr;
  int32_t* cand_idx = nullptr;
  int32_t* cand_cnt = nullptr;
  float* am_val = nullptr;
  int32_t* am_idx = nullptr;
  // control
  int32_t n_steps = 1;
  const int32_t* stop = nullptr;  // device [n_stop]
  int32_t n_stop = 0;
  int32_t* steps_done = nullptr;  // [2]: steps run; 1 when the host must sample the next token
  unsigned* bar = nullptr;  // grid barrier word
  unsigned* err = nullptr;  // nonzero after a bounded wait gave up
  int32_t splits = 1;       // attention blocks per KV head
  // Failure path: polls of one tagged-word wait before it gives up (0: the
  // built-in limit), and a test hook that leaves one word of the first qkv
  // phase unpublished, so the attention phase's wait for it runs out
  // (RPGB_TEST_WAIT_LIMIT / RPGB_TEST_DROP_WORD, read by the host per launch).
  uint32_t ll_limit = 0;
  int32_t test_drop_word = 0;
  // shared-memory plan, filled in by the launcher
  int32_t ring = 0, max_tiles = 0, nb_max = 0, x_max = 0;
  int32_t slot = 0;  // ring slot bytes: the largest block group of the model's matrices
  int32_t scratch_bytes = 0;
  Trace trace;  // records carry id = step * (5 n_layers + 2) + phase
  double ns_per_cycle = 0.0;  // SM clock period, to turn cycle counts of the trace into nanoseconds
  // tensor parallel (tp >= 1; 0 = one GPU): the exchange buffer of every rank
  // (xpeer[tp_rank] is this rank's own; the others are peers' memory mapped
  // over NVLink), laid out by LoopExchangeWords.  lm_head holds vocabulary
  // rows [vocab0, vocab0 + lm_head.rows).
  int32_t tp = 0, tp_rank = 0, vocab0 = 0;
  uint64_t* xpeer[8] = {};
};
constexpr int kLoopMaxStop = 16;
constexpr int kLoopMaxTp = 8;
// Tagged words of a rank's exchange buffer: partial rows of attn_output and
// ffn_down from every rank ([2][kLoopMaxTp][hidden]) and the lm_head argmax
// of every rank's blocks ([kLoopMaxTp][grid][2]).
size_t LoopExchangeWords(int hidden, int grid);
// Tagged words of the attention split records for `splits` blocks per KV head.
size_t LoopPartialWords(int n_kv, int group, int splits);
// Tags one launch of n_steps steps consumes (the next launch's epoch0 is at least this much higher).
uint32_t LoopTagsPerLaunch(int n_layers, int n_steps);
// Attention blocks per KV head for a grid of num_sms blocks and contexts up to max_seq.
int LoopSplits(int n_kv, int num_sms, int64_t max_seq);
// Group sizes (q heads per KV head) the loop kernel is built for.
bool LoopSupportsGroup(int group);
void PrepareLoopKernels(int num_sms);
void LaunchDecodeLoop(const LoopParams& p, int group, int num_sms, cudaStream_t s);

}  // namespace rpgb
