// engine.h -- a decoding session: fp16 KV cache, scratch, stream, decode loop.
//
// Reference counterparts: GpuKvCache (src/kv_cache_gpu.h:50-100), GpuScratch
// (src/qwen3_gpu.h:79-98), GpuForwardFull (src/qwen3_gpu.cu:236-276),
// GpuGenerate / GenerateGraph / GenerateNoGraph (src/qwen3_gpu.cu:451-640).
//
// Differences by design:
//  * every session owns its stream, position counter and buffers (the
//    reference keeps a process-global stream and pos0 staging), so sessions on
//    several GPUs run concurrently;
//  * a generate call is one cooperative launch of the decode loop kernel
//    (k_step.cu) that runs every step on the device; the step graph (embedding
//    -> 5 fused launches per layer -> lm_head with a fused argmax or the
//    sampler, recorded once as a CUDA graph) remains for group sizes the loop
//    kernel is not built for and for tensor-parallel sampled decode;
//  * the sampled token, its position and the position counter never leave the
//    device inside the loop; the host reads the generated ids once per launch.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "kernels.h"
#include "model.h"

namespace rpgb {

struct SampleOpts {
  float temperature = 0.f;
  int32_t top_k = 0;
  float top_p = 1.f;
};

class Session {
 public:
  Session(const Model* m, int64_t max_seq);
  ~Session();
  Session(const Session&) = delete;
  Session& operator=(const Session&) = delete;

  const Model& model() const { return *m_; }
  int64_t len() const { return len_; }
  int64_t max_seq() const { return max_seq_; }
  void SetLen(int64_t n);
  cudaStream_t stream() const { return stream_; }

  // Appends tokens at positions len .. len+n-1 and leaves the logits of the
  // last position on the device (optionally copied to last_logits[vocab]).
  void Prefill(const int32_t* tokens, int64_t n, float* last_logits);

  // Samples from the current logits and forwards every returned token (stop
  // token included), exactly the reference's GpuGenerate loop.  Returns the
  // number of ids written to out.
  int Generate(const SampleOpts& opt, uint64_t seed, int32_t max_tokens, const int32_t* stop, int32_t n_stop,
               int32_t* out, float* step_logits);

  // Device pointers for instrumentation / tests.
  const float* logits_dev() const { return logits_; }
  int graph_launches() const { return graph_launches_; }
  bool graph_ready() const { return graph_ != nullptr || loop_ready_; }
  int kernels_per_step() const { return kernels_per_step_; }

  // Tensor parallel decode inside the loop kernel: every rank's session
  // exports its exchange buffer (a CUDA IPC handle, 64 bytes) and attaches
  // the handles of all ranks in rank order (collective; its own is used in
  // place).  Without it a tensor-parallel session decodes through the step
  // graph and NCCL.
  void TpHandle(uint8_t* out) const;
  void TpAttach(const uint8_t* handles);
  bool tp_attached() const { return tp_attached_; }

  // Device timeline of the decode-step launches (see Trace in kernels.h).
  // EnableTrace(cap) allocates room for `cap` records and re-records the step
  // graph with tracing on (cap 0 turns it off); TakeTrace copies the records
  // gathered so far and clears them.
  void EnableTrace(int32_t cap);
  int32_t TakeTrace(TraceRec* out, int32_t cap);

 private:
  void EnqueueStep(const SampleOpts& opt, uint64_t seed);
  // Prefill of fewer than kTcMinTokens tokens: out[t] = W x[t] per token with
  // the decode matvec (segments of w stacked at out_off; resid: out += W x).
  void RowwiseMatvec(const DevMat* w, const int* out_off, int n_seg, const float* x, int ldx, float* out, int ldo,
                     bool resid, Epi epi, int n_tok, cudaStream_t s);
  // Tensor parallel: out = W x (this rank's columns) into y, summed over the
  // group, then added to the residual x (n rows of hidden).
  void ReduceIntoResidual(float* x, float* y, int64_t n, cudaStream_t s);
  // Tensor parallel: gathers every rank's vocabulary rows of the logits.
  void GatherLogits(cudaStream_t s);
  int GenerateLoop(const SampleOpts& opt, uint64_t seed, int32_t max_tokens, const int32_t* stop, int32_t n_stop,
                   int32_t* out, float* step_logits, int64_t start);
  LoopParams MakeLoopParams(const SampleOpts& opt, uint64_t seed) const;
  int LoopMode(const SampleOpts& opt) const;
  void EnqueueSample(const SampleOpts& opt, uint64_t seed, int pos_bump, bool pdl = false, int32_t trace_id = -1);
  void EnsurePrefill(int64_t n);
  void DropGraph();

  const Model* m_;
  int64_t max_seq_ = 0;
  int64_t len_ = 0;
  bool logits_valid_ = false;
  cudaStream_t stream_ = nullptr;

  // KV cache [layer][kv_head][max_seq][128] fp16
  __half* kc_ = nullptr;
  __half* vc_ = nullptr;
  size_t layer_elems_ = 0;

  // decode state (device)
  uint8_t* dec_arena_ = nullptr;
  float *x_ = nullptr, *qkv_ = nullptr, *attn_ = nullptr, *h_ = nullptr, *logits_ = nullptr, *probs_ = nullptr;
  float* y_ = nullptr;  // tensor parallel: this rank's partial of attn_output / ffn_down, then the sum
  int64_t* pos_ = nullptr;
  int32_t* tok_ = nullptr;
  int32_t* out_ids_ = nullptr;  // [max_seq]: token forwarded at each position
  float* attn_part_ = nullptr;
  uint32_t* tickets_ = nullptr;  // [n_kv] attention + [1] argmax
  float* am_val_ = nullptr;
  int32_t* am_idx_ = nullptr;
  float* cand_val_ = nullptr;
  int32_t* cand_idx_ = nullptr;
  int32_t* cand_cnt_ = nullptr;
  int32_t* flag_ = nullptr;
  unsigned* err_ = nullptr;  // set by a bounded device wait that gave up
  int n_splits_ = 1;
  // decode loop kernel state
  unsigned* bar_ = nullptr;       // grid barrier word
  int32_t* steps_done_ = nullptr;
  int32_t* stop_dev_ = nullptr;   // [kLoopMaxStop]
  int32_t* loop_host_ = nullptr;  // pinned: steps done, host-sample request
  float* step_logits_dev_ = nullptr;  // [cap][vocab]: per-step logits of a loop launch (parity checks)
  int64_t step_logits_cap_ = 0;
  int loop_splits_ = 1;
  bool loop_ready_ = false;
  uint64_t* ll_ = nullptr;  // tagged words (x, qkv, ffn activation, attention records, merged attention)
  uint32_t* tickets_loop_ = nullptr;
  size_t ll_words_ = 0;
  uint32_t epoch_ = 1;      // first tag base of the next launch
  // tensor parallel: this rank's exchange buffer and every rank's (peers' by IPC)
  uint64_t* xbuf_ = nullptr;
  size_t xbuf_words_ = 0;
  uint64_t* xpeer_[kLoopMaxTp] = {};
  bool tp_attached_ = false;

  // prefill scratch (grow-only)
  int64_t pf_cap_ = 0;
  uint8_t* pf_arena_ = nullptr;
  float *pf_x_ = nullptr, *pf_xn_ = nullptr, *pf_qkv_ = nullptr, *pf_q_ = nullptr, *pf_attn_ = nullptr,
        *pf_h_ = nullptr, *pf_y_ = nullptr;
  float* pf_part_ = nullptr;  // key-split partials of the flash attention (appended turns)
  int32_t* pf_tok_ = nullptr;
  __half* pf_tc_ = nullptr;  // fp16 operands of the tensor-core GEMM
  size_t pf_tc_halves_ = 0;
  float* pf_gpart_ = nullptr;  // split-K partial tiles of the tensor-core GEMM
  size_t pf_gpart_floats_ = 0;
  __half* pf_xs_ = nullptr;  // normalised rows as fp16 hi / lo GEMM operands ([cap][hidden] each)
  int32_t* host_ids_ = nullptr;  // pinned staging
  int64_t host_ids_cap_ = 0;

  // decode graph
  cudaGraphExec_t graph_ = nullptr;
  SampleOpts graph_opt_;
  uint64_t graph_seed_ = 0;
  int graph_launches_ = 0;
  int kernels_per_step_ = 0;

  // timeline trace (off unless EnableTrace)
  TraceRec* trace_rec_ = nullptr;
  uint32_t* trace_count_ = nullptr;
  uint32_t trace_cap_ = 0;
  Trace NextTrace(int32_t* id) const {
    Trace t;
    if (trace_rec_ != nullptr) {
      t.rec = trace_rec_;
      t.count = trace_count_;
      t.cap = trace_cap_;
      t.id = (*id)++;
    }
    return t;
  }
};

}  // namespace rpgb
