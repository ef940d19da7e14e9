// engine.cu -- session state, prefill, decode step graph, generate loop.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "common.h"

namespace rpgb {

namespace {

constexpr size_t kAlign = 256;
size_t AlignUp(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Positions handled per attention split in decode; a graph is recorded once per
// session, so the split count is fixed from max_seq and short contexts simply
// leave the tail splits empty.
constexpr int kPositionsPerSplit = kAttnSplitPositions;

class Carver {
 public:
  void Add(size_t bytes) { total_ += AlignUp(bytes); }
  size_t total() const { return total_; }
  void Begin(uint8_t* base) {
    base_ = base;
    off_ = 0;
  }
  template <typename T>
  T* Take(size_t count) {
    T* p = reinterpret_cast<T*>(base_ + off_);
    off_ += AlignUp(count * sizeof(T));
    return p;
  }

 private:
  size_t total_ = 0, off_ = 0;
  uint8_t* base_ = nullptr;
};

bool SameOpts(const SampleOpts& a, const SampleOpts& b) {
  return a.temperature == b.temperature && a.top_k == b.top_k && a.top_p == b.top_p;
}

}  // namespace

Session::Session(const Model* m, int64_t max_seq) : m_(m), max_seq_(max_seq) {
  const ModelMeta& c = m->meta();
  RPGB_CHECK(max_seq > 0, "max_seq must be positive (got %lld)", static_cast<long long>(max_seq));
  RPGB_CHECK(max_seq <= m->rope_positions(), "max_seq %lld exceeds the %d positions of the RoPE table",
             static_cast<long long>(max_seq), m->rope_positions());
  RPGB_CUDA(cudaSetDevice(m->device()));
  RPGB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));

  layer_elems_ = static_cast<size_t>(c.n_kv_heads) * static_cast<size_t>(max_seq) * c.head_dim;
  const size_t kv_bytes = layer_elems_ * c.n_layers * sizeof(__half);
  RPGB_CUDA(cudaMalloc(&kc_, kv_bytes));
  RPGB_CUDA(cudaMalloc(&vc_, kv_bytes));
  // Positions >= len are never read, but zero the cache once so stale memory
  // from another allocation can never leak into a result.
  RPGB_CUDA(cudaMemsetAsync(kc_, 0, kv_bytes, stream_));
  RPGB_CUDA(cudaMemsetAsync(vc_, 0, kv_bytes, stream_));

  // about one attention block per SM at full length, never more stages than positions
  {
    const int64_t stages = (max_seq + kPositionsPerSplit - 1) / kPositionsPerSplit;
    const int64_t per_head = std::max(1, m->num_sms() / c.n_kv_heads);
    n_splits_ = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>({stages, per_head, kMaxAttnCluster})));
    // RPGB_ATTN_SPLITS caps the split count (more 128-position stages per
    // block); used by tests to exercise multi-stage blocks on short models.
    if (const char* e = std::getenv("RPGB_ATTN_SPLITS")) {
      const int cap = std::atoi(e);
      if (cap >= 1) n_splits_ = std::min(n_splits_, cap);
    }
  }
  loop_splits_ = LoopSplits(c.n_kv_heads, m->num_sms(), max_seq);
  if (const char* e = std::getenv("RPGB_ATTN_SPLITS")) {
    const int cap = std::atoi(e);
    if (cap >= 1) loop_splits_ = std::min(loop_splits_, cap);
  }
  const size_t part_floats = AttentionPartialFloats(c.n_kv_heads, c.group(), n_splits_);
  ll_words_ = static_cast<size_t>(c.hidden) + (c.q_dim() + 2 * c.kv_dim()) + c.ffn +
              LoopPartialWords(c.n_kv_heads, c.group(), loop_splits_) + c.q_dim();
  const int am_grid = std::max(MatvecGrid(c.vocab, 4, m->num_sms()), m->num_sms());
  const int qkv = c.q_dim() + 2 * c.kv_dim();
  Carver cv;
  cv.Add(sizeof(float) * c.hidden);   // x
  cv.Add(sizeof(float) * c.hidden);   // y
  cv.Add(sizeof(float) * qkv);        // qkv
  cv.Add(sizeof(float) * c.q_dim());  // attn
  cv.Add(sizeof(float) * c.ffn);      // h
  cv.Add(sizeof(float) * c.vocab);    // logits
  cv.Add(sizeof(float) * c.vocab);    // probs
  cv.Add(sizeof(int64_t));            // pos
  cv.Add(sizeof(int32_t));            // tok
  cv.Add(sizeof(int32_t) * (max_seq + 1));
  cv.Add(sizeof(float) * part_floats);
  cv.Add(sizeof(uint32_t) * (c.n_kv_heads + 1));
  cv.Add(sizeof(float) * am_grid);
  cv.Add(sizeof(int32_t) * am_grid);
  cv.Add(sizeof(float) * kCandBlocks * kFastTopK);
  cv.Add(sizeof(int32_t) * kCandBlocks * kFastTopK);
  cv.Add(sizeof(int32_t) * kCandBlocks);
  cv.Add(sizeof(int32_t));
  cv.Add(sizeof(unsigned));
  cv.Add(sizeof(unsigned));                   // grid barrier word
  cv.Add(sizeof(int32_t) * 2);                // steps done, host-sample request
  cv.Add(sizeof(int32_t) * kLoopMaxStop);     // stop ids
  cv.Add(sizeof(uint64_t) * ll_words_);       // tagged words of the decode loop
  cv.Add(sizeof(uint32_t) * c.n_kv_heads);    // attention tickets
  RPGB_CUDA(cudaMalloc(&dec_arena_, cv.total()));
  RPGB_CUDA(cudaMemsetAsync(dec_arena_, 0, cv.total(), stream_));
  cv.Begin(dec_arena_);
  x_ = cv.Take<float>(c.hidden);
  y_ = cv.Take<float>(c.hidden);
  qkv_ = cv.Take<float>(qkv);
  attn_ = cv.Take<float>(c.q_dim());
  h_ = cv.Take<float>(c.ffn);
  logits_ = cv.Take<float>(c.vocab);
  probs_ = cv.Take<float>(c.vocab);
  pos_ = cv.Take<int64_t>(1);
  tok_ = cv.Take<int32_t>(1);
  out_ids_ = cv.Take<int32_t>(max_seq + 1);
  attn_part_ = cv.Take<float>(part_floats);
  tickets_ = cv.Take<uint32_t>(c.n_kv_heads + 1);
  am_val_ = cv.Take<float>(am_grid);
  am_idx_ = cv.Take<int32_t>(am_grid);
  cand_val_ = cv.Take<float>(kCandBlocks * kFastTopK);
  cand_idx_ = cv.Take<int32_t>(kCandBlocks * kFastTopK);
  cand_cnt_ = cv.Take<int32_t>(kCandBlocks);
  flag_ = cv.Take<int32_t>(1);
  err_ = cv.Take<unsigned>(1);
  bar_ = cv.Take<unsigned>(1);
  steps_done_ = cv.Take<int32_t>(2);
  stop_dev_ = cv.Take<int32_t>(kLoopMaxStop);
  ll_ = cv.Take<uint64_t>(ll_words_);  // zeroed with the arena: tag 0 is never a valid tag
  tickets_loop_ = cv.Take<uint32_t>(c.n_kv_heads);
  RPGB_CUDA(cudaMallocHost(&loop_host_, sizeof(int32_t) * 2));
  if (m->tp() != nullptr) {  // its own allocation: the CUDA IPC handle covers exactly this buffer
    xbuf_words_ = LoopExchangeWords(c.hidden, m->num_sms());
    RPGB_CUDA(cudaMalloc(&xbuf_, sizeof(uint64_t) * xbuf_words_));
    RPGB_CUDA(cudaMemsetAsync(xbuf_, 0, sizeof(uint64_t) * xbuf_words_, stream_));
  }
  RPGB_CUDA(cudaStreamSynchronize(stream_));
}

void Session::TpHandle(uint8_t* out) const {
  RPGB_CHECK(xbuf_ != nullptr, "the session's model is not tensor parallel");
  cudaIpcMemHandle_t h;
  RPGB_CUDA(cudaSetDevice(m_->device()));
  RPGB_CUDA(cudaIpcGetMemHandle(&h, xbuf_));
  std::memcpy(out, &h, sizeof(h));
}

void Session::TpAttach(const uint8_t* handles) {
  RPGB_CHECK(xbuf_ != nullptr, "the session's model is not tensor parallel");
  RPGB_CHECK(!tp_attached_, "the session is attached already");
  const TpGroup& g = *m_->tp();
  RPGB_CHECK(g.size() <= kLoopMaxTp, "tensor parallel decode loop: at most %d ranks", kLoopMaxTp);
  RPGB_CUDA(cudaSetDevice(m_->device()));
  for (int k = 0; k < g.size(); ++k) {
    if (k == g.rank()) {
      xpeer_[k] = xbuf_;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + static_cast<size_t>(k) * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < k; ++j) {
        if (j != g.rank() && xpeer_[j] != nullptr) cudaIpcCloseMemHandle(xpeer_[j]);
        xpeer_[j] = nullptr;
      }
      Throw("tensor parallel: opening rank %d's exchange buffer failed: %s", k, cudaGetErrorString(e));
    }
    xpeer_[k] = static_cast<uint64_t*>(p);
  }
  tp_attached_ = true;
}

Session::~Session() {
  cudaSetDevice(m_->device());
  if (stream_ != nullptr) cudaStreamSynchronize(stream_);
  DropGraph();
  if (m_->tp() != nullptr) {
    for (int k = 0; k < kLoopMaxTp; ++k) {
      if (xpeer_[k] != nullptr && xpeer_[k] != xbuf_) cudaIpcCloseMemHandle(xpeer_[k]);
    }
  }
  cudaFree(xbuf_);
  cudaFree(kc_);
  cudaFree(vc_);
  cudaFree(dec_arena_);
  cudaFree(pf_arena_);
  cudaFree(trace_rec_);
  cudaFree(trace_count_);
  cudaFree(step_logits_dev_);
  if (host_ids_ != nullptr) cudaFreeHost(host_ids_);
  if (loop_host_ != nullptr) cudaFreeHost(loop_host_);
  if (stream_ != nullptr) cudaStreamDestroy(stream_);
}

void Session::DropGraph() {
  if (graph_ != nullptr) {
    cudaGraphExecDestroy(graph_);
    graph_ = nullptr;
  }
}

void Session::EnableTrace(int32_t cap) {
  RPGB_CHECK(cap >= 0 && cap <= (1 << 24), "trace capacity %d out of range", cap);
  RPGB_CUDA(cudaSetDevice(m_->device()));
  RPGB_CUDA(cudaStreamSynchronize(stream_));
  DropGraph();
  cudaFree(trace_rec_);
  cudaFree(trace_count_);
  cudaFree(step_logits_dev_);
  trace_rec_ = nullptr;
  trace_count_ = nullptr;
  trace_cap_ = 0;
  if (cap == 0) return;
  RPGB_CUDA(cudaMalloc(&trace_rec_, sizeof(TraceRec) * static_cast<size_t>(cap)));
  RPGB_CUDA(cudaMalloc(&trace_count_, sizeof(uint32_t)));
  RPGB_CUDA(cudaMemset(trace_count_, 0, sizeof(uint32_t)));
  trace_cap_ = static_cast<uint32_t>(cap);
}

int32_t Session::TakeTrace(TraceRec* out, int32_t cap) {
  if (trace_rec_ == nullptr) return 0;
  RPGB_CUDA(cudaSetDevice(m_->device()));
  RPGB_CUDA(cudaStreamSynchronize(stream_));
  uint32_t n = 0;
  RPGB_CUDA(cudaMemcpy(&n, trace_count_, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  n = std::min<uint32_t>(n, trace_cap_);
  const uint32_t m = std::min<uint32_t>(n, static_cast<uint32_t>(std::max(cap, 0)));
  if (m > 0) RPGB_CUDA(cudaMemcpy(out, trace_rec_, sizeof(TraceRec) * m, cudaMemcpyDeviceToHost));
  RPGB_CUDA(cudaMemset(trace_count_, 0, sizeof(uint32_t)));
  return static_cast<int32_t>(m);
}

void Session::SetLen(int64_t n) {
  RPGB_CHECK(n >= 0 && n <= max_seq_, "length %lld out of range [0, %lld]", static_cast<long long>(n),
             static_cast<long long>(max_seq_));
  if (n != len_) logits_valid_ = false;
  len_ = n;
}

void Session::EnsurePrefill(int64_t n) {
  if (n <= pf_cap_) return;
  const ModelMeta& c = m_->meta();
  int64_t cap = std::max<int64_t>(n, 64);
  cap = (cap + 63) / 64 * 64;
  Carver cv;
  const int qkv = c.q_dim() + 2 * c.kv_dim();
  cv.Add(sizeof(float) * cap * c.hidden);
  cv.Add(sizeof(float) * cap * c.hidden);
  cv.Add(sizeof(float) * cap * qkv);
  cv.Add(sizeof(float) * cap * c.q_dim());
  cv.Add(sizeof(float) * cap * c.q_dim());
  cv.Add(sizeof(float) * cap * c.ffn);
  cv.Add(sizeof(float) * (m_->tp() != nullptr ? cap * c.hidden : 0));
  const size_t split_floats =
      FlashSupports(c.group(), c.head_dim) ? FlashSplitFloats(c.n_heads, c.n_kv_heads, m_->num_sms()) : 0;
  cv.Add(sizeof(float) * split_floats);
  cv.Add(sizeof(int32_t) * cap);
  // fp16 operands of the tensor-core GEMM: the widest activations' hi/lo
  // terms, and the largest layer matrix's unless the model keeps fp16 copies
  const int64_t kmax = std::max<int64_t>(c.hidden, std::max<int64_t>(c.q_dim(), c.ffn));
  const int64_t wmax = m_->half_bytes() > 0 ? 0
                                            : std::max<int64_t>(static_cast<int64_t>(2) * c.ffn * c.hidden,
                                                                static_cast<int64_t>(c.q_dim()) * c.hidden);
  const size_t tc_halves = 2 * static_cast<size_t>(wmax) + 2 * static_cast<size_t>(cap) * kmax;
  cv.Add(sizeof(__half) * tc_halves);
  // split-K partial tiles: the few-tiles case, or two halves of the
  // hidden-size outputs (attn_output, ffn_down) of the whole prompt
  const size_t gpart_floats =
      std::max(TcGemmPartFloats(m_->num_sms()), 2 * static_cast<size_t>(cap) * static_cast<size_t>(c.hidden));
  cv.Add(sizeof(float) * gpart_floats);
  cv.Add(sizeof(__half) * 2 * cap * c.hidden);  // normalised rows as fp16 hi/lo GEMM operands
  RPGB_CUDA(cudaStreamSynchronize(stream_));
  cudaFree(pf_arena_);
  pf_arena_ = nullptr;
  RPGB_CUDA(cudaMalloc(&pf_arena_, cv.total()));
  cv.Begin(pf_arena_);
  pf_x_ = cv.Take<float>(cap * c.hidden);
  pf_xn_ = cv.Take<float>(cap * c.hidden);
  pf_qkv_ = cv.Take<float>(cap * qkv);
  pf_q_ = cv.Take<float>(cap * c.q_dim());
  pf_attn_ = cv.Take<float>(cap * c.q_dim());
  pf_h_ = cv.Take<float>(cap * c.ffn);
  pf_y_ = m_->tp() != nullptr ? cv.Take<float>(cap * c.hidden) : nullptr;
  pf_part_ = split_floats > 0 ? cv.Take<float>(split_floats) : nullptr;
  pf_tok_ = cv.Take<int32_t>(cap);
  pf_tc_ = cv.Take<__half>(tc_halves);
  pf_tc_halves_ = tc_halves;
  pf_gpart_ = cv.Take<float>(gpart_floats);
  pf_gpart_floats_ = gpart_floats;
  pf_xs_ = cv.Take<__half>(2 * cap * c.hidden);
  pf_cap_ = cap;
}

void Session::RowwiseMatvec(const DevMat* w, const int* out_off, int n_seg, const float* x, int ldx, float* out,
                            int ldo, bool resid, Epi epi, int n_tok, cudaStream_t s) {
  // one multi-token launch per matrix: its weights stream once per pass of
  // up to four tokens (k_matvec_n.cu)
  for (int i = 0; i < n_seg; ++i) {
    MvnParams p;
    p.w = w[i];
    p.x = x;
    p.out = out;
    p.n_tok = n_tok;
    p.ldx = ldx;
    p.ldo = ldo;
    p.out_off = out_off[i];
    p.epi = resid ? Epi::kResid : epi;
    p.err = err_;
    LaunchMatvecTokens(p, m_->num_sms(), s);
  }
}

void Session::Prefill(const int32_t* tokens, int64_t n, float* last_logits) {
  const ModelMeta& c = m_->meta();
  RPGB_CHECK(n > 0, "prompt is empty");
  RPGB_CHECK(len_ + n <= max_seq_, "position %lld exceeds the KV cache capacity %lld",
             static_cast<long long>(len_ + n), static_cast<long long>(max_seq_));
  for (int64_t t = 0; t < n; ++t) {
    RPGB_CHECK(tokens[t] >= 0 && tokens[t] < c.vocab, "token #%lld has id %d, out of range (vocab %d)",
               static_cast<long long>(t), tokens[t], c.vocab);
  }
  RPGB_CUDA(cudaSetDevice(m_->device()));
  EnsurePrefill(n);
  const cudaStream_t s = stream_;
  const int64_t pos0 = len_;
  RPGB_CUDA(cudaMemcpyAsync(pf_tok_, tokens, sizeof(int32_t) * n, cudaMemcpyHostToDevice, s));
  RPGB_CUDA(cudaMemcpyAsync(pos_, &pos0, sizeof(int64_t), cudaMemcpyHostToDevice, s));

  const int H = c.hidden, qd = c.q_dim(), kvd = c.kv_dim(), qkv = qd + 2 * kvd;
  const int nt = static_cast<int>(n);
  // Short prompts: GEMM tiles would leave most SMs idle (and the tensor-core
  // path would first expand every weight to fp16), so they run the
  // multi-token matvec: the decode matvec's units applied to up to four
  // tokens per pass while each weight unit is in shared memory.
  const bool rowwise = nt < kTcMinTokens;
  // the RMSNorm kernels write the GEMM's fp16 activation terms directly when
  // every GEMM reading their output runs on the tensor cores
  __half* xs_h = pf_xs_;
  __half* xs_l = pf_xs_ + static_cast<size_t>(pf_cap_) * H;
  LaunchEmbed(m_->embd(), pf_tok_, nt, pf_x_, nullptr, nullptr, s);
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m_->layers()[static_cast<size_t>(l)];
    __half* kc = kc_ + layer_elems_ * l;
    __half* vc = vc_ + layer_elems_ * l;
    const bool split_a = !rowwise && L.q.rows % 128 == 0 && L.k.rows % 128 == 0 && L.v.rows % 128 == 0;
    if (split_a) {
      LaunchRmsNormRows(pf_x_, L.attn_norm, nt, H, c.rms_eps, nullptr, s, xs_h, xs_l);
    } else {
      LaunchRmsNormRows(pf_x_, L.attn_norm, nt, H, c.rms_eps, pf_xn_, s);
    }
    if (rowwise) {
      const DevMat w3[3] = {L.q, L.k, L.v};
      const int off3[3] = {0, qd, qd + kvd};
      RowwiseMatvec(w3, off3, 3, pf_xn_, H, pf_qkv_, qkv, false, Epi::kStore, nt, s);
    } else {
      GemmParams g;
      g.tc_scratch = pf_tc_;
      g.tc_scratch_halves = pf_tc_halves_;
      g.part = pf_gpart_;
      g.part_floats = pf_gpart_floats_;
      g.num_sms = m_->num_sms();
      g.err = err_;
      g.X = pf_xn_;
      g.xh = split_a ? xs_h : nullptr;
      g.xl = split_a ? xs_l : nullptr;
      g.n_tok = nt;
      g.ldx = H;
      g.out = pf_qkv_;
      g.ldo = qkv;
      g.out_off = 0;
      if (L.qkv.wh != nullptr && L.qkv.rows % 128 == 0) {  // one GEMM over the fp16 [q; k; v] terms
        g.w = L.qkv;
        LaunchGemm(g, Epi::kStore, s);
      } else {
        g.w = L.q;
        LaunchGemm(g, Epi::kStore, s);
        g.w = L.k;
        g.out_off = qd;
        LaunchGemm(g, Epi::kStore, s);
        g.w = L.v;
        g.out_off = qd + kvd;
        LaunchGemm(g, Epi::kStore, s);
      }
    }
    LaunchQkRopeKv(pf_qkv_, nt, qd, kvd, L.q_norm, L.k_norm, m_->rope(), c.rms_eps, pos_, kc, vc,
                   static_cast<int32_t>(max_seq_), c.n_heads, c.n_kv_heads, pf_q_, s);
    AttnParams a;
    a.q = pf_q_;
    a.q_stride = qd;
    a.kc = kc;
    a.vc = vc;
    a.max_seq = static_cast<int32_t>(max_seq_);
    a.pos = pos_;
    a.n_heads = c.n_heads;
    a.n_kv = c.n_kv_heads;
    a.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
    a.out = pf_attn_;
    a.n_splits = 1;
    a.fused = 0;
    a.err = err_;
    if (FlashSupports(c.group(), c.head_dim)) {
      a.part = pf_part_;
      LaunchFlashPrefill(a, nt, pos0, m_->num_sms(), s);
    } else {
      LaunchAttention(a, nt, s);
    }
    if (rowwise) {
      const int off0[1] = {0};
      if (m_->tp() != nullptr) {
        RowwiseMatvec(&L.o, off0, 1, pf_attn_, qd, pf_y_, H, false, Epi::kStore, nt, s);
        ReduceIntoResidual(pf_x_, pf_y_, n, s);
      } else {
        RowwiseMatvec(&L.o, off0, 1, pf_attn_, qd, pf_x_, H, true, Epi::kResid, nt, s);
      }
    } else {
      GemmParams o;
      o.tc_scratch = pf_tc_;
      o.tc_scratch_halves = pf_tc_halves_;
      o.part = pf_gpart_;
      o.part_floats = pf_gpart_floats_;
      o.num_sms = m_->num_sms();
      o.err = err_;
      o.w = L.o;
      o.X = pf_attn_;
      o.n_tok = nt;
      o.ldx = qd;
      o.ldo = H;
      if (m_->tp() != nullptr) {
        o.out = pf_y_;
        LaunchGemm(o, Epi::kStore, s);
        ReduceIntoResidual(pf_x_, pf_y_, n, s);
      } else {
        o.out = pf_x_;
        o.resid = pf_x_;
        o.ldr = H;
        LaunchGemm(o, Epi::kResid, s);
      }
    }
    const bool split_f = !rowwise && L.gateup.rows % 128 == 0;
    if (split_f) {
      LaunchRmsNormRows(pf_x_, L.ffn_norm, nt, H, c.rms_eps, nullptr, s, xs_h, xs_l);
    } else {
      LaunchRmsNormRows(pf_x_, L.ffn_norm, nt, H, c.rms_eps, pf_xn_, s);
    }
    if (rowwise) {
      const int off0[1] = {0};
      RowwiseMatvec(&L.gateup, off0, 1, pf_xn_, H, pf_h_, c.ffn, false, Epi::kSilu, nt, s);
      if (m_->tp() != nullptr) {
        RowwiseMatvec(&L.down, off0, 1, pf_h_, c.ffn, pf_y_, H, false, Epi::kStore, nt, s);
        ReduceIntoResidual(pf_x_, pf_y_, n, s);
      } else {
        RowwiseMatvec(&L.down, off0, 1, pf_h_, c.ffn, pf_x_, H, true, Epi::kResid, nt, s);
      }
      continue;
    }
    GemmParams gu;
    gu.tc_scratch = pf_tc_;
    gu.tc_scratch_halves = pf_tc_halves_;
    gu.part = pf_gpart_;
    gu.part_floats = pf_gpart_floats_;
    gu.num_sms = m_->num_sms();
    gu.err = err_;
    gu.w = L.gateup;
    gu.X = pf_xn_;
    gu.xh = split_f ? xs_h : nullptr;
    gu.xl = split_f ? xs_l : nullptr;
    gu.n_tok = nt;
    gu.ldx = H;
    gu.out = pf_h_;
    gu.ldo = c.ffn;
    // the gate/up epilogue writes ffn_down's fp16 operand terms into pf_h_'s
    // space (2 cap ffn halves) in place of the FP32 rows
    const bool split_d = split_f && L.down.rows % 128 == 0;
    __half* const hd_h = reinterpret_cast<__half*>(pf_h_);
    __half* const hd_l = hd_h + static_cast<size_t>(pf_cap_) * c.ffn;
    if (split_d) {
      gu.out_h = hd_h;
      gu.out_l = hd_l;
    }
    LaunchGemm(gu, Epi::kSilu, s);
    GemmParams dn;
    dn.tc_scratch = pf_tc_;
    dn.tc_scratch_halves = pf_tc_halves_;
    dn.part = pf_gpart_;
    dn.part_floats = pf_gpart_floats_;
    dn.num_sms = m_->num_sms();
    dn.err = err_;
    dn.w = L.down;
    dn.X = pf_h_;
    dn.xh = split_d ? hd_h : nullptr;
    dn.xl = split_d ? hd_l : nullptr;
    dn.n_tok = nt;
    dn.ldx = c.ffn;
    dn.ldo = H;
    if (m_->tp() != nullptr) {
      dn.out = pf_y_;
      LaunchGemm(dn, Epi::kStore, s);
      ReduceIntoResidual(pf_x_, pf_y_, n, s);
    } else {
      dn.out = pf_x_;
      dn.resid = pf_x_;
      dn.ldr = H;
      LaunchGemm(dn, Epi::kResid, s);
    }
  }
  // final norm + lm_head on the last position only (the reference computes all
  // rows and keeps the last one, src/qwen3_gpu.cu:163-170)
  MvParams mv;
  mv.seg[0].w = m_->lm_head();
  mv.n_seg = 1;
  mv.total_rows = m_->lm_head().rows;  // the vocabulary, or this rank's rows of it
  mv.x = pf_x_ + static_cast<int64_t>(n - 1) * H;
  mv.norm_w = m_->out_norm();
  mv.eps = c.rms_eps;
  mv.out = logits_ + m_->shard().vocab0;
  LaunchMatvec(mv, Epi::kStore, 4, m_->num_sms(), s);
  if (m_->tp() != nullptr) GatherLogits(s);
  if (last_logits != nullptr) {
    RPGB_CUDA(cudaMemcpyAsync(last_logits, logits_, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s));
  }
  unsigned err = 0;
  RPGB_CUDA(cudaMemcpyAsync(&err, err_, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
  RPGB_CUDA(cudaStreamSynchronize(s));
  if (err != 0) {
    RPGB_CUDA(cudaMemset(err_, 0, sizeof(unsigned)));
    logits_valid_ = false;
    Throw("prefill failed: a bounded device wait gave up (error flags 0x%x)", err);
  }
  len_ = pos0 + n;
  logits_valid_ = true;
}

void Session::ReduceIntoResidual(float* x, float* y, int64_t n, cudaStream_t s) {
  const int64_t count = n * m_->meta().hidden;
  m_->tp()->AllReduceSum(y, static_cast<size_t>(count), s);
  LaunchAddInPlace(x, y, count, s);
}

void Session::GatherLogits(cudaStream_t s) {
  m_->tp()->AllGatherInPlace(logits_, static_cast<size_t>(m_->shard().vocab_rows), s);
}

void Session::EnqueueSample(const SampleOpts& opt, uint64_t seed, int pos_bump, bool pdl, int32_t trace_id) {
  const ModelMeta& c = m_->meta();
  SampleParams sp;
  sp.logits = logits_;
  sp.n = c.vocab;
  sp.temperature = opt.temperature;
  sp.top_k = opt.top_k;
  sp.top_p = opt.top_p;
  sp.seed = seed;
  sp.pos = pos_;
  sp.pos_bump = pos_bump;
  sp.probs = probs_;
  sp.tok_out = tok_;
  sp.cand_val = cand_val_;
  sp.cand_idx = cand_idx_;
  sp.cand_cnt = cand_cnt_;
  sp.flag = flag_;
  if (trace_id >= 0) sp.trace = NextTrace(&trace_id);
  LaunchSample(sp, false, stream_, pdl);
}

void Session::EnqueueStep(const SampleOpts& opt, uint64_t seed) {
  const ModelMeta& c = m_->meta();
  const cudaStream_t s = stream_;
  const int H = c.hidden, qd = c.q_dim(), kvd = c.kv_dim();
  const int sms = m_->num_sms();
  const bool tp = m_->tp() != nullptr;
  int launches = 0;
  int32_t tid = 0;  // trace id of the next launch
  LaunchEmbed(m_->embd(), tok_, 1, x_, pos_, out_ids_, s, false, NextTrace(&tid));
  ++launches;
  for (int l = 0; l < c.n_layers; ++l) {
    const DevLayer& L = m_->layers()[static_cast<size_t>(l)];
    MvParams q;
    q.seg[0].w = L.q;
    q.seg[0].out_off = 0;
    q.seg[1].w = L.k;
    q.seg[1].out_off = qd;
    q.seg[2].w = L.v;
    q.seg[2].out_off = qd + kvd;
    q.n_seg = 3;
    q.total_rows = qd + 2 * kvd;
    q.x = x_;
    q.norm_w = L.attn_norm;
    q.eps = c.rms_eps;
    q.out = qkv_;
    q.err = err_;
    q.trace = NextTrace(&tid);
    LaunchMatvec(q, Epi::kStore, 2, sms, s, true);

    AttnParams a;
    a.q = qkv_;
    a.q_stride = 0;
    a.k_raw = qkv_ + qd;
    a.v_raw = qkv_ + qd + kvd;
    a.q_norm = L.q_norm;
    a.k_norm = L.k_norm;
    a.rope = m_->rope();
    a.eps = c.rms_eps;
    a.kc = kc_ + layer_elems_ * l;
    a.vc = vc_ + layer_elems_ * l;
    a.max_seq = static_cast<int32_t>(max_seq_);
    a.pos = pos_;
    a.n_heads = c.n_heads;
    a.n_kv = c.n_kv_heads;
    a.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
    a.out = attn_;
    a.part = attn_part_;
    a.ticket = tickets_;
    a.n_splits = n_splits_;
    a.fused = 1;
    a.err = err_;
    a.trace = NextTrace(&tid);
    LaunchAttention(a, 1, s, true);

    MvParams o;
    o.seg[0].w = L.o;
    o.total_rows = H;
    o.x = attn_;
    o.err = err_;
    o.trace = NextTrace(&tid);
    if (tp) {
      o.out = y_;
      LaunchMatvec(o, Epi::kStore, 1, sms, s, true);
      ReduceIntoResidual(x_, y_, 1, s);
      ++launches;
    } else {
      o.out = x_;
      o.resid = x_;
      LaunchMatvec(o, Epi::kResid, 1, sms, s, true);
    }

    MvParams gu;
    gu.seg[0].w = L.gateup;
    gu.total_rows = 2 * c.ffn;
    gu.x = x_;
    gu.norm_w = L.ffn_norm;
    gu.eps = c.rms_eps;
    gu.out = h_;
    gu.err = err_;
    gu.trace = NextTrace(&tid);
    LaunchMatvec(gu, Epi::kSilu, 2, sms, s, true);

    MvParams dn;
    dn.seg[0].w = L.down;
    dn.total_rows = H;
    dn.x = h_;
    dn.err = err_;
    dn.trace = NextTrace(&tid);
    if (tp) {
      dn.out = y_;
      LaunchMatvec(dn, Epi::kStore, 1, sms, s, true);
      ReduceIntoResidual(x_, y_, 1, s);
      ++launches;
    } else {
      dn.out = x_;
      dn.resid = x_;
      LaunchMatvec(dn, Epi::kResid, 1, sms, s, true);
    }
    launches += 5;
  }
  MvParams lm;
  lm.seg[0].w = m_->lm_head();
  lm.total_rows = m_->lm_head().rows;
  lm.x = x_;
  lm.norm_w = m_->out_norm();
  lm.eps = c.rms_eps;
  lm.out = logits_ + m_->shard().vocab0;
  lm.err = err_;
  lm.trace = NextTrace(&tid);
  if (tp) {
    // every rank samples the same gathered logits and so draws the same token
    LaunchMatvec(lm, Epi::kStore, 4, sms, s, true);
    GatherLogits(s);
    EnqueueSample(opt, seed, 1, false, trace_rec_ != nullptr ? tid : -1);
    const bool fast = opt.temperature > 0.0f && opt.top_k > 1 && opt.top_k <= kFastTopK && opt.top_k < c.vocab;
    launches += fast ? 4 : 2;
  } else if (!(opt.temperature > 0.0f)) {
    lm.part_val = am_val_;
    lm.part_idx = am_idx_;
    lm.ticket = tickets_ + c.n_kv_heads;
    lm.tok_out = tok_;
    lm.pos = pos_;
    lm.pos_bump = 1;
    LaunchMatvec(lm, Epi::kArgmax, 4, sms, s, true);
    launches += 1;
  } else {
    LaunchMatvec(lm, Epi::kStore, 4, sms, s, true);
    EnqueueSample(opt, seed, 1, true, trace_rec_ != nullptr ? tid : -1);
    const bool fast = opt.top_k > 1 && opt.top_k <= kFastTopK && opt.top_k < c.vocab;
    launches += fast ? 4 : 2;
  }
  kernels_per_step_ = launches;
}

int Session::Generate(const SampleOpts& opt, uint64_t seed, int32_t max_tokens, const int32_t* stop, int32_t n_stop,
                      int32_t* out, float* step_logits) {
  const ModelMeta& c = m_->meta();
  RPGB_CHECK(max_tokens > 0, "max_tokens must be positive, got %d", max_tokens);
  RPGB_CHECK(logits_valid_, "no logits for the next position: run a prefill first");
  RPGB_CHECK(len_ + max_tokens <= max_seq_,
             "context is full: %lld positions + %d tokens exceed max_seq %lld (use a larger max_seq or reset)",
             static_cast<long long>(len_), max_tokens, static_cast<long long>(max_seq_));
  RPGB_CUDA(cudaSetDevice(m_->device()));
  const cudaStream_t s = stream_;
  const int64_t start = len_;

  // first token: sampled from the current logits with counter = len
  RPGB_CUDA(cudaMemcpyAsync(pos_, &start, sizeof(int64_t), cudaMemcpyHostToDevice, s));
  if (step_logits != nullptr) {
    RPGB_CUDA(cudaMemcpyAsync(step_logits, logits_, sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s));
  }
  EnqueueSample(opt, seed, 0);

  // Tensor parallel decode runs in the loop kernel with the ranks' partials
  // and sampler candidates exchanged over NVLink (after TpAttach; greedy or
  // the fast sampler); otherwise a tensor-parallel step runs as the step
  // graph with NCCL between launches.
  const bool loop_tp = m_->tp() == nullptr || (tp_attached_ && LoopMode(opt) != 2 && step_logits == nullptr);
  if (LoopSupportsGroup(c.group()) && loop_tp && std::getenv("RPGB_DECODE_GRAPH") == nullptr) {
    return GenerateLoop(opt, seed, max_tokens, stop, n_stop, out, step_logits, start);
  }

  // (re)record the step graph when the sampling parameters change
  if (graph_ == nullptr || !SameOpts(opt, graph_opt_) || seed != graph_seed_) {
    DropGraph();
    cudaGraph_t g = nullptr;
    RPGB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    const int64_t before = LaunchCount();
    try {
      EnqueueStep(opt, seed);
      CountLaunches(before - LaunchCount());  // recorded, not launched
    } catch (...) {
      cudaStreamEndCapture(s, &g);
      if (g != nullptr) cudaGraphDestroy(g);
      throw;
    }
    RPGB_CUDA(cudaStreamEndCapture(s, &g));
    const cudaError_t ie = cudaGraphInstantiateWithFlags(&graph_, g, 0);
    cudaGraphDestroy(g);
    RPGB_CUDA(ie);
    graph_opt_ = opt;
    graph_seed_ = seed;
  }

  if (host_ids_cap_ < max_tokens) {
    if (host_ids_ != nullptr) cudaFreeHost(host_ids_);
    host_ids_ = nullptr;
    RPGB_CUDA(cudaMallocHost(&host_ids_, sizeof(int32_t) * max_tokens));
    host_ids_cap_ = max_tokens;
  }

  // Steps are launched in chunks without a host round trip; with stop ids the
  // chunk is small so little work runs past a stop token.
  const int chunk = step_logits != nullptr ? 1 : (n_stop > 0 ? 8 : max_tokens);
  int produced = 0, launched = 0;
  bool stopped = false;
  while (produced < max_tokens && !stopped) {
    const int todo = std::min(chunk, max_tokens - produced);
    launched += todo;
    for (int i = 0; i < todo; ++i) {
      RPGB_CUDA(cudaGraphLaunch(graph_, s));
      ++graph_launches_;
      CountLaunches(kernels_per_step_);
      if (step_logits != nullptr && produced + i + 1 < max_tokens) {
        RPGB_CUDA(cudaMemcpyAsync(step_logits + static_cast<int64_t>(produced + i + 1) * c.vocab, logits_,
                                  sizeof(float) * c.vocab, cudaMemcpyDeviceToHost, s));
      }
    }
    RPGB_CUDA(cudaMemcpyAsync(host_ids_ + produced, out_ids_ + start + produced, sizeof(int32_t) * todo,
                              cudaMemcpyDeviceToHost, s));
    RPGB_CUDA(cudaStreamSynchronize(s));
    for (int i = 0; i < todo; ++i) {
      const int32_t id = host_ids_[produced + i];
      bool is_stop = false;
      for (int j = 0; j < n_stop; ++j) is_stop = is_stop || stop[j] == id;
      if (is_stop) {
        produced += i + 1;
        stopped = true;
        break;
      }
    }
    if (!stopped) produced += todo;
  }
  unsigned err = 0;
  RPGB_CUDA(cudaMemcpy(&err, err_, sizeof(unsigned), cudaMemcpyDeviceToHost));
  if (err != 0) {
    RPGB_CUDA(cudaMemset(err_, 0, sizeof(unsigned)));
    Throw("a device-side wait for streamed weights timed out during decode (results discarded)");
  }
  std::memcpy(out, host_ids_, sizeof(int32_t) * produced);
  // Every returned token (stop included) was forwarded: len = prompt + generated.
  const bool ran_past = launched > produced;
  len_ = start + produced;
  // after a stop inside a chunk the device logits belong to a later step
  logits_valid_ = !ran_past;
  if (ran_past) {
    RPGB_CUDA(cudaMemcpyAsync(pos_, &len_, sizeof(int64_t), cudaMemcpyHostToDevice, s));
    RPGB_CUDA(cudaStreamSynchronize(s));
  }
  return produced;
}

// The decode loop's sampler: 0 greedy, 1 the fast candidate path (1 <
// top_k <= kFastTopK, each block's lm_head rows one candidate slice), 2 the
// general one-block sampler.
int Session::LoopMode(const SampleOpts& opt) const {
  const int sms = m_->num_sms();
  const int rows = m_->lm_head().rows;  // this GPU's rows of the vocabulary
  const int lm_rows_per_block = (rows / 16 + sms - 1) / sms * 16;
  if (!(opt.temperature > 0.0f)) return 0;
  if (opt.top_k > 1 && opt.top_k <= kFastTopK && opt.top_k < rows && sms <= kCandBlocks && lm_rows_per_block <= 2048) {
    return 1;
  }
  return 2;
}

LoopParams Session::MakeLoopParams(const SampleOpts& opt, uint64_t seed) const {
  const ModelMeta& c = m_->meta();
  LoopParams lp;
  if (const char* e = std::getenv("RPGB_TEST_WAIT_LIMIT")) lp.ll_limit = static_cast<uint32_t>(std::strtoul(e, nullptr, 10));
  if (const char* e = std::getenv("RPGB_TEST_DROP_WORD")) lp.test_drop_word = std::atoi(e);
  lp.layers = m_->layers_dev();
  lp.n_layers = c.n_layers;
  lp.slot = std::max(2048, GroupBytes(m_->lm_head().type));  // 2048: a K + V attention chunk
  for (const DevLayer& L : m_->layers()) {
    for (const DevMat* w : {&L.q, &L.k, &L.v, &L.o, &L.gateup, &L.down}) lp.slot = std::max(lp.slot, GroupBytes(w->type));
  }
  lp.embd = m_->embd();
  lp.lm_head = m_->lm_head();
  lp.out_norm = m_->out_norm();
  lp.rope = m_->rope();
  lp.hidden = c.hidden;
  lp.n_heads = c.n_heads;
  lp.n_kv = c.n_kv_heads;
  lp.ffn = c.ffn;
  lp.vocab = c.vocab;
  lp.max_seq = static_cast<int32_t>(max_seq_);
  lp.eps = c.rms_eps;
  lp.scale = 1.0f / sqrtf(static_cast<float>(c.head_dim));
  lp.kc = kc_;
  lp.vc = vc_;
  lp.layer_elems = static_cast<int64_t>(layer_elems_);
  lp.v_minus_k = reinterpret_cast<const char*>(vc_) - reinterpret_cast<const char*>(kc_);
  lp.llx = ll_;
  lp.llqkv = lp.llx + c.hidden;
  lp.llh = lp.llqkv + (c.q_dim() + 2 * c.kv_dim());
  lp.llrec = lp.llh + c.ffn;
  lp.llattn = lp.llrec + LoopPartialWords(c.n_kv_heads, c.group(), loop_splits_);
  lp.tickets = tickets_loop_;
  lp.logits = logits_;
  lp.probs = probs_;
  lp.pos = pos_;
  lp.tok = tok_;
  lp.out_ids = out_ids_;
  lp.temperature = opt.temperature;
  lp.top_k = opt.top_k;
  lp.top_p = opt.top_p;
  lp.seed = seed;
  lp.mode = LoopMode(opt);
  lp.cand_val = cand_val_;
  lp.cand_idx = cand_idx_;
  lp.cand_cnt = cand_cnt_;
  lp.am_val = am_val_;
  lp.am_idx = am_idx_;
  lp.steps_done = steps_done_;
  lp.stop = stop_dev_;
  lp.bar = bar_;
  lp.err = err_;
  lp.splits = loop_splits_;
  lp.vocab0 = m_->shard().vocab0;
  if (m_->tp() != nullptr && tp_attached_) {
    lp.tp = m_->tp()->size();
    lp.tp_rank = m_->tp()->rank();
    for (int k = 0; k < lp.tp; ++k) lp.xpeer[k] = xpeer_[k];
  }
  if (trace_rec_ != nullptr) {
    int khz = 0;
    RPGB_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, m_->device()));
    lp.ns_per_cycle = 1.0e6 / static_cast<double>(std::max(khz, 1));
    lp.trace.rec = trace_rec_;
    lp.trace.count = trace_count_;
    lp.trace.cap = trace_cap_;
    lp.trace.id = 0;
  }
  return lp;
}

// The decode loop in one cooperative kernel per chunk of steps (k_step.cu).
// The first token is sampled from the current logits by the standalone
// sampler (counter = len); the kernel then forwards it and every following
// token, stopping on a stop id by itself when the list fits on the device.
int Session::GenerateLoop(const SampleOpts& opt, uint64_t seed, int32_t max_tokens, const int32_t* stop,
                          int32_t n_stop, int32_t* out, float* step_logits, int64_t start) {
  const ModelMeta& c = m_->meta();
  const cudaStream_t s = stream_;
  if (host_ids_cap_ < max_tokens) {
    if (host_ids_ != nullptr) cudaFreeHost(host_ids_);
    host_ids_ = nullptr;
    RPGB_CUDA(cudaMallocHost(&host_ids_, sizeof(int32_t) * max_tokens));
    host_ids_cap_ = max_tokens;
  }
  LoopParams lp = MakeLoopParams(opt, seed);
  const bool dev_stop = n_stop <= kLoopMaxStop;
  if (dev_stop && n_stop > 0) {
    RPGB_CUDA(cudaMemcpyAsync(stop_dev_, stop, sizeof(int32_t) * n_stop, cudaMemcpyHostToDevice, s));
  }
  lp.n_stop = dev_stop ? n_stop : 0;
  RPGB_CUDA(cudaMemsetAsync(steps_done_ + 1, 0, sizeof(int32_t), s));
  // With stop ids the device cannot see, chunks stay short so little work runs past a stop.
  const int chunk = dev_stop ? max_tokens : 8;
  if (step_logits != nullptr) {
    // every step's logits row is kept on the device and copied after the
    // launch, so the launch runs the same steps as without them
    if (step_logits_cap_ < chunk) {
      cudaFree(step_logits_dev_);
      step_logits_dev_ = nullptr;
      step_logits_cap_ = 0;
      RPGB_CUDA(cudaMalloc(&step_logits_dev_, sizeof(float) * static_cast<size_t>(chunk) * c.vocab));
      step_logits_cap_ = chunk;
    }
    lp.step_logits = step_logits_dev_;
  }
  int produced = 0, launched = 0;
  bool stopped = false;
  while (produced < max_tokens && !stopped) {
    const int todo = std::min(chunk, max_tokens - produced);
    lp.n_steps = todo;
    const uint32_t need = LoopTagsPerLaunch(c.n_layers, todo);
    if (epoch_ > 0xFFFFFFFFu - need) {  // tags would wrap: clear every tag and start over
      RPGB_CUDA(cudaMemsetAsync(ll_, 0, sizeof(uint64_t) * ll_words_, s));
      if (lp.tp > 0) {
        // every rank wraps at the same launch; no rank may store into a peer's
        // buffer before that peer cleared it, so the group meets after the clear
        RPGB_CUDA(cudaMemsetAsync(xbuf_, 0, sizeof(uint64_t) * xbuf_words_, s));
        m_->tp()->AllReduceSum(y_, 1, s);
      }
      epoch_ = 1;
    }
    lp.epoch0 = epoch_;
    epoch_ += need;
    LaunchDecodeLoop(lp, c.group(), m_->num_sms(), s);
    if (lp.tp > 0) GatherLogits(s);  // the next call samples its first token from the whole row
    loop_ready_ = true;
    RPGB_CUDA(cudaMemcpyAsync(loop_host_, steps_done_, sizeof(int32_t) * 2, cudaMemcpyDeviceToHost, s));
    RPGB_CUDA(cudaMemcpyAsync(host_ids_ + produced, out_ids_ + start + produced, sizeof(int32_t) * todo,
                              cudaMemcpyDeviceToHost, s));
    RPGB_CUDA(cudaStreamSynchronize(s));
    const int done = loop_host_[0];
    const bool host_sample = loop_host_[1] != 0;
    unsigned err = 0;
    RPGB_CUDA(cudaMemcpy(&err, err_, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (err != 0 || done < 1 || done > todo) {
      RPGB_CUDA(cudaMemset(err_, 0, sizeof(unsigned)));
      len_ = start + produced;
      logits_valid_ = false;
      Throw("decode loop failed (device error flags 0x%x, %d of %d steps): a bounded device wait gave up", err,
            done, todo);
    }
    graph_launches_ += done;
    launched += done;
    int take = done;
    for (int i = 0; i < done; ++i) {
      const int32_t id = host_ids_[produced + i];
      bool is_stop = false;
      for (int j = 0; j < n_stop; ++j) is_stop = is_stop || stop[j] == id;
      if (is_stop) {
        take = i + 1;
        stopped = true;
        break;
      }
    }
    if (step_logits != nullptr) {
      // launch step i forwarded token produced + i; its logits choose token produced + i + 1
      const int rows = std::min(take, max_tokens - produced - 1);
      if (rows > 0) {
        RPGB_CUDA(cudaMemcpy(step_logits + static_cast<int64_t>(produced + 1) * c.vocab, step_logits_dev_,
                             sizeof(float) * static_cast<size_t>(rows) * c.vocab, cudaMemcpyDeviceToHost));
      }
    }
    produced += take;
    if (host_sample) {
      // the tensor-parallel sampler's candidates overflowed at the last step:
      // the next token comes from the gathered row (counter = the new len)
      RPGB_CUDA(cudaMemsetAsync(steps_done_ + 1, 0, sizeof(int32_t), s));
      if (!stopped && produced < max_tokens) EnqueueSample(opt, seed, 0);
    }
  }
  kernels_per_step_ = 1;
  std::memcpy(out, host_ids_, sizeof(int32_t) * produced);
  const bool ran_past = launched > produced;
  len_ = start + produced;
  logits_valid_ = !ran_past;
  if (ran_past) {
    RPGB_CUDA(cudaMemcpyAsync(pos_, &len_, sizeof(int64_t), cudaMemcpyHostToDevice, s));
    RPGB_CUDA(cudaStreamSynchronize(s));
  }
  return produced;
}

}  // namespace rpgb
