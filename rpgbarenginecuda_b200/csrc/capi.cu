// capi.cc -- extern "C" entry points of include/rpg_b200.h.
//
// Registries follow the reference ABI's rules (src/engine.cc:136-163): handles
// are increasing integers never reused, lookups under one mutex, and every
// entry catches exceptions into the thread-local last error.
#include "../../include/rpg_b200.h"

#include <cuda_runtime.h>

#include <cstring>
#include <map>
#include <vector>
#include <memory>
#include <mutex>

#include "common.h"
#include "engine.h"
#include "kernels.cuh"
#include "kernels.h"
#include "gguf.h"
#include "model.h"
#include "tp.h"

namespace rpgb {
namespace {

struct MatrixEntry {
  int device = 0;
  int num_sms = 0;
  int64_t rows = 0;  // logical rows (storage is padded to whole 32-row groups)
  DevMat m;
  void* mem = nullptr;
  // tensor-core GEMM scratch (grown on demand), its error word and the
  // pinned host copy of that word the next call reads
  std::mutex tc_mu;
  __half* tc = nullptr;
  size_t tc_halves = 0;
  // the matrix dequantised once into fp16 hi/lo terms for the tensor-core
  // GEMM (made by the first call that runs it; lo follows hi)
  __half* wh = nullptr;
  // split-K partial tiles (grown on demand)
  float* part = nullptr;
  size_t part_floats = 0;
  unsigned* err = nullptr;
  unsigned* err_host = nullptr;
};

std::mutex g_mu;
std::map<int32_t, std::shared_ptr<Model>> g_models;
std::map<int32_t, std::shared_ptr<Session>> g_sessions;
std::map<int32_t, std::shared_ptr<MatrixEntry>> g_mats;
std::map<int32_t, std::shared_ptr<TpGroup>> g_groups;
std::map<int32_t, int32_t> g_session_model;
int32_t g_next = 1;

// Per-device scratch for the operator-level sampler entry.
struct SampleScratch {
  float* cand_val = nullptr;
  int32_t* cand_idx = nullptr;
  int32_t* cand_cnt = nullptr;
  int32_t* flag = nullptr;
  int64_t* counter = nullptr;
  float* probs = nullptr;
  int32_t probs_n = 0;
};
std::map<int, SampleScratch> g_sample_scratch;

std::shared_ptr<Model> GetModel(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_models.find(h);
  RPGB_CHECK(it != g_models.end(), "invalid model handle %d", h);
  return it->second;
}
std::shared_ptr<Session> GetSession(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sessions.find(h);
  RPGB_CHECK(it != g_sessions.end(), "invalid session handle %d", h);
  return it->second;
}
std::shared_ptr<MatrixEntry> GetMatrix(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_mats.find(h);
  RPGB_CHECK(it != g_mats.end(), "invalid matrix handle %d", h);
  return it->second;
}

}  // namespace
}  // namespace rpgb

using namespace rpgb;

#define RPGB_CATCH(ret)                                  \
  catch (const std::exception& e) {                      \
    SetLastError(e.what());                              \
    return ret;                                          \
  }                                                      \
  catch (...) {                                          \
    SetLastError("unknown exception (not std::exception)"); \
    return ret;                                          \
  }

extern "C" {

const char* rpgb_version(void) { return "0.1.0-b200"; }
const char* rpgb_last_error(void) { return LastError(); }

int32_t rpgb_model_load(const char* path, int32_t device, int32_t max_pos) {
  try {
    SetLastError("");
    RPGB_CHECK(path != nullptr && *path != '\0', "model path is empty");
    std::shared_ptr<Model> m(Model::Load(path, device, max_pos > 0 ? max_pos : 4096).release());
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next++;
    g_models[h] = m;
    return h;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_tp_shard_plan(const int32_t* shape, int32_t rank, int32_t size, int32_t* out) {
  try {
    SetLastError("");
    RPGB_CHECK(shape != nullptr && out != nullptr, "tp_shard_plan: null argument");
    const ShardPlan p = MakeShardPlan(shape[0], shape[1], shape[2], shape[3], shape[4], rank, size);
    out[0] = p.heads;
    out[1] = p.kv_heads;
    out[2] = p.ffn;
    out[3] = p.vocab0;
    out[4] = p.vocab_rows;
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_tp_unique_id(uint8_t* id_out) {
  try {
    SetLastError("");
    RPGB_CHECK(id_out != nullptr, "tp_unique_id: null buffer");
    TpUniqueId(id_out);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_tp_group_create(const uint8_t* id, int32_t rank, int32_t size, int32_t device) {
  try {
    SetLastError("");
    std::shared_ptr<TpGroup> grp = TpGroup::Create(id, rank, size, device);
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next++;
    g_groups[h] = grp;
    return h;
  }
  RPGB_CATCH(-1)
}

void rpgb_tp_group_free(int32_t group) {
  try {
    std::shared_ptr<TpGroup> grp;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_groups.find(group);
      if (it == g_groups.end()) return;
      grp = it->second;
      g_groups.erase(it);
    }
    // models on the group hold it until they are freed
  } catch (...) {
  }
}

int32_t rpgb_model_load_tp(const char* path, int32_t device, int32_t max_pos, int32_t group) {
  try {
    SetLastError("");
    RPGB_CHECK(path != nullptr && *path != '\0', "model path is empty");
    std::shared_ptr<TpGroup> grp;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_groups.find(group);
      RPGB_CHECK(it != g_groups.end(), "invalid tensor-parallel group handle %d", group);
      grp = it->second;
    }
    std::shared_ptr<Model> m(Model::Load(path, device, max_pos > 0 ? max_pos : 4096, grp).release());
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next++;
    g_models[h] = m;
    return h;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_tp_handle(int32_t session, uint8_t* handle_out) {
  try {
    SetLastError("");
    RPGB_CHECK(handle_out != nullptr, "session_tp_handle: null buffer");
    GetSession(session)->TpHandle(handle_out);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_tp_attach(int32_t session, const uint8_t* handles) {
  try {
    SetLastError("");
    RPGB_CHECK(handles != nullptr, "session_tp_attach: null handles");
    GetSession(session)->TpAttach(handles);
    return 0;
  }
  RPGB_CATCH(-1)
}

void rpgb_model_free(int32_t model) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    for (auto it = g_session_model.begin(); it != g_session_model.end();) {
      if (it->second == model) {
        g_sessions.erase(it->first);
        it = g_session_model.erase(it);
      } else {
        ++it;
      }
    }
    g_models.erase(model);
  } catch (...) {
  }
}

int32_t rpgb_model_shape(int32_t model, int32_t* out, int32_t n_out) {
  try {
    SetLastError("");
    auto m = GetModel(model);
    const ModelMeta& c = m->global_meta();
    const int32_t v[12] = {c.n_layers, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn,
                           c.vocab, c.context_length, m->rope_positions(), c.eos_id, m->device(), m->num_sms()};
    for (int i = 0; i < n_out && i < 12; ++i) out[i] = v[i];
    return 0;
  }
  RPGB_CATCH(-1)
}

int64_t rpgb_model_device_bytes(int32_t model) {
  try {
    return GetModel(model)->device_bytes();
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_create(int32_t model, int64_t max_seq) {
  try {
    SetLastError("");
    auto m = GetModel(model);
    auto s = std::make_shared<Session>(m.get(), max_seq);
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next++;
    g_sessions[h] = s;
    g_session_model[h] = model;
    return h;
  }
  RPGB_CATCH(-1)
}

void rpgb_session_free(int32_t session) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    g_sessions.erase(session);
    g_session_model.erase(session);
  } catch (...) {
  }
}

int64_t rpgb_session_len(int32_t session) {
  try {
    return GetSession(session)->len();
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_set_len(int32_t session, int64_t len) {
  try {
    SetLastError("");
    GetSession(session)->SetLen(len);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_prefill(int32_t session, const int32_t* tokens, int64_t n, float* last_logits) {
  try {
    SetLastError("");
    RPGB_CHECK(tokens != nullptr, "tokens is NULL");
    GetSession(session)->Prefill(tokens, n, last_logits);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_generate(int32_t session, const rpgb_sample_options* opt, uint64_t seed, int32_t max_tokens,
                      const int32_t* stop_ids, int32_t n_stop, int32_t* out_ids, int32_t* n_out,
                      float* step_logits) {
  try {
    SetLastError("");
    RPGB_CHECK(out_ids != nullptr && n_out != nullptr, "out_ids / n_out is NULL");
    RPGB_CHECK(n_stop == 0 || stop_ids != nullptr, "stop_ids is NULL");
    SampleOpts o;
    if (opt != nullptr) {
      o.temperature = opt->temperature;
      o.top_k = opt->top_k;
      o.top_p = opt->top_p;
    }
    *n_out = GetSession(session)->Generate(o, seed, max_tokens, stop_ids, n_stop, out_ids, step_logits);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_stats(int32_t session, int32_t* kernels_per_step, int32_t* graph_ready,
                           int64_t* graph_launches) {
  try {
    auto s = GetSession(session);
    if (kernels_per_step) *kernels_per_step = s->kernels_per_step();
    if (graph_ready) *graph_ready = s->graph_ready() ? 1 : 0;
    if (graph_launches) *graph_launches = s->graph_launches();
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_trace_enable(int32_t session, int32_t cap) {
  try {
    SetLastError("");
    GetSession(session)->EnableTrace(cap);
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_session_trace_take(int32_t session, rpgb_trace_rec* out, int32_t cap) {
  try {
    SetLastError("");
    static_assert(sizeof(rpgb_trace_rec) == sizeof(TraceRec), "trace record layout");
    RPGB_CHECK(out != nullptr || cap == 0, "null trace buffer");
    return GetSession(session)->TakeTrace(reinterpret_cast<TraceRec*>(out), cap);
  }
  RPGB_CATCH(-1)
}

void* rpgb_session_stream(int32_t session) {
  try {
    return GetSession(session)->stream();
  }
  RPGB_CATCH(nullptr)
}

int64_t rpgb_launch_count(void) { return LaunchCount(); }

int32_t rpgb_matrix_upload(int32_t device, uint32_t type, int64_t rows, int64_t cols, const void* bytes) {
  try {
    SetLastError("");
    RPGB_CHECK(bytes != nullptr, "matrix bytes are NULL");
    RPGB_CHECK(rows > 0 && cols > 0 && cols % 256 == 0 && rows < (1 << 30), "bad matrix shape %lld x %lld",
               static_cast<long long>(rows), static_cast<long long>(cols));
    // storage holds whole 16-row tiles; padding rows are zero blocks
    const int64_t prow = (rows + kTileRows - 1) / kTileRows * kTileRows;
    const size_t bytes_dev = DevMatBytes(type, prow, cols);
    auto e = std::make_shared<MatrixEntry>();
    e->rows = rows;
    e->device = device;
    RPGB_CUDA(cudaSetDevice(device));
    RPGB_CUDA(cudaDeviceGetAttribute(&e->num_sms, cudaDevAttrMultiProcessorCount, device));
    PrepareMatvecKernels();
    PrepareMatvecTokensKernels();
    PrepareSampleKernels();
    PrepareTcGemmKernels();
    const int64_t rb = GgmlRowBytes(type, cols);
    std::vector<uint8_t> src(static_cast<size_t>(prow * rb), 0);
    std::memcpy(src.data(), bytes, static_cast<size_t>(rows * rb));
    std::vector<uint8_t> host(bytes_dev, 0);
    RepackRows(type, src.data(), prow, cols, host.data());
    RPGB_CUDA(cudaMalloc(&e->mem, host.size()));
    RPGB_CUDA(cudaMemcpy(e->mem, host.data(), host.size(), cudaMemcpyHostToDevice));
    e->m.type = type;
    e->m.rows = static_cast<int32_t>(prow);
    e->m.cols = static_cast<int32_t>(cols);
    e->m.nb = static_cast<int32_t>(cols / 256);
    e->m.q = static_cast<uint8_t*>(e->mem);
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next++;
    g_mats[h] = e;
    return h;
  }
  RPGB_CATCH(-1)
}

void rpgb_matrix_free(int32_t matrix) {
  try {
    std::shared_ptr<MatrixEntry> e;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      auto it = g_mats.find(matrix);
      if (it == g_mats.end()) return;
      e = it->second;
      g_mats.erase(it);
    }
    cudaSetDevice(e->device);
    cudaFree(e->mem);
    cudaFree(e->tc);
    cudaFree(e->wh);
    cudaFree(e->part);
    cudaFree(e->err);
    if (e->err_host != nullptr) cudaFreeHost(e->err_host);
  } catch (...) {
  }
}

int32_t rpgb_matrix_dequant(int32_t matrix, int64_t row0, int64_t n_rows, float* dst_dev, void* stream) {
  try {
    SetLastError("");
    auto e = GetMatrix(matrix);
    RPGB_CUDA(cudaSetDevice(e->device));
    RPGB_CHECK(row0 >= 0 && n_rows > 0 && row0 + n_rows <= e->rows, "dequant: rows [%lld, %lld) out of range",
               static_cast<long long>(row0), static_cast<long long>(row0 + n_rows));
    LaunchDequantRows(e->m, row0, n_rows, dst_dev, static_cast<cudaStream_t>(stream));
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_matrix_matvec(int32_t matrix, const float* x_dev, int64_t n_tok, float* out_dev, void* stream) {
  try {
    SetLastError("");
    auto e = GetMatrix(matrix);
    RPGB_CHECK(x_dev != nullptr && out_dev != nullptr, "null device pointer");
    RPGB_CHECK(n_tok > 0 && n_tok < (1 << 24), "bad token count");
    RPGB_CUDA(cudaSetDevice(e->device));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    RPGB_CHECK(e->rows % kTileRows == 0, "matvec: %lld rows; the kernels need a multiple of %d rows",
               static_cast<long long>(e->rows), kTileRows);
    if (n_tok == 1) {
      MvParams p;
      p.seg[0].w = e->m;
      p.n_seg = 1;
      p.total_rows = e->m.rows;
      p.x = x_dev;
      p.out = out_dev;
      const int rw = e->m.rows % 4 == 0 ? 4 : (e->m.rows % 2 == 0 ? 2 : 1);
      // programmatic launch: the weights stream in while the previous kernel
      // on the stream finishes (the kernel waits for it before reading x)
      LaunchMatvec(p, Epi::kStore, rw, e->num_sms, s, true);
    } else if (n_tok < kTcMinTokens || e->m.rows % 128 != 0) {
      MvnParams q;
      q.w = e->m;
      q.x = x_dev;
      q.out = out_dev;
      q.n_tok = static_cast<int32_t>(n_tok);
      q.ldx = e->m.cols;
      q.ldo = e->m.rows;
      LaunchMatvecTokens(q, e->num_sms, s, true);
    } else {
      GemmParams g;
      g.w = e->m;
      g.X = x_dev;
      g.n_tok = static_cast<int32_t>(n_tok);
      g.ldx = e->m.cols;
      g.out = out_dev;
      g.ldo = e->m.rows;
      if (n_tok >= kTcMinTokens && e->m.rows % 128 == 0) {
        // tensor-core path: fp16 operand scratch kept with the matrix.  The
        // call does not wait for the GEMM (launches can be captured in a
        // graph); the GEMM's error word is copied to pinned host memory
        // behind it and the next call on the matrix reports a wait that gave up
        std::lock_guard<std::mutex> lk(e->tc_mu);
        if (e->err == nullptr) {
          RPGB_CUDA(cudaMalloc(&e->err, sizeof(unsigned)));
          RPGB_CUDA(cudaMemset(e->err, 0, sizeof(unsigned)));
          RPGB_CUDA(cudaMallocHost(&e->err_host, sizeof(unsigned)));
          *e->err_host = 0;
        }
        const unsigned prev = *reinterpret_cast<volatile unsigned*>(e->err_host);
        if (prev != 0) {
          RPGB_CUDA(cudaStreamSynchronize(s));
          RPGB_CUDA(cudaMemset(e->err, 0, sizeof(unsigned)));
          *e->err_host = 0;
          Throw("matvec: a bounded device wait of an earlier tensor-core GEMM on this matrix gave up (0x%x)", prev);
        }
        const size_t wn = static_cast<size_t>(e->m.rows) * e->m.cols;
        if (e->wh == nullptr) {
          RPGB_CUDA(cudaMalloc(&e->wh, 2 * wn * sizeof(__half)));
          LaunchDequantSplit(e->m, e->wh, e->wh + wn, s);
        }
        g.w.wh = e->wh;
        g.w.wl = e->wh + wn;
        const size_t need = TcGemmScratchHalves(e->m.rows, n_tok, e->m.cols, true);
        if (e->tc_halves < need) {
          RPGB_CUDA(cudaStreamSynchronize(s));
          cudaFree(e->tc);
          e->tc = nullptr;
          e->tc_halves = 0;
          RPGB_CUDA(cudaMalloc(&e->tc, need * sizeof(__half)));
          e->tc_halves = need;
        }
        g.tc_scratch = e->tc;
        g.tc_scratch_halves = e->tc_halves;
        // split-K partials: exactly what this shape's split needs
        const int sp = TcGemmSplits(e->m.rows, n_tok, e->m.cols, e->num_sms, TcGemmPartFloats(e->num_sms));
        const size_t pneed = sp > 1 ? static_cast<size_t>(sp) * n_tok * e->m.rows : 0;
        if (e->part_floats < pneed) {
          RPGB_CUDA(cudaStreamSynchronize(s));
          cudaFree(e->part);
          e->part = nullptr;
          e->part_floats = 0;
          RPGB_CUDA(cudaMalloc(&e->part, pneed * sizeof(float)));
          e->part_floats = pneed;
        }
        g.part = e->part;
        g.part_floats = e->part_floats;
        g.num_sms = e->num_sms;
        g.err = e->err;
        LaunchGemm(g, Epi::kStore, s);
        RPGB_CUDA(cudaMemcpyAsync(e->err_host, e->err, sizeof(unsigned), cudaMemcpyDeviceToHost, s));
      } else {
        LaunchGemm(g, Epi::kStore, s);
      }
    }
    return 0;
  }
  RPGB_CATCH(-1)
}

int32_t rpgb_sample(const float* logits_dev, int32_t n, const rpgb_sample_options* opt, uint64_t seed,
                    uint64_t counter, float* probs_dev, int32_t* out_tok_dev, void* stream) {
  try {
    SetLastError("");
    RPGB_CHECK(logits_dev != nullptr && out_tok_dev != nullptr && opt != nullptr, "null argument");
    RPGB_CHECK(n > 0, "vocabulary size must be positive");
    int dev = 0;
    RPGB_CUDA(cudaGetDevice(&dev));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    SampleScratch* sc;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      sc = &g_sample_scratch[dev];
      if (sc->flag == nullptr) {
        PrepareSampleKernels();
        RPGB_CUDA(cudaMalloc(&sc->cand_val, sizeof(float) * kCandBlocks * kFastTopK));
        RPGB_CUDA(cudaMalloc(&sc->cand_idx, sizeof(int32_t) * kCandBlocks * kFastTopK));
        RPGB_CUDA(cudaMalloc(&sc->cand_cnt, sizeof(int32_t) * kCandBlocks));
        RPGB_CUDA(cudaMalloc(&sc->flag, sizeof(int32_t)));
        RPGB_CUDA(cudaMalloc(&sc->counter, sizeof(int64_t)));
      }
      if (probs_dev == nullptr && sc->probs_n < n) {
        cudaFree(sc->probs);
        RPGB_CUDA(cudaMalloc(&sc->probs, sizeof(float) * n));
        sc->probs_n = n;
      }
    }
    const int64_t ctr = static_cast<int64_t>(counter);
    RPGB_CUDA(cudaMemcpyAsync(sc->counter, &ctr, sizeof(int64_t), cudaMemcpyHostToDevice, s));
    SampleParams p;
    p.logits = logits_dev;
    p.n = n;
    p.temperature = opt->temperature;
    p.top_k = opt->top_k;
    p.top_p = opt->top_p;
    p.seed = seed;
    p.counter_override = sc->counter;
    p.probs = probs_dev != nullptr ? probs_dev : sc->probs;
    p.tok_out = out_tok_dev;
    p.cand_val = sc->cand_val;
    p.cand_idx = sc->cand_idx;
    p.cand_cnt = sc->cand_cnt;
    p.flag = sc->flag;
    LaunchSample(p, probs_dev != nullptr, s);
    // the counter staging is reused: finish before the host value goes out of scope
    RPGB_CUDA(cudaStreamSynchronize(s));
    return 0;
  }
  RPGB_CATCH(-1)
}

float rpgb_counter_uniform(uint64_t seed, uint64_t counter) { return dev::CounterUniform(seed, counter); }

}  // extern "C"
