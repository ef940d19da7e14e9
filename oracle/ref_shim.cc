// ref_shim.cc -- extern "C" bridge into the reference implementation, compiled
// from the reference's own sources by oracle/Makefile into oracle/_ref/.
//
// TEST INFRASTRUCTURE ONLY: loaded by tests/ and by the golden-fixture
// scripts to produce the reference's own outputs; the engine never links it.
//
// Two builds of this file:
//   libref_quant.so  host sources only (src/quant.cc): the bit-exact host
//                    dequantiser.
//   libref_emu.so    the whole reference engine -- its CUDA sources included --
//                    compiled for the host CPU against the SIMT emulation layer
//                    in oracle/emu (RPG_REF_EMU).  No GPU is touched: kernels
//                    run as fibers on the host cores.
// The entries call the same internal API the reference's own tools call:
//   DequantizeRow            src/quant.cc:416            (tools/dequant_check.cu)
//   DevCounterUniform        src/sampler_gpu.cu:364      (tools/sample_check.cu)
//   GpuFilterToProbs / GpuSampleToken  src/sampler_gpu.cu:393-440 (tools/sample_check.cu)
//   GpuMatMulQuant           src/kernels_gpu.cu:939      (tools/matmul_bench.cu)
//   GpuModel::Load / GpuForwardFull / GpuGenerate       (tools/gen_check.cu)
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "dtypes.h"
#include "quant.h"

#ifdef RPG_REF_EMU
#include "cuda_common.h"
#include "gpu_model.h"
#include "kernels_gpu.h"
#include "kv_cache_gpu.h"
#include "qwen3_gpu.h"
#include "sampler_gpu.h"
#endif

namespace {
thread_local std::string g_err;

#ifdef RPG_REF_EMU
struct RefSession {
  std::unique_ptr<rpg::GpuModel> model;
  std::unique_ptr<rpg::GpuKvCache> kv;
  rpg::GpuScratch scratch;
  const float* last = nullptr;
};
std::map<int, std::unique_ptr<RefSession>> g_sessions;
int g_next = 1;
#endif
}  // namespace

#define SHIM_TRY try {
#define SHIM_CATCH                    \
  }                                   \
  catch (const std::exception& e) {   \
    g_err = e.what();                 \
    return -1;                        \
  }

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

int ref_dequantize_row(uint32_t type, const uint8_t* src, int64_t n, float* dst) {
  SHIM_TRY
  rpg::DequantizeRow(type, src, n, dst);
  return 0;
  SHIM_CATCH
}

float ref_f16_to_f32(uint16_t h) { return rpg::F16ToF32(h); }

#ifdef RPG_REF_EMU
float ref_counter_uniform(uint64_t seed, uint64_t counter) { return rpg::DevCounterUniform(seed, counter); }

// The reference's dequant kernel (GpuDequantRow) on one row of blocks.
int ref_kernel_dequant(uint32_t type, const uint8_t* bytes, int64_t n_elems, float* out) {
  SHIM_TRY
  const int64_t nb = rpg::TypeRowBytes(type, n_elems);
  rpg::DeviceBuffer src(static_cast<size_t>(nb)), dst(static_cast<size_t>(n_elems) * 4);
  src.Upload(bytes, static_cast<size_t>(nb));
  rpg::GpuDequantRow(type, static_cast<const uint8_t*>(src.data()), n_elems, static_cast<float*>(dst.data()));
  dst.Download(out, static_cast<size_t>(n_elems) * 4);
  return 0;
  SHIM_CATCH
}

// OUT[n_tok, rows] = X[n_tok, cols] * W^T through the reference's GpuMatMulQuant.
int ref_matmul(uint32_t type, const uint8_t* bytes, int64_t rows, int64_t cols, const float* x, int64_t n_tok,
               float* out) {
  SHIM_TRY
  rpg::GpuTensor w;
  w.type = type;
  w.matrix = true;
  w.rows = rows;
  w.cols = cols;
  w.n_elements = rows * cols;
  const size_t nbytes = static_cast<size_t>(rpg::TypeRowBytes(type, cols) * rows);
  w.buf.Alloc(nbytes);
  w.buf.Upload(bytes, nbytes);
  rpg::DeviceBuffer xd(static_cast<size_t>(n_tok * cols) * 4), od(static_cast<size_t>(n_tok * rows) * 4);
  xd.Upload(x, static_cast<size_t>(n_tok * cols) * 4);
  rpg::GpuMatMulQuant(w, static_cast<const float*>(xd.data()), n_tok, static_cast<float*>(od.data()));
  od.Download(out, static_cast<size_t>(n_tok * rows) * 4);
  return 0;
  SHIM_CATCH
}

// The reference sampler on one logits row: the filtered distribution
// (GpuFilterToProbs, when probs != nullptr) and the drawn token
// (GpuSampleToken with the counter-based u of (seed, counter)).
int ref_sample(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p, uint64_t seed,
               uint64_t counter, float* probs, int32_t* tok) {
  SHIM_TRY
  rpg::SampleOptions opt;
  opt.temperature = temperature;
  opt.top_k = top_k;
  opt.top_p = top_p;
  rpg::DeviceBuffer lg(static_cast<size_t>(n) * 4), pr(static_cast<size_t>(n) * 4), idx(4);
  lg.Upload(logits, static_cast<size_t>(n) * 4);
  if (probs != nullptr) {
    rpg::GpuFilterToProbs(static_cast<const float*>(lg.data()), n, opt, static_cast<float*>(pr.data()));
    pr.Download(probs, static_cast<size_t>(n) * 4);
  }
  rpg::GpuSampleToken(static_cast<const float*>(lg.data()), n, opt, seed, counter, static_cast<float*>(pr.data()),
                      static_cast<int32_t*>(idx.data()));
  idx.Download(tok, 4);
  return 0;
  SHIM_CATCH
}

int ref_session_open(const char* gguf, int32_t max_pos, int32_t max_seq) {
  SHIM_TRY
  auto s = std::make_unique<RefSession>();
  s->model = std::make_unique<rpg::GpuModel>(rpg::GpuModel::Load(gguf, max_pos));
  s->kv = std::make_unique<rpg::GpuKvCache>(s->model->config(), max_seq);
  const int h = g_next++;
  g_sessions[h] = std::move(s);
  return h;
  SHIM_CATCH
}

void ref_session_close(int h) { g_sessions.erase(h); }

// Prefill of n tokens at the session's position; writes the last row's
// logits.  hidden (optional): the residual stream after the embedding and
// after each layer, [n_layers + 1][n][hidden], as captured by the reference's
// own GpuForwardOptions::capture_hidden (src/qwen3_gpu.cu:130-153).
int ref_session_prefill(int h, const int32_t* toks, int64_t n, float* last_logits, float* hidden) {
  SHIM_TRY
  RefSession* s = g_sessions.at(h).get();
  rpg::GpuForwardOptions fo;
  std::vector<float> hid;
  if (hidden != nullptr) fo.capture_hidden = &hid;
  rpg::GpuForwardFull(*s->model, toks, n, &s->scratch, nullptr, fo, s->kv.get());
  const int32_t V = s->model->config().vocab;
  s->last = static_cast<const float*>(s->scratch.logits.data()) + (n - 1) * V;
  if (last_logits != nullptr) {
    RPG_CUDA_CHECK(cudaMemcpy(last_logits, s->last, static_cast<size_t>(V) * 4, cudaMemcpyDeviceToHost));
  }
  if (hidden != nullptr) std::memcpy(hidden, hid.data(), hid.size() * 4);
  return 0;
  SHIM_CATCH
}

int ref_session_generate(int h, float temperature, int32_t top_k, float top_p, uint64_t seed, int32_t max_tokens,
                         const int32_t* stop, int32_t n_stop, int32_t* out, int32_t* n_out, float* step_logits) {
  SHIM_TRY
  RefSession* s = g_sessions.at(h).get();
  rpg::GpuGenerateOptions g;
  g.max_tokens = max_tokens;
  g.stop_ids.assign(stop, stop + n_stop);
  g.sample.temperature = temperature;
  g.sample.top_k = top_k;
  g.sample.top_p = top_p;
  g.seed = seed;
  std::vector<float> steps;
  if (step_logits != nullptr) g.step_logits = &steps;
  g.use_graph = false;  // the emulation has no graphs; the reference's per-step path
  std::vector<int32_t> ids;
  rpg::GpuGenerate(*s->model, s->kv.get(), &s->scratch, s->last, g, &ids);
  std::memcpy(out, ids.data(), ids.size() * 4);
  *n_out = static_cast<int32_t>(ids.size());
  if (step_logits != nullptr) std::memcpy(step_logits, steps.data(), steps.size() * 4);
  s->last = static_cast<const float*>(s->scratch.logits.data());
  return 0;
  SHIM_CATCH
}

int64_t ref_session_len(int h) { return g_sessions.at(h)->kv->len(); }
#endif

}  // extern "C"
