// model.cu -- metadata, weight repack + upload, RoPE table.
#include "model.h"

#include <cmath>
#include <cstring>
#include <functional>
#include <thread>

#include "common.h"
#include "kernels.h"

namespace rpgb {

namespace {

constexpr size_t kAlign = 256;
size_t AlignUp(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Half -> float on the host (exact; used only for F16 norm weights).
float HalfToFloat(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, out;
  if (e == 0) {
    if (m == 0) {
      out = sign;
    } else {
      int ee = 113;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        --ee;
      }
      out = sign | (static_cast<uint32_t>(ee) << 23) | ((m & 0x3FFu) << 13);
    }
  } else if (e == 31) {
    out = sign | 0x7F800000u | (m << 13);
  } else {
    out = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

// Pinned staging buffer for host -> device uploads (load time only).
class Staging {
 public:
  explicit Staging(size_t cap) : cap_(cap) {
    RPGB_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    RPGB_CUDA(cudaMallocHost(&buf_, cap_));
  }
  ~Staging() {
    cudaStreamSynchronize(stream_);
    cudaFreeHost(buf_);
    cudaStreamDestroy(stream_);
  }
  size_t cap() const { return cap_; }
  uint8_t* buf() { return buf_; }
  // Copies [buf, buf+bytes) to dst and waits, so buf can be refilled.
  void Push(void* dst, const uint8_t* from, size_t bytes) {
    RPGB_CUDA(cudaMemcpyAsync(dst, from, bytes, cudaMemcpyHostToDevice, stream_));
  }
  void Wait() { RPGB_CUDA(cudaStreamSynchronize(stream_)); }

 private:
  size_t cap_;
  cudaStream_t stream_ = nullptr;
  uint8_t* buf_ = nullptr;
};

void ParallelRows(int64_t rows, const std::function<void(int64_t, int64_t)>& fn) {
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 4;
  if (nt > 16) nt = 16;
  if (rows < 4096) nt = 1;
  std::vector<std::thread> th;
  const int64_t per = (rows + nt - 1) / nt;
  for (unsigned i = 0; i < nt; ++i) {
    const int64_t a = i * per, b = std::min<int64_t>(rows, a + per);
    if (a >= b) break;
    th.emplace_back(fn, a, b);
  }
  for (auto& t : th) t.join();
}

}  // namespace

ModelMeta ReadModelMeta(const GgufFile& g) {
  ModelMeta m;
  m.arch = g.GetStr("general.architecture");
  RPGB_CHECK(m.arch == "qwen3", "architecture is '%s'; this engine implements qwen3 only", m.arch.c_str());
  m.name = g.GetStr("general.name", g.GetStr("general.basename", "(unnamed)"));
  auto ai = [&](const char* k, int64_t def) { return g.GetInt(m.arch + "." + k, def); };
  m.n_layers = static_cast<int32_t>(ai("block_count", 0));
  m.hidden = static_cast<int32_t>(ai("embedding_length", 0));
  m.n_heads = static_cast<int32_t>(ai("attention.head_count", 0));
  m.n_kv_heads = static_cast<int32_t>(ai("attention.head_count_kv", m.n_heads));
  m.ffn = static_cast<int32_t>(ai("feed_forward_length", 0));
  m.context_length = static_cast<int32_t>(ai("context_length", 4096));
  // head_dim comes only from key_length (src/model_meta.cc:29-41 explains why
  // hidden / n_heads is not a valid fallback in general).
  const int64_t key_len = ai("attention.key_length", 0);
  if (key_len > 0) {
    m.head_dim = static_cast<int32_t>(key_len);
  } else {
    RPGB_CHECK(m.n_heads > 0 && m.hidden % m.n_heads == 0, "missing attention.key_length");
    m.head_dim = m.hidden / m.n_heads;
  }
  const int64_t value_len = ai("attention.value_length", m.head_dim);
  m.rope_theta = static_cast<float>(g.GetFloat(m.arch + ".rope.freq_base", 10000.0));
  m.rms_eps = static_cast<float>(g.GetFloat(m.arch + ".attention.layer_norm_rms_epsilon", 1e-6));
  m.bos_id = static_cast<int32_t>(g.GetInt("tokenizer.ggml.bos_token_id", -1));
  m.eos_id = static_cast<int32_t>(g.GetInt("tokenizer.ggml.eos_token_id", -1));
  m.pad_id = static_cast<int32_t>(g.GetInt("tokenizer.ggml.padding_token_id", -1));
  m.add_bos = g.GetBool("tokenizer.ggml.add_bos_token", false);
  const GgufTensor* emb = g.Find("token_embd.weight");
  RPGB_CHECK(emb != nullptr, "token_embd.weight is missing");
  m.vocab = static_cast<int32_t>(emb->rows());
  RPGB_CHECK(m.n_layers > 0 && m.hidden > 0 && m.n_heads > 0 && m.n_kv_heads > 0 && m.head_dim > 0 &&
                 m.ffn > 0 && m.vocab > 0,
             "incomplete GGUF metadata: layers=%d hidden=%d heads=%d kv=%d head_dim=%d ffn=%d vocab=%d",
             m.n_layers, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn, m.vocab);
  RPGB_CHECK(m.n_heads % m.n_kv_heads == 0, "%d query heads are not a multiple of %d KV heads", m.n_heads,
             m.n_kv_heads);
  RPGB_CHECK(value_len == m.head_dim, "value_length %lld != key_length %d", static_cast<long long>(value_len),
             m.head_dim);
  RPGB_CHECK(m.head_dim == 128, "head_dim %d: the attention kernels are specialised for 128", m.head_dim);
  RPGB_CHECK(m.group() <= 8, "GQA group %d is larger than the supported 8", m.group());
  m.tied = g.Find("output.weight") == nullptr && g.Find("lm_head.weight") == nullptr;
  for (const GgufTensor& t : g.tensors()) m.weight_bytes += t.n_bytes > 0 ? t.n_bytes : 0;
  return m;
}

void DevMatBytes(uint32_t type, int64_t rows, int64_t cols, size_t* q, size_t* s, size_t* d) {
  const size_t blocks = static_cast<size_t>(rows) * static_cast<size_t>(cols / 256);
  if (type == kGgmlQ4_K) {
    *q = blocks * 128;
    *s = blocks * 16;
    *d = 0;
  } else if (type == kGgmlQ6_K) {
    *q = blocks * 192;
    *s = blocks * 16;
    *d = blocks * 2;
  } else {
    Throw("matrix type %s is not supported (Q4_K and Q6_K are)", GgmlTypeName(type));
  }
}

void RepackGroup(uint32_t type, const uint8_t* const* src, int64_t nb, uint8_t* dq, uint8_t* ds, uint16_t* dd) {
  RPGB_CHECK(type == kGgmlQ4_K || type == kGgmlQ6_K, "matrix type %s is not supported (Q4_K and Q6_K are)",
             GgmlTypeName(type));
  const bool q4 = type == kGgmlQ4_K;
  const int nc = q4 ? 8 : 12;
  const int bb = q4 ? 144 : 210;
  for (int64_t b = 0; b < nb; ++b) {
    for (int r = 0; r < 32; ++r) {
      const uint8_t* blk = src[r] + b * bb;
      const uint8_t* qbytes = q4 ? blk + 16 : blk;  // Q4_K qs follow the 16-byte header
      for (int c = 0; c < nc; ++c) std::memcpy(dq + ((b * nc + c) * 512 + r * 16), qbytes + 16 * c, 16);
      if (q4) {
        std::memcpy(ds + (b * 32 + r) * 16, blk, 16);
      } else {
        std::memcpy(ds + (b * 32 + r) * 16, blk + 192, 16);
        std::memcpy(dd + b * 32 + r, blk + 208, 2);
      }
    }
  }
}

void RepackRows(uint32_t type, const uint8_t* src, int64_t rows, int64_t cols, uint8_t* dq, uint8_t* ds,
                uint16_t* dd) {
  RPGB_CHECK(rows % 32 == 0, "rows %lld are not a multiple of 32", static_cast<long long>(rows));
  const int64_t nb = cols / 256;
  const int64_t rb = GgmlRowBytes(type, cols);
  size_t qg, sg, dg;
  DevMatBytes(type, 32, cols, &qg, &sg, &dg);
  for (int64_t g = 0; g < rows / 32; ++g) {
    const uint8_t* ptrs[32];
    for (int r = 0; r < 32; ++r) ptrs[r] = src + (g * 32 + r) * rb;
    RepackGroup(type, ptrs, nb, dq + g * qg, ds + g * sg, dd ? dd + g * (dg / 2) : nullptr);
  }
}

Model::~Model() {
  if (arena_ != nullptr) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device_);
    cudaFree(arena_);
    cudaSetDevice(cur);
  }
}

std::unique_ptr<Model> Model::Load(const std::string& path, int device, int32_t max_pos) {
  std::unique_ptr<Model> m(new Model());
  m->gguf_ = std::make_unique<GgufFile>();
  m->gguf_->Open(path);
  const GgufFile& g = *m->gguf_;
  m->meta_ = ReadModelMeta(g);
  const ModelMeta& c = m->meta_;
  m->device_ = device;

  int n_dev = 0;
  RPGB_CUDA(cudaGetDeviceCount(&n_dev));
  RPGB_CHECK(device >= 0 && device < n_dev, "device %d does not exist (%d visible)", device, n_dev);
  RPGB_CUDA(cudaSetDevice(device));
  RPGB_CUDA(cudaDeviceGetAttribute(&m->num_sms_, cudaDevAttrMultiProcessorCount, device));
  PrepareMatvecKernels();
  PrepareSampleKernels();

  auto require = [&](const std::string& name) -> const GgufTensor& {
    const GgufTensor* t = g.Find(name);
    RPGB_CHECK(t != nullptr, "tensor %s is missing", name.c_str());
    return *t;
  };
  auto check_mat = [&](const GgufTensor& t, int64_t rows, int64_t cols) {
    RPGB_CHECK(t.dims.size() == 2 && t.rows() == rows && t.cols() == cols,
               "tensor %s has shape [%lld,%lld], expected [%lld,%lld]", t.name.c_str(),
               static_cast<long long>(t.rows()), static_cast<long long>(t.cols()), static_cast<long long>(rows),
               static_cast<long long>(cols));
    RPGB_CHECK(t.type == kGgmlQ4_K || t.type == kGgmlQ6_K,
               "tensor %s has type %s; the kernels implement Q4_K and Q6_K", t.name.c_str(),
               GgmlTypeName(t.type));
  };
  auto check_norm = [&](const GgufTensor& t, int64_t n) {
    RPGB_CHECK(t.n_elements == n, "norm %s has %lld elements, expected %lld", t.name.c_str(),
               static_cast<long long>(t.n_elements), static_cast<long long>(n));
    RPGB_CHECK(t.type == kGgmlF32 || t.type == kGgmlF16, "norm %s has type %s (F32 or F16 expected)",
               t.name.c_str(), GgmlTypeName(t.type));
  };

  // ---- plan the arena
  struct MatJob {
    const GgufTensor* a;
    const GgufTensor* b;  // interleaved partner (gate/up) or null
    DevMat* dst;
  };
  struct NormJob {
    const GgufTensor* t;
    const float** dst;
  };
  std::vector<MatJob> mats;
  std::vector<NormJob> norms;
  m->layers_.resize(static_cast<size_t>(c.n_layers));

  const GgufTensor& emb = require("token_embd.weight");
  check_mat(emb, c.vocab, c.hidden);
  mats.push_back({&emb, nullptr, &m->embd_});
  const GgufTensor* out_w = g.Find("output.weight");
  if (out_w == nullptr) out_w = g.Find("lm_head.weight");
  if (out_w != nullptr) {
    check_mat(*out_w, c.vocab, c.hidden);
    mats.push_back({out_w, nullptr, &m->lm_head_});
  }
  const GgufTensor& on = require("output_norm.weight");
  check_norm(on, c.hidden);
  norms.push_back({&on, &m->out_norm_});
  for (int l = 0; l < c.n_layers; ++l) {
    DevLayer& L = m->layers_[static_cast<size_t>(l)];
    const std::string p = "blk." + std::to_string(l) + ".";
    const GgufTensor& an = require(p + "attn_norm.weight");
    const GgufTensor& fn = require(p + "ffn_norm.weight");
    const GgufTensor& qn = require(p + "attn_q_norm.weight");
    const GgufTensor& kn = require(p + "attn_k_norm.weight");
    check_norm(an, c.hidden);
    check_norm(fn, c.hidden);
    check_norm(qn, c.head_dim);
    check_norm(kn, c.head_dim);
    norms.push_back({&an, &L.attn_norm});
    norms.push_back({&fn, &L.ffn_norm});
    norms.push_back({&qn, &L.q_norm});
    norms.push_back({&kn, &L.k_norm});
    const GgufTensor& q = require(p + "attn_q.weight");
    const GgufTensor& k = require(p + "attn_k.weight");
    const GgufTensor& v = require(p + "attn_v.weight");
    const GgufTensor& o = require(p + "attn_output.weight");
    const GgufTensor& ga = require(p + "ffn_gate.weight");
    const GgufTensor& up = require(p + "ffn_up.weight");
    const GgufTensor& dn = require(p + "ffn_down.weight");
    check_mat(q, c.q_dim(), c.hidden);
    check_mat(k, c.kv_dim(), c.hidden);
    check_mat(v, c.kv_dim(), c.hidden);
    check_mat(o, c.hidden, c.q_dim());
    check_mat(ga, c.ffn, c.hidden);
    check_mat(up, c.ffn, c.hidden);
    check_mat(dn, c.hidden, c.ffn);
    RPGB_CHECK(ga.type == up.type, "layer %d: ffn_gate (%s) and ffn_up (%s) must share a type", l,
               GgmlTypeName(ga.type), GgmlTypeName(up.type));
    mats.push_back({&q, nullptr, &L.q});
    mats.push_back({&k, nullptr, &L.k});
    mats.push_back({&v, nullptr, &L.v});
    mats.push_back({&o, nullptr, &L.o});
    mats.push_back({&ga, &up, &L.gateup});
    mats.push_back({&dn, nullptr, &L.down});
  }

  size_t total = 0;
  for (const MatJob& j : mats) {
    size_t q, s, d;
    const int64_t rows = j.a->rows() * (j.b ? 2 : 1);
    DevMatBytes(j.a->type, rows, j.a->cols(), &q, &s, &d);
    total += AlignUp(q) + AlignUp(s) + AlignUp(d);
  }
  for (const NormJob& n : norms) total += AlignUp(static_cast<size_t>(n.t->n_elements) * 4);
  m->rope_pos_ = std::max<int32_t>(1, std::min<int32_t>(max_pos, c.context_length));
  const size_t rope_bytes = static_cast<size_t>(m->rope_pos_) * c.head_dim * 4;
  total += AlignUp(rope_bytes);

  RPGB_CUDA(cudaMalloc(&m->arena_, total));
  m->arena_bytes_ = static_cast<int64_t>(total);
  size_t cursor = 0;
  auto carve = [&](size_t bytes) {
    uint8_t* p = m->arena_ + cursor;
    cursor += AlignUp(bytes);
    return p;
  };

  Staging up(64u << 20);
  // Copies `bytes` of host data through the staging buffer.
  auto upload_plain = [&](void* dst, const void* src, size_t bytes) {
    size_t off = 0;
    while (off < bytes) {
      const size_t n = std::min(up.cap(), bytes - off);
      std::memcpy(up.buf(), static_cast<const uint8_t*>(src) + off, n);
      up.Push(static_cast<uint8_t*>(dst) + off, up.buf(), n);
      up.Wait();
      off += n;
    }
  };

  for (const MatJob& j : mats) {
    const uint32_t type = j.a->type;
    const int64_t cols = j.a->cols();
    const int64_t src_rows = j.a->rows();
    const int64_t rows = src_rows * (j.b ? 2 : 1);
    size_t qb, sb, db;
    DevMatBytes(type, rows, cols, &qb, &sb, &db);
    DevMat dm;
    dm.type = type;
    dm.rows = static_cast<int32_t>(rows);
    dm.cols = static_cast<int32_t>(cols);
    dm.nb = static_cast<int32_t>(cols / 256);
    uint8_t* dq = carve(qb);
    uint8_t* ds = carve(sb);
    uint8_t* dd = db ? carve(db) : nullptr;
    dm.q = dq;
    dm.s = ds;
    dm.d = reinterpret_cast<const uint16_t*>(dd);
    *j.dst = dm;

    const int64_t row_src_bytes = GgmlRowBytes(type, cols);
    size_t qg, sg, dg;  // bytes of one 32-row group
    DevMatBytes(type, 32, cols, &qg, &sg, &dg);
    RPGB_CHECK(rows % 32 == 0, "tensor %s: %lld rows are not a multiple of 32", j.a->name.c_str(),
               static_cast<long long>(rows));
    const int64_t groups = rows / 32;
    const int64_t groups_per_chunk = std::max<int64_t>(1, static_cast<int64_t>(up.cap() / (qg + sg + dg)));
    for (int64_t g0 = 0; g0 < groups; g0 += groups_per_chunk) {
      const int64_t ng = std::min(groups_per_chunk, groups - g0);
      uint8_t* sq = up.buf();
      uint8_t* ss = sq + ng * qg;
      uint16_t* sd = reinterpret_cast<uint16_t*>(ss + ng * sg);
      ParallelRows(ng * 32, [&](int64_t a, int64_t b) {
        for (int64_t gi = a / 32; gi * 32 < b; ++gi) {
          if (gi * 32 < a) continue;
          const uint8_t* ptrs[32];
          for (int r = 0; r < 32; ++r) {
            const int64_t dst_row = (g0 + gi) * 32 + r;
            const GgufTensor* src_t = j.a;
            int64_t src_row = dst_row;
            if (j.b != nullptr) {  // gate/up interleave: 2i = gate row i, 2i+1 = up row i
              src_t = (dst_row & 1) ? j.b : j.a;
              src_row = dst_row >> 1;
            }
            ptrs[r] = g.TensorData(*src_t) + src_row * row_src_bytes;
          }
          RepackGroup(type, ptrs, cols / 256, sq + gi * qg, ss + gi * sg, dg ? sd + gi * (dg / 2) : nullptr);
        }
      });
      up.Push(dq + g0 * qg, sq, ng * qg);
      up.Push(ds + g0 * sg, ss, ng * sg);
      if (dg) up.Push(dd + g0 * dg, reinterpret_cast<const uint8_t*>(sd), ng * dg);
      up.Wait();
    }
  }
  if (out_w == nullptr) m->lm_head_ = m->embd_;

  std::vector<float> tmp;
  for (const NormJob& n : norms) {
    float* dst = reinterpret_cast<float*>(carve(static_cast<size_t>(n.t->n_elements) * 4));
    tmp.resize(static_cast<size_t>(n.t->n_elements));
    if (n.t->type == kGgmlF32) {
      std::memcpy(tmp.data(), g.TensorData(*n.t), tmp.size() * 4);
    } else {
      const uint16_t* h = reinterpret_cast<const uint16_t*>(g.TensorData(*n.t));
      for (size_t i = 0; i < tmp.size(); ++i) tmp[i] = HalfToFloat(h[i]);
    }
    upload_plain(dst, tmp.data(), tmp.size() * 4);
    *n.dst = dst;
  }

  // RoPE table, same algorithm as the reference (src/gpu_model.cu:90-120):
  // angles in double, cos in the first half of each row and sin in the second.
  {
    const int32_t half = c.head_dim / 2;
    std::vector<float> rope(static_cast<size_t>(m->rope_pos_) * c.head_dim);
    std::vector<double> inv(static_cast<size_t>(half));
    for (int32_t i = 0; i < half; ++i) {
      inv[i] = 1.0 / std::pow(static_cast<double>(c.rope_theta),
                              static_cast<double>(2 * i) / static_cast<double>(c.head_dim));
    }
    for (int64_t p = 0; p < m->rope_pos_; ++p) {
      float* row = rope.data() + p * c.head_dim;
      for (int32_t i = 0; i < half; ++i) {
        const double ang = static_cast<double>(p) * inv[i];
        row[i] = static_cast<float>(std::cos(ang));
        row[half + i] = static_cast<float>(std::sin(ang));
      }
    }
    m->rope_ = reinterpret_cast<float*>(carve(rope_bytes));
    upload_plain(m->rope_, rope.data(), rope_bytes);
  }
  up.Wait();
  RPGB_CHECK(cursor <= total, "arena overflow (%zu > %zu)", cursor, total);
  RPGB_INFO("loaded %s: %d layers, hidden %d, vocab %d, %.2f GiB on device %d", c.name.c_str(), c.n_layers,
            c.hidden, c.vocab, static_cast<double>(total) / (1 << 30), device);
  return m;
}

}  // namespace rpgb
