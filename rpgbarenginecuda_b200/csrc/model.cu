// model.cu -- metadata, weight repack + upload, RoPE table.
#include "model.h"

#include <cmath>
#include <cstdlib>
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
  if (rows < 64) nt = 1;
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

int GroupBytes(uint32_t type) {
  if (type == kGgmlQ4_K) return 16 * 144;
  if (type == kGgmlQ6_K) return 16 * 210;
  if (type == kGgmlQ5_K || type == kGgmlQ8_0) return kByteGroupBytes;
  Throw("matrix type %s is not supported (Q4_K, Q5_K, Q6_K and Q8_0 are)", GgmlTypeName(type));
}

size_t DevMatBytes(uint32_t type, int64_t rows, int64_t cols) {
  RPGB_CHECK(rows % kTileRows == 0 && cols % 256 == 0, "matrix %lld x %lld is not whole 16-row tiles",
             static_cast<long long>(rows), static_cast<long long>(cols));
  return static_cast<size_t>(rows / kTileRows) * static_cast<size_t>(cols / 256) * GroupBytes(type);
}

namespace {

// 6-bit value (0..63) of element e of a GGUF Q6_K block (src/quant.cc:321-354 layout).
inline int Q6kRaw(const uint8_t* blk, int e) {
  const int hh = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
  const uint8_t byte = blk[hh * 64 + l + ((quarter & 1) ? 32 : 0)];
  const int nib = quarter < 2 ? (byte & 15) : (byte >> 4);
  const int hi = (blk[128 + hh * 32 + l] >> (2 * quarter)) & 3;
  return nib | (hi << 4);
}

// 5-bit value (0..31) of element e of a GGUF Q5_K block (src/quant.cc:281-313
// layout: low nibbles in qs[32 j + l] for the 64-column group j, fifth bits in
// bit 2 j (first 32 columns) or 2 j + 1 (next 32) of qh[l]).
inline int Q5kRaw(const uint8_t* blk, int e) {
  const int j = e >> 6, hi = (e >> 5) & 1, l = e & 31;
  const uint8_t q = blk[48 + 32 * j + l];
  const int nib = hi ? (q >> 4) : (q & 15);
  return nib | (((blk[16 + l] >> (2 * j + hi)) & 1) << 4);
}

}  // namespace

// Block-group byte order (lane = 4 * g + t, g = 0..7, t = 0..3; rows g and g + 8
// of the tile belong to lane group g):
//   Q4_K  [0, 2048)     per pair c (0..3) and lane, 16 B = words (h, rs) for
//                       h, rs in {0,1}: qs[32c + 16h + 4t .. +3] of row g + 8rs
//         [2048, 2304)  row r: the 16 GGUF header bytes (d, dmin, scales[12])
//   Q6_K  [0, 3072)     per MMA m (0..7) and lane, 12 B = words X, Y, Z holding
//                       the 6-bit values a0 (row g, sub-block 4(m>>1) + (m&1)),
//                       a1 (row g + 8, same), a2 (row g, sub-block + 2), a3 (row
//                       g + 8, sub-block + 2) at positions 4t .. 4t+3: byte e of
//                       X = a0 | a3[1:0] << 6, Y = a1 | a3[3:2] << 6, Z = a2 |
//                       a3[5:4] << 6.  Lane records of MMAs 4q .. 4q+3 are
//                       adjacent (48 B), so a lane reads them as 3 x 16 B.
//         [3072, 3328)  row r: sc[16] (int8)
//         [3328, 3360)  d (f16) of row g + 8rs at index 2g + rs
//   Q5_K, Q8_0 (one byte per weight)
//         [0, 4096)     per pair c (0..3) and lane, 32 B = words (h, half, rs)
//                       at 4 (4h + 2 half + rs): the values of columns
//                       64c + 32 half + 16h + 4t .. +3 of row g + 8rs (Q5_K:
//                       0..31; Q8_0: int8) -- the four A registers of the MMA
//                       of (c, h) read as one 16-byte load
//         [4096, 4352)  row r: Q5_K the 16 header bytes (d, dmin, scales[12]);
//                       Q8_0 the 8 f16 scales of its 32-column blocks
void RepackTile(uint32_t type, const uint8_t* const* src, int64_t nb, uint8_t* dst) {
  const int gb = GroupBytes(type);
  for (int64_t b = 0; b < nb; ++b) {
    uint8_t* o = dst + b * gb;
    if (type == kGgmlQ5_K || type == kGgmlQ8_0) {
      for (int r = 0; r < 16; ++r) {
        if (type == kGgmlQ5_K) {
          std::memcpy(o + 4096 + 16 * r, src[r] + b * 176, 16);
        } else {
          for (int k = 0; k < 8; ++k) std::memcpy(o + 4096 + 16 * r + 2 * k, src[r] + (b * 8 + k) * 34, 2);
        }
      }
      for (int c = 0; c < 4; ++c) {
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, t = lane & 3;
          for (int h = 0; h < 2; ++h) {
            for (int half = 0; half < 2; ++half) {
              for (int rs = 0; rs < 2; ++rs) {
                uint8_t* w = o + (c * 32 + lane) * 32 + 4 * (4 * h + 2 * half + rs);
                for (int e = 0; e < 4; ++e) {
                  const int col = 64 * c + 32 * half + 16 * h + 4 * t + e;
                  const uint8_t* row = src[g + 8 * rs];
                  w[e] = type == kGgmlQ5_K ? static_cast<uint8_t>(Q5kRaw(row + b * 176, col))
                                           : row[(b * 8 + (col >> 5)) * 34 + 2 + (col & 31)];
                }
              }
            }
          }
        }
      }
    } else if (type == kGgmlQ4_K) {
      for (int r = 0; r < 16; ++r) std::memcpy(o + 2048 + 16 * r, src[r] + b * 144, 16);
      for (int c = 0; c < 4; ++c) {
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, t = lane & 3;
          for (int h = 0; h < 2; ++h) {
            for (int rs = 0; rs < 2; ++rs) {
              const uint8_t* qs = src[g + 8 * rs] + b * 144 + 16;
              std::memcpy(o + (c * 32 + lane) * 16 + (2 * h + rs) * 4, qs + 32 * c + 16 * h + 4 * t, 4);
            }
          }
        }
      }
    } else {
      int v[16][256];
      for (int r = 0; r < 16; ++r) {
        const uint8_t* blk = src[r] + b * 210;
        for (int e = 0; e < 256; ++e) v[r][e] = Q6kRaw(blk, e);
        std::memcpy(o + 3072 + 16 * r, blk + 192, 16);
        const int g = r & 7, rs = r >> 3;
        std::memcpy(o + 3328 + 2 * (2 * g + rs), blk + 208, 2);
      }
      for (int m = 0; m < 8; ++m) {
        const int sb0 = 4 * (m >> 1) + (m & 1), sb1 = sb0 + 2;
        for (int lane = 0; lane < 32; ++lane) {
          const int g = lane >> 2, t = lane & 3;
          uint8_t* w = o + ((m >> 2) * 32 + lane) * 48 + (m & 3) * 12;
          for (int e = 0; e < 4; ++e) {
            const int a0 = v[g][16 * sb0 + 4 * t + e], a1 = v[g + 8][16 * sb0 + 4 * t + e];
            const int a2 = v[g][16 * sb1 + 4 * t + e], a3 = v[g + 8][16 * sb1 + 4 * t + e];
            w[e] = static_cast<uint8_t>(a0 | ((a3 & 3) << 6));
            w[4 + e] = static_cast<uint8_t>(a1 | (((a3 >> 2) & 3) << 6));
            w[8 + e] = static_cast<uint8_t>(a2 | (((a3 >> 4) & 3) << 6));
          }
        }
      }
    }
  }
}

void RepackRows(uint32_t type, const uint8_t* src, int64_t rows, int64_t cols, uint8_t* dst) {
  RPGB_CHECK(rows % kTileRows == 0, "rows %lld are not a multiple of %d", static_cast<long long>(rows), kTileRows);
  const int64_t nb = cols / 256;
  const int64_t rb = GgmlRowBytes(type, cols);
  const size_t tile_bytes = static_cast<size_t>(nb) * GroupBytes(type);
  for (int64_t t = 0; t < rows / kTileRows; ++t) {
    const uint8_t* ptrs[kTileRows];
    for (int r = 0; r < kTileRows; ++r) ptrs[r] = src + (t * kTileRows + r) * rb;
    RepackTile(type, ptrs, nb, dst + t * tile_bytes);
  }
}

Model::~Model() {
  if (arena_ != nullptr || half_arena_ != nullptr) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device_);
    if (arena_ != nullptr) cudaFree(arena_);
    if (half_arena_ != nullptr) cudaFree(half_arena_);
    cudaSetDevice(cur);
  }
}

std::unique_ptr<Model> Model::Load(const std::string& path, int device, int32_t max_pos,
                                   std::shared_ptr<TpGroup> tp) {
  std::unique_ptr<Model> m(new Model());
  m->gguf_ = std::make_unique<GgufFile>();
  m->gguf_->Open(path);
  const GgufFile& g = *m->gguf_;
  m->gmeta_ = ReadModelMeta(g);
  const ModelMeta& c = m->gmeta_;
  const int tp_rank = tp ? tp->rank() : 0, tp_size = tp ? tp->size() : 1;
  RPGB_CHECK(!tp || tp->device() == device, "tensor parallel: the group is on device %d, the model on %d",
             tp ? tp->device() : -1, device);
  m->shard_ = MakeShardPlan(c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab, tp_rank, tp_size);
  const ShardPlan& sp = m->shard_;
  m->tp_ = tp;  // a group of one still takes the tensor-parallel path (tests run it on one GPU)
  m->meta_ = c;
  m->meta_.n_heads = sp.heads;
  m->meta_.n_kv_heads = sp.kv_heads;
  m->meta_.ffn = sp.ffn;
  m->device_ = device;

  int n_dev = 0;
  RPGB_CUDA(cudaGetDeviceCount(&n_dev));
  RPGB_CHECK(device >= 0 && device < n_dev, "device %d does not exist (%d visible)", device, n_dev);
  RPGB_CUDA(cudaSetDevice(device));
  RPGB_CUDA(cudaDeviceGetAttribute(&m->num_sms_, cudaDevAttrMultiProcessorCount, device));
  PrepareMatvecKernels();
  PrepareMatvecTokensKernels();
  PrepareSampleKernels();
  PrepareAttentionKernels();
  PrepareLoopKernels(m->num_sms_);
  PrepareTcGemmKernels();
  PrepareFlashKernels();

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
    RPGB_CHECK(MatrixTypeSupported(t.type),
               "tensor %s has type %s; the kernels implement Q4_K, Q5_K, Q6_K and Q8_0", t.name.c_str(),
               GgmlTypeName(t.type));
  };
  auto check_norm = [&](const GgufTensor& t, int64_t n) {
    RPGB_CHECK(t.n_elements == n, "norm %s has %lld elements, expected %lld", t.name.c_str(),
               static_cast<long long>(t.n_elements), static_cast<long long>(n));
    RPGB_CHECK(t.type == kGgmlF32 || t.type == kGgmlF16, "norm %s has type %s (F32 or F16 expected)",
               t.name.c_str(), GgmlTypeName(t.type));
  };

  // ---- plan the arena
  // A matrix to repack: source rows [row0, row0 + rows) of a (and of b) and
  // 256-column super-blocks [blk0, blk0 + nb) of each row.
  struct MatJob {
    const GgufTensor* a;
    const GgufTensor* b;  // interleaved partner (gate/up) or null
    DevMat* dst;
    int64_t row0 = 0, rows = -1, blk0 = 0, nb = -1;
  };
  auto job = [](const GgufTensor* a, const GgufTensor* b, DevMat* dst, int64_t row0, int64_t rows, int64_t blk0,
                int64_t nb) {
    MatJob j{a, b, dst};
    j.row0 = row0;
    j.rows = rows;
    j.blk0 = blk0;
    j.nb = nb;
    return j;
  };
  struct NormJob {
    const GgufTensor* t;
    const float** dst;
  };
  std::vector<MatJob> mats;
  std::vector<NormJob> norms;
  m->layers_.resize(static_cast<size_t>(c.n_layers));

  const int64_t hb = c.hidden / 256;  // super-blocks of a hidden-wide row
  const GgufTensor& emb = require("token_embd.weight");
  check_mat(emb, c.vocab, c.hidden);
  mats.push_back(job(&emb, nullptr, &m->embd_, 0, c.vocab, 0, hb));
  const GgufTensor* out_w = g.Find("output.weight");
  if (out_w == nullptr) out_w = g.Find("lm_head.weight");
  if (out_w != nullptr) {
    check_mat(*out_w, c.vocab, c.hidden);
    mats.push_back(job(out_w, nullptr, &m->lm_head_, sp.vocab0, sp.vocab_rows, 0, hb));
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
    const int64_t lq = static_cast<int64_t>(sp.heads) * c.head_dim, lkv = static_cast<int64_t>(sp.kv_heads) * c.head_dim;
    mats.push_back(job(&q, nullptr, &L.q, sp.rank * lq, lq, 0, hb));
    mats.push_back(job(&k, nullptr, &L.k, sp.rank * lkv, lkv, 0, hb));
    mats.push_back(job(&v, nullptr, &L.v, sp.rank * lkv, lkv, 0, hb));
    mats.push_back(job(&o, nullptr, &L.o, 0, c.hidden, sp.rank * lq / 256, lq / 256));
    mats.push_back(job(&ga, &up, &L.gateup, static_cast<int64_t>(sp.rank) * sp.ffn, sp.ffn, 0, hb));
    mats.push_back(job(&dn, nullptr, &L.down, 0, c.hidden, static_cast<int64_t>(sp.rank) * sp.ffn / 256,
                       sp.ffn / 256));
  }

  size_t total = 0;
  for (const MatJob& j : mats) {
    const int64_t rows = j.rows * (j.b ? 2 : 1);
    RPGB_CHECK(rows % kTileRows == 0, "tensor %s: %lld rows are not a multiple of %d", j.a->name.c_str(),
               static_cast<long long>(rows), kTileRows);
    RPGB_CHECK(j.row0 >= 0 && j.row0 + j.rows <= j.a->rows() && j.blk0 >= 0 && j.nb > 0 &&
                   (j.blk0 + j.nb) * 256 <= j.a->cols(),
               "tensor %s: shard out of range", j.a->name.c_str());
    total += AlignUp(DevMatBytes(j.a->type, rows, j.nb * 256));
  }
  for (const NormJob& n : norms) total += AlignUp(static_cast<size_t>(n.t->n_elements) * 4);
  m->rope_pos_ = std::max<int32_t>(1, std::min<int32_t>(max_pos, c.context_length));
  const size_t rope_bytes = static_cast<size_t>(m->rope_pos_) * c.head_dim * 4;
  total += AlignUp(rope_bytes);
  const size_t layer_table_bytes = sizeof(DevLayer) * static_cast<size_t>(c.n_layers);
  total += AlignUp(layer_table_bytes);

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
    const int64_t cols = j.nb * 256;
    const int64_t rows = j.rows * (j.b ? 2 : 1);
    DevMat dm;
    dm.type = type;
    dm.rows = static_cast<int32_t>(rows);
    dm.cols = static_cast<int32_t>(cols);
    dm.nb = static_cast<int32_t>(cols / 256);
    uint8_t* dq = carve(DevMatBytes(type, rows, cols));
    dm.q = dq;
    *j.dst = dm;

    const int64_t row_src_bytes = GgmlRowBytes(type, j.a->cols());
    const int64_t col_off = GgmlRowBytes(type, 256) * j.blk0;  // first super-block of the shard
    const size_t tile_bytes = static_cast<size_t>(dm.nb) * GroupBytes(type);
    const int64_t tiles = rows / kTileRows;
    const int64_t tiles_per_chunk = std::max<int64_t>(1, static_cast<int64_t>(up.cap() / tile_bytes));
    for (int64_t t0 = 0; t0 < tiles; t0 += tiles_per_chunk) {
      const int64_t nt = std::min(tiles_per_chunk, tiles - t0);
      uint8_t* sq = up.buf();
      ParallelRows(nt, [&](int64_t a, int64_t b) {
        for (int64_t ti = a; ti < b; ++ti) {
          const uint8_t* ptrs[kTileRows];
          for (int r = 0; r < kTileRows; ++r) {
            const int64_t dst_row = (t0 + ti) * kTileRows + r;
            const GgufTensor* src_t = j.a;
            int64_t src_row = dst_row;
            if (j.b != nullptr) {  // gate/up interleave: 2i = gate row i, 2i+1 = up row i
              src_t = (dst_row & 1) ? j.b : j.a;
              src_row = dst_row >> 1;
            }
            ptrs[r] = g.TensorData(*src_t) + (j.row0 + src_row) * row_src_bytes + col_off;
          }
          RepackTile(type, ptrs, dm.nb, sq + ti * tile_bytes);
        }
      });
      up.Push(dq + t0 * tile_bytes, sq, static_cast<size_t>(nt) * tile_bytes);
      up.Wait();
    }
  }
  if (out_w == nullptr) {  // tied: this rank's vocabulary rows of the embedding (whole tiles)
    m->lm_head_ = m->embd_;
    m->lm_head_.rows = sp.vocab_rows;
    m->lm_head_.q = m->embd_.q + static_cast<int64_t>(sp.vocab0 / kTileRows) * m->embd_.nb * GroupBytes(m->embd_.type);
  }

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
  // fp16 hi/lo copies of the layer matrices for the tensor-core prefill GEMM,
  // made once here instead of per prefill call (all hi terms, then all lo
  // terms at the same offsets; q, k, v adjacent so that one GEMM covers
  // them); kept only when the device has room to spare (4 GiB beyond them),
  // otherwise the GEMM expands each matrix into its scratch per call
  {
    size_t halves = 0;
    for (const DevLayer& L : m->layers_) {
      for (const DevMat* w : {&L.q, &L.k, &L.v, &L.o, &L.gateup, &L.down}) {
        halves += static_cast<size_t>(w->rows) * w->cols;
      }
    }
    size_t free_b = 0, total_b = 0;
    RPGB_CUDA(cudaMemGetInfo(&free_b, &total_b));
    // RPGB_PREFILL_COPIES=0: keep no copies (a host that needs the memory)
    const char* env = std::getenv("RPGB_PREFILL_COPIES");
    const bool want = env == nullptr || std::atoi(env) != 0;
    if (want && halves > 0 && free_b > halves * 4 + (static_cast<size_t>(4) << 30) &&
        cudaMalloc(&m->half_arena_, halves * 4) == cudaSuccess) {
      m->half_bytes_ = static_cast<int64_t>(halves * 4);
      __half* h = m->half_arena_;
      for (DevLayer& L : m->layers_) {
        L.qkv = DevMat{};
        L.qkv.rows = L.q.rows + L.k.rows + L.v.rows;
        L.qkv.cols = L.q.cols;
        L.qkv.nb = L.q.nb;
        L.qkv.wh = h;
        L.qkv.wl = h + halves;
        for (DevMat* w : {&L.q, &L.k, &L.v, &L.o, &L.gateup, &L.down}) {
          LaunchDequantSplit(*w, h, h + halves, nullptr);
          w->wh = h;
          w->wl = h + halves;
          h += static_cast<size_t>(w->rows) * w->cols;
        }
      }
      RPGB_CUDA(cudaDeviceSynchronize());
    } else {
      cudaGetLastError();  // a failed allocation leaves no sticky error
    }
  }
  // the layer table read by the decode loop kernel (pointers into this arena)
  {
    DevLayer* t = reinterpret_cast<DevLayer*>(carve(layer_table_bytes));
    upload_plain(t, m->layers_.data(), layer_table_bytes);
    m->layers_dev_ = t;
  }
  up.Wait();
  RPGB_CHECK(cursor <= total, "arena overflow (%zu > %zu)", cursor, total);
  RPGB_INFO("loaded %s: %d layers, hidden %d, vocab %d, %.2f GiB (+ %.2f GiB fp16 prefill operands) on device %d",
            c.name.c_str(), c.n_layers, c.hidden, c.vocab, static_cast<double>(total) / (1 << 30),
            static_cast<double>(m->half_bytes_) / (1 << 30), device);
  return m;
}

}  // namespace rpgb
