// model.h -- Qwen3 metadata and the device-resident, repacked weights.
//
// Reference counterparts: ModelMeta / ReadModelMeta (src/model_meta.h:27-62,
// src/model_meta.cc:11-77), GpuModel::Load (src/gpu_model.cu:148-246) and
// BuildRopeTable (src/gpu_model.cu:90-120).
//
// Difference by design: the reference uploads raw GGUF blocks (144 B Q4_K,
// 210 B Q6_K) and reads them byte by byte.  Here a matrix is stored as 16-row
// tiles; the 16 blocks of one tile and one 256-column super-block form a
// contiguous "block group" (Q4_K 2304 B, Q6_K 3360 B -- exactly 16 GGUF
// blocks) whose bytes are laid out in the register order of the integer
// tensor-core fragments used by the decode matvec (see kernels.cuh).  The
// repack is lossless: dequantisation reproduces src/quant.cc bit for bit.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "gguf.h"
#include "tp.h"

namespace rpgb {

struct ModelMeta {
  std::string arch, name;
  int32_t n_layers = 0, hidden = 0, n_heads = 0, n_kv_heads = 0, head_dim = 0, ffn = 0;
  int32_t vocab = 0, context_length = 0;
  float rope_theta = 10000.0f, rms_eps = 1e-6f;
  int32_t bos_id = -1, eos_id = -1, pad_id = -1;
  bool add_bos = false, tied = true;
  int64_t weight_bytes = 0;
  int32_t q_dim() const { return n_heads * head_dim; }
  int32_t kv_dim() const { return n_kv_heads * head_dim; }
  int32_t group() const { return n_heads / n_kv_heads; }
};

ModelMeta ReadModelMeta(const GgufFile& g);

// One quantised matrix in the repacked device layout (passed to kernels by value).
// Block group (tile t, super-block b) starts at q + (t * nb + b) * GroupBytes(type).
// wh / wl, when set, are the same matrix dequantised once into two fp16
// terms (row-major [rows][cols]; wh + wl is the bit-exact dequantised value
// to ~22 bits): the operands of the tensor-core prefill GEMM, which then
// needs no per-call expansion.
struct DevMat {
  uint32_t type = 0;  // kGgmlQ4_K, kGgmlQ5_K, kGgmlQ6_K or kGgmlQ8_0
  int32_t rows = 0, cols = 0, nb = 0;
  const uint8_t* q = nullptr;
  const __half* wh = nullptr;
  const __half* wl = nullptr;
};

struct DevLayer {
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  DevMat q, k, v, o;
  DevMat gateup;  // rows interleaved: 2i = ffn_gate row i, 2i+1 = ffn_up row i
  DevMat down;
  // q, k and v as one fp16 matrix [q rows; k rows; v rows] (only wh / wl
  // are set; null when the model keeps no fp16 copy): one prefill GEMM
  // writes the concatenated q | k | v row of every token
  DevMat qkv;
};

// Host-side repack of GGUF blocks into the device layout.  RepackTile takes
// the 16 source rows of one tile by pointer (gate/up interleave) and writes
// nb block groups; RepackRows takes `rows` (a multiple of 16) contiguous GGUF
// rows.  DevMatBytes = rows / 16 * nb * GroupBytes(type).
constexpr int kTileRows = 16;
// Bytes of a Q5_K or Q8_0 block group (one byte per weight plus 256 bytes of
// per-row scales); Q4_K groups are 2304 bytes, Q6_K 3360.
constexpr int kByteGroupBytes = 4352;
int GroupBytes(uint32_t type);
void RepackTile(uint32_t type, const uint8_t* const* src_rows, int64_t nb, uint8_t* dst);
void RepackRows(uint32_t type, const uint8_t* src, int64_t rows, int64_t cols, uint8_t* dst);
size_t DevMatBytes(uint32_t type, int64_t rows, int64_t cols);

class Model {
 public:
  // Loads weights onto `device`, builds the RoPE table for min(max_pos, context).
  // With a tensor-parallel group (size > 1) only this rank's shard is loaded:
  // its heads' q / k / v rows and attn_output columns, its FFN rows (gate, up)
  // and columns (down), its vocabulary rows of lm_head; embedding and norms in
  // full (ShardPlan in tp.h).
  static std::unique_ptr<Model> Load(const std::string& path, int device, int32_t max_pos,
                                     std::shared_ptr<TpGroup> tp = nullptr);
  ~Model();

  // The shapes this device computes with: heads, KV heads and ffn are the
  // shard's (the whole model without a group); hidden, vocab and the rest are
  // the model's.
  const ModelMeta& meta() const { return meta_; }
  // The model's own shapes (what the GGUF holds).
  const ModelMeta& global_meta() const { return gmeta_; }
  const TpGroup* tp() const { return tp_.get(); }
  const ShardPlan& shard() const { return shard_; }
  const GgufFile& gguf() const { return *gguf_; }
  int device() const { return device_; }
  int num_sms() const { return num_sms_; }
  const std::vector<DevLayer>& layers() const { return layers_; }
  const DevLayer* layers_dev() const { return layers_dev_; }  // the same table in device memory
  const DevMat& embd() const { return embd_; }
  const DevMat& lm_head() const { return lm_head_; }
  const float* out_norm() const { return out_norm_; }
  const float* rope() const { return rope_; }
  int32_t rope_positions() const { return rope_pos_; }
  int64_t device_bytes() const { return arena_bytes_ + half_bytes_; }
  // Bytes of the fp16 hi/lo copies of the layer matrices (0 when there is no room for them).
  int64_t half_bytes() const { return half_bytes_; }

 private:
  Model() = default;
  std::unique_ptr<GgufFile> gguf_;
  ModelMeta meta_, gmeta_;
  std::shared_ptr<TpGroup> tp_;
  ShardPlan shard_;
  int device_ = 0;
  int num_sms_ = 0;
  uint8_t* arena_ = nullptr;
  int64_t arena_bytes_ = 0;
  __half* half_arena_ = nullptr;
  int64_t half_bytes_ = 0;
  std::vector<DevLayer> layers_;
  const DevLayer* layers_dev_ = nullptr;
  DevMat embd_, lm_head_;
  const float* out_norm_ = nullptr;
  float* rope_ = nullptr;
  int32_t rope_pos_ = 0;
};

}  // namespace rpgb
