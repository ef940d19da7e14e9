// tp.h -- tensor parallelism: the shard plan of a model over `size` GPUs and
// the NCCL group that joins them.
//
// No counterpart in the reference, which runs one GPU.  The split follows
// the usual Megatron layout for a Qwen3 block: each rank holds size-th of
// the query and KV heads (q / k / v rows, attn_output columns) and of the
// FFN (gate / up rows, ffn_down columns), so the only exchange of a layer is
// one sum of a [tokens, hidden] partial after attn_output and one after
// ffn_down.  The embedding, the norms and the residual stream are
// replicated; lm_head rows (the vocabulary) are split and the logits are
// gathered, after which every rank runs the same sampler on the same bytes
// and so draws the same token.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>

namespace rpgb {

struct ModelMeta;

constexpr int kTpIdBytes = 128;  // sizeof(ncclUniqueId)

// Local counts of one rank.  Throws when the model does not split evenly:
// KV heads by size, the rank's attn_output columns (heads x head_dim) and
// FFN columns into whole 256-column super-blocks, vocabulary rows into whole
// 16-row tiles.
struct ShardPlan {
  int rank = 0, size = 1;
  int heads = 0, kv_heads = 0, ffn = 0;
  int vocab0 = 0, vocab_rows = 0;  // lm_head rows [vocab0, vocab0 + vocab_rows)
};
ShardPlan MakeShardPlan(int n_heads, int n_kv_heads, int head_dim, int ffn, int vocab, int rank, int size);

// ncclGetUniqueId: rank 0 creates the id and every rank passes the same bytes.
void TpUniqueId(uint8_t* out);

class TpGroup {
 public:
  // ncclCommInitRank on `device` (collective: every rank calls it).
  static std::shared_ptr<TpGroup> Create(const uint8_t* id, int rank, int size, int device);
  ~TpGroup();
  TpGroup(const TpGroup&) = delete;
  TpGroup& operator=(const TpGroup&) = delete;

  int rank() const { return rank_; }
  int size() const { return size_; }
  int device() const { return device_; }

  // In-place sum of n floats over the group, on stream s.
  void AllReduceSum(float* buf, size_t n, cudaStream_t s) const;
  // In-place gather: rank r's n floats sit at buf + r * n on entry; on exit
  // every rank holds all size * n.
  void AllGatherInPlace(float* buf, size_t n, cudaStream_t s) const;

 private:
  TpGroup() = default;
  void* comm_ = nullptr;  // ncclComm_t
  int rank_ = 0, size_ = 1, device_ = 0;
};

// x[i] += y[i] for i < n (the residual add after a reduced partial).
void LaunchAddInPlace(float* x, const float* y, int64_t n, cudaStream_t s);

}  // namespace rpgb
