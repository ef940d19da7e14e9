// tp.cu -- shard plan, NCCL group (NCCL is opened with dlopen when a group is
// first made, so the library loads and runs one-GPU work without it), and
// the residual add that follows a reduced partial.
#include "tp.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>

#include "common.h"
#include "kernels.h"

namespace rpgb {

ShardPlan MakeShardPlan(int n_heads, int n_kv_heads, int head_dim, int ffn, int vocab, int rank, int size) {
  RPGB_CHECK(size >= 1 && rank >= 0 && rank < size, "tensor parallel: rank %d of %d", rank, size);
  RPGB_CHECK(n_kv_heads > 0 && n_heads % n_kv_heads == 0, "tensor parallel: %d heads over %d KV heads", n_heads,
             n_kv_heads);
  RPGB_CHECK(n_kv_heads % size == 0, "tensor parallel: %d KV heads do not split over %d ranks", n_kv_heads, size);
  ShardPlan s;
  s.rank = rank;
  s.size = size;
  s.heads = n_heads / size;
  s.kv_heads = n_kv_heads / size;
  RPGB_CHECK(s.heads * head_dim % 256 == 0,
             "tensor parallel: %d heads x %d per rank is not a whole number of 256-column super-blocks of "
             "attn_output",
             s.heads, head_dim);
  RPGB_CHECK(ffn % (size * 256) == 0, "tensor parallel: ffn %d does not split into 256-column super-blocks over %d",
             ffn, size);
  s.ffn = ffn / size;
  RPGB_CHECK(vocab % (size * 16) == 0, "tensor parallel: vocabulary %d does not split into 16-row tiles over %d",
             vocab, size);
  s.vocab_rows = vocab / size;
  s.vocab0 = rank * s.vocab_rows;
  return s;
}

namespace {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& Nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string error;
  std::call_once(once, [] {
    // the process may already hold an NCCL (torch's); the same soname reuses it
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      error = std::string("tensor parallel needs NCCL: dlopen(libnccl.so.2) failed: ") + dlerror();
      return;
    }
    auto sym = [&](const char* name) {
      void* p = dlsym(h, name);
      if (p == nullptr && error.empty()) error = std::string("NCCL symbol missing: ") + name;
      return p;
    };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(sym("ncclAllReduce"));
    api.AllGather = reinterpret_cast<decltype(api.AllGather)>(sym("ncclAllGather"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
  });
  if (!error.empty()) Throw("%s", error.c_str());
  return api;
}

#define RPGB_NCCL(call)                                                                   \
  do {                                                                                    \
    const ncclResult_t r_ = (call);                                                       \
    if (r_ != ncclSuccess) Throw("%s failed: %s", #call, Nccl().GetErrorString(r_));      \
  } while (0)

__global__ void AddInPlaceKernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
  const int64_t n4 = n / 4;
  float4* x4 = reinterpret_cast<float4*>(x);
  const float4* y4 = reinterpret_cast<const float4*>(y);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = x4[i];
    const float4 b = y4[i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    x4[i] = a;
  }
  for (int64_t i = 4 * n4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    x[i] += y[i];
  }
}

}  // namespace

void TpUniqueId(uint8_t* out) {
  static_assert(sizeof(ncclUniqueId) == kTpIdBytes, "ncclUniqueId size");
  ncclUniqueId id;
  RPGB_NCCL(Nccl().GetUniqueId(&id));
  std::memcpy(out, &id, kTpIdBytes);
}

std::shared_ptr<TpGroup> TpGroup::Create(const uint8_t* id, int rank, int size, int device) {
  RPGB_CHECK(id != nullptr, "tensor parallel: no group id");
  RPGB_CHECK(size >= 1 && rank >= 0 && rank < size, "tensor parallel: rank %d of %d", rank, size);
  const NcclApi& api = Nccl();
  RPGB_CUDA(cudaSetDevice(device));
  ncclUniqueId uid;
  std::memcpy(&uid, id, kTpIdBytes);
  ncclComm_t comm = nullptr;
  RPGB_NCCL(api.CommInitRank(&comm, size, uid, rank));
  std::shared_ptr<TpGroup> g(new TpGroup());
  g->comm_ = comm;
  g->rank_ = rank;
  g->size_ = size;
  g->device_ = device;
  return g;
}

TpGroup::~TpGroup() {
  if (comm_ != nullptr) {
    cudaSetDevice(device_);
    Nccl().CommDestroy(static_cast<ncclComm_t>(comm_));
  }
}

void TpGroup::AllReduceSum(float* buf, size_t n, cudaStream_t s) const {
  RPGB_NCCL(Nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm_), s));
}

void TpGroup::AllGatherInPlace(float* buf, size_t n, cudaStream_t s) const {
  RPGB_NCCL(Nccl().AllGather(buf + static_cast<size_t>(rank_) * n, buf, n, ncclFloat32,
                             static_cast<ncclComm_t>(comm_), s));
}

void LaunchAddInPlace(float* x, const float* y, int64_t n, cudaStream_t s) {
  RPGB_CHECK(n > 0, "add: no elements");
  RPGB_CHECK(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0,
             "add: unaligned rows");
  const int64_t blocks = std::min<int64_t>((n / 4 + 255) / 256 + 1, 1184);
  AddInPlaceKernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, y, n);
  RPGB_CUDA(cudaGetLastError());
  CountLaunches(1);
}

}  // namespace rpgb
