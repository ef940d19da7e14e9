// sample_noalloc.cu -- rpgb_sample_noalloc: the token sampler without any
// device-memory allocation.
//
// Why: some hosts of this library cannot allocate GPU memory at the moment
// they sample.  A game or UI thread that drives generation must never block,
// and cudaMalloc / cudaFree synchronise the whole device; a process that has
// handed all of its GPU memory to another allocator's pool (a framework's
// caching allocator, a fixed budget planned at start-up) gets a failure from a
// late cudaMalloc.  rpgb_sample keeps its scratch in per-device buffers that
// its first call allocates; this entry point instead uses one fixed array that
// is part of the library image itself.
//
// Limits and sharing rules:
//  * vocabulary size n <= kNoAllocMaxVocab (262144); larger n is rejected;
//  * the scratch array (about 1.1 MiB) belongs to this file's code module.
//    CUDA loads modules lazily by default, so the array is placed on a GPU
//    when the first call on that device looks up its address (and the sampler
//    kernels' module with it); from then on it is held until the process
//    exits.  With CUDA_MODULE_LOADING=EAGER it is placed when the library's
//    context starts instead.  A host whose GPU memory will later belong to
//    another allocator should make one call per device at set-up;
//  * every call on a device uses the same array and leaves its contents
//    behind.  Nothing in it needs to start at zero: the candidate kernel
//    writes every count it reads and the small sampler kernel always writes
//    the fast-path flag before the general kernel reads it (the flag is also
//    cleared up front, defensively).  Two calls whose GPU work overlaps
//    (different streams, or another thread) race on the array and may return
//    wrong tokens -- serialise them;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) and sets the sampler kernels' shared-memory limit;
//    make that first call before any stream capture is in progress.
#include "../../include/rpg_b200.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.h"
#include "kernels.h"

namespace rpgb {
namespace {

constexpr int kNoAllocMaxVocab = RPGB_SAMPLE_NOALLOC_MAX_VOCAB;
constexpr int kMaxDevices = 64;

// Byte offsets inside the scratch array (each piece 256-byte aligned).
constexpr size_t Al(size_t v) { return (v + 255) / 256 * 256; }
constexpr size_t kOffProbs = 0;
constexpr size_t kOffCandVal = kOffProbs + Al(sizeof(float) * kNoAllocMaxVocab);
constexpr size_t kOffCandIdx = kOffCandVal + Al(sizeof(float) * kCandBlocks * kFastTopK);
constexpr size_t kOffCandCnt = kOffCandIdx + Al(sizeof(int32_t) * kCandBlocks * kFastTopK);
constexpr size_t kOffFlag = kOffCandCnt + Al(sizeof(int32_t) * kCandBlocks);
constexpr size_t kOffCounter = kOffFlag + Al(sizeof(int32_t));
constexpr size_t kScratchBytes = kOffCounter + Al(sizeof(int64_t));

// Host code must never use this name as a device address: it only stands in
// for the symbol.  The device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
uint8_t* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
uint8_t* ScratchOnCurrentDevice() {
  int dev = 0;
  RPGB_CUDA(cudaGetDevice(&dev));
  RPGB_CHECK(dev >= 0 && dev < kMaxDevices, "device %d is beyond the %d devices this entry point serves", dev,
             kMaxDevices);
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    RPGB_CHECK(e == cudaSuccess && p != nullptr, "sample_noalloc: scratch address lookup failed on device %d: %s",
               dev, cudaGetErrorString(e));
    PrepareSampleKernels();
    g_scratch_addr[dev] = static_cast<uint8_t*>(p);
  }
  return g_scratch_addr[dev];
}

}  // namespace
}  // namespace rpgb

using namespace rpgb;

extern "C" {

int32_t rpgb_sample_noalloc(const float* logits_dev, int32_t n, const rpgb_sample_options* opt, uint64_t seed,
                            uint64_t counter, int32_t* out_tok_dev, void* stream) {
  try {
    SetLastError("");
    RPGB_CHECK(logits_dev != nullptr && out_tok_dev != nullptr && opt != nullptr, "null argument");
    RPGB_CHECK(n > 0, "vocabulary size must be positive");
    RPGB_CHECK(n <= kNoAllocMaxVocab, "sample_noalloc: vocabulary %d exceeds the fixed scratch limit of %d", n,
               kNoAllocMaxVocab);
    uint8_t* base = ScratchOnCurrentDevice();
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t ctr = static_cast<int64_t>(counter);
    int64_t* d_counter = reinterpret_cast<int64_t*>(base + kOffCounter);
    int32_t* d_flag = reinterpret_cast<int32_t*>(base + kOffFlag);
    RPGB_CUDA(cudaMemcpyAsync(d_counter, &ctr, sizeof(int64_t), cudaMemcpyHostToDevice, s));
    RPGB_CUDA(cudaMemsetAsync(d_flag, 0, sizeof(int32_t), s));  // defensive: the small kernel writes it
    SampleParams p;
    p.logits = logits_dev;
    p.n = n;
    p.temperature = opt->temperature;
    p.top_k = opt->top_k;
    p.top_p = opt->top_p;
    p.seed = seed;
    p.counter_override = d_counter;
    p.probs = reinterpret_cast<float*>(base + kOffProbs);
    p.tok_out = out_tok_dev;
    p.cand_val = reinterpret_cast<float*>(base + kOffCandVal);
    p.cand_idx = reinterpret_cast<int32_t*>(base + kOffCandIdx);
    p.cand_cnt = reinterpret_cast<int32_t*>(base + kOffCandCnt);
    p.flag = d_flag;
    LaunchSample(p, false, s);
    // the counter is copied from this stack frame: finish before returning
    RPGB_CUDA(cudaStreamSynchronize(s));
    return 0;
  } catch (const std::exception& e) {
    SetLastError(e.what());
    return -1;
  } catch (...) {
    SetLastError("unknown exception (not std::exception)");
    return -1;
  }
}

}  // extern "C"
