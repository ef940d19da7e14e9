// SIMT emulation layer, host API half.  TEST INFRASTRUCTURE ONLY.
//
// The reference's CUDA sources (src/*.cu of RPGBarEngineCUDA) are compiled for
// the host CPU against these headers instead of the CUDA toolkit's, so that the
// reference's own engine and sampler produce golden outputs on a machine with
// no GPU.  "Device" memory is host memory, every stream is synchronous, graph
// capture reports itself unsupported (the reference then takes its own
// per-step launch path, src/qwen3_gpu.cu:532-595), and a kernel launch runs
// every thread of every block as a fiber (simt.cc).  Only the API surface the
// reference uses is declared; names and signatures follow the CUDA runtime so
// the reference compiles unchanged.
#ifndef RPG_ORACLE_EMU_CUDA_RUNTIME_API_H_
#define RPG_ORACLE_EMU_CUDA_RUNTIME_API_H_

#include <cstddef>
#include <cstdint>

enum cudaError_t {
  cudaSuccess = 0,
  cudaErrorInvalidValue = 1,
  cudaErrorMemoryAllocation = 2,
  cudaErrorInvalidDevice = 101,
  cudaErrorNotSupported = 801,
  cudaErrorStreamCaptureUnsupported = 900,
  cudaErrorLaunchFailure = 719,
};

enum cudaMemcpyKind {
  cudaMemcpyHostToHost = 0,
  cudaMemcpyHostToDevice = 1,
  cudaMemcpyDeviceToHost = 2,
  cudaMemcpyDeviceToDevice = 3,
  cudaMemcpyDefault = 4,
};

enum cudaStreamCaptureStatus {
  cudaStreamCaptureStatusNone = 0,
  cudaStreamCaptureStatusActive = 1,
  cudaStreamCaptureStatusInvalidated = 2,
};

enum cudaStreamCaptureMode {
  cudaStreamCaptureModeGlobal = 0,
  cudaStreamCaptureModeThreadLocal = 1,
  cudaStreamCaptureModeRelaxed = 2,
};

enum cudaFuncAttribute {
  cudaFuncAttributeMaxDynamicSharedMemorySize = 8,
};

#define cudaStreamDefault 0x00
#define cudaStreamNonBlocking 0x01

struct CUstream_st;
typedef CUstream_st* cudaStream_t;
struct CUgraph_st;
typedef CUgraph_st* cudaGraph_t;
struct CUgraphExec_st;
typedef CUgraphExec_st* cudaGraphExec_t;

struct cudaDeviceProp {
  char name[256];
  size_t totalGlobalMem;
  size_t sharedMemPerBlock;
  int major;
  int minor;
  int multiProcessorCount;
  int maxThreadsPerBlock;
};

struct dim3 {
  unsigned x, y, z;
  constexpr dim3(unsigned vx = 1, unsigned vy = 1, unsigned vz = 1) : x(vx), y(vy), z(vz) {}
};
struct uint3 {
  unsigned x, y, z;
};

const char* cudaGetErrorString(cudaError_t e);
cudaError_t cudaGetLastError();
cudaError_t cudaPeekAtLastError();
cudaError_t cudaGetDeviceCount(int* n);
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* p, int dev);
cudaError_t cudaSetDevice(int dev);
cudaError_t cudaGetDevice(int* dev);
cudaError_t cudaMemGetInfo(size_t* free_b, size_t* total_b);
cudaError_t cudaDriverGetVersion(int* v);
cudaError_t cudaRuntimeGetVersion(int* v);
cudaError_t cudaDeviceSynchronize();

cudaError_t cudaMalloc(void** p, size_t bytes);
template <class T>
inline cudaError_t cudaMalloc(T** p, size_t bytes) {
  return cudaMalloc(reinterpret_cast<void**>(p), bytes);
}
cudaError_t cudaFree(void* p);
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind);
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s = nullptr);
cudaError_t cudaMemset(void* dst, int value, size_t bytes);
cudaError_t cudaMemsetAsync(void* dst, int value, size_t bytes, cudaStream_t s = nullptr);

cudaError_t cudaStreamCreate(cudaStream_t* s);
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned flags);
cudaError_t cudaStreamDestroy(cudaStream_t s);
cudaError_t cudaStreamSynchronize(cudaStream_t s);
cudaError_t cudaStreamIsCapturing(cudaStream_t s, cudaStreamCaptureStatus* st);
cudaError_t cudaStreamBeginCapture(cudaStream_t s, cudaStreamCaptureMode mode);
cudaError_t cudaStreamEndCapture(cudaStream_t s, cudaGraph_t* g);
cudaError_t cudaGraphInstantiateWithFlags(cudaGraphExec_t* e, cudaGraph_t g, unsigned long long flags);
cudaError_t cudaGraphLaunch(cudaGraphExec_t e, cudaStream_t s);
cudaError_t cudaGraphDestroy(cudaGraph_t g);
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t e);

template <class F>
inline cudaError_t cudaFuncSetAttribute(F*, cudaFuncAttribute, int) {
  return cudaSuccess;
}

#endif  // RPG_ORACLE_EMU_CUDA_RUNTIME_API_H_
