// SIMT emulation layer runtime.  TEST INFRASTRUCTURE ONLY (see
// cuda_runtime_api.h).
//
// Execution model: a launch hands its blocks to a pool of worker threads (one
// per host core; RPGEMU_THREADS overrides).  A worker runs a block by giving
// each of its threads a fiber (its own stack, switched with a six-register
// context switch) and resuming them in order: a thread runs until it reaches
// __syncthreads() or returns, so one pass over the block's unfinished fibers
// is exactly one barrier interval.  Blocks of one launch run concurrently on
// different workers and never share state, as on a GPU.
//
// Memory: "device" allocations are host allocations filled with 0xFF bytes
// (NaN as floats), so that reads of never-written memory show up in the
// outputs instead of reading as zeros; see Slack() for their size.
#include <sys/mman.h>
#include <unistd.h>

#include <atomic>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "cuda_runtime.h"

thread_local uint3 threadIdx;
thread_local uint3 blockIdx;
thread_local dim3 blockDim;
thread_local dim3 gridDim;

extern "C" void rpgemu_switch(void** save_sp, void* new_sp);

// Saves the callee-saved registers of the System V x86-64 ABI on the current
// stack, stores the stack pointer in *save_sp, loads new_sp and restores the
// registers saved there.
asm(R"(
.text
.globl rpgemu_switch
.type rpgemu_switch,@function
rpgemu_switch:
  pushq %rbp
  pushq %rbx
  pushq %r12
  pushq %r13
  pushq %r14
  pushq %r15
  movq %rsp, (%rdi)
  movq %rsi, %rsp
  popq %r15
  popq %r14
  popq %r13
  popq %r12
  popq %rbx
  popq %rbp
  ret
.size rpgemu_switch, .-rpgemu_switch
)");

namespace {

constexpr size_t kStack = 256 * 1024;  // per emulated thread
constexpr size_t kGuard = 4096;

thread_local cudaError_t t_last_error = cudaSuccess;

struct Fiber {
  void* sp = nullptr;
  char* base = nullptr;  // mapping including the guard page
  bool done = false;
  uint3 tid{0, 0, 0};
};

struct Job {
  dim3 grid, block;
  size_t smem = 0;
  void (*body)(const void*) = nullptr;
  const void* ctx = nullptr;
  int64_t n_blocks = 0;
  std::atomic<int64_t> next{0};
};

struct Worker {
  std::vector<Fiber> fibers;
  std::vector<unsigned char> smem;
  void* sched_sp = nullptr;
  Fiber* cur = nullptr;
  const Job* job = nullptr;
};

thread_local Worker t_worker;

[[noreturn]] void FiberEntry() {
  Worker& w = t_worker;
  w.job->body(w.job->ctx);
  w.cur->done = true;
  rpgemu_switch(&w.cur->sp, w.sched_sp);
  std::abort();  // a finished fiber is never resumed
}

void EnsureFibers(Worker& w, size_t n) {
  while (w.fibers.size() < n) {
    Fiber f;
    void* m = mmap(nullptr, kStack + kGuard, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE,
                   -1, 0);
    if (m == MAP_FAILED) {
      std::fprintf(stderr, "rpgemu: cannot map a fiber stack\n");
      std::abort();
    }
    mprotect(m, kGuard, PROT_NONE);  // a stack overflow faults instead of corrupting a neighbour
    f.base = static_cast<char*>(m);
    w.fibers.push_back(f);
  }
}

void ResetFiber(Fiber& f) {
  uintptr_t* sp = reinterpret_cast<uintptr_t*>(f.base + kGuard + kStack);  // 16-byte aligned top
  *--sp = 0;                                          // return address slot of FiberEntry's frame
  *--sp = reinterpret_cast<uintptr_t>(&FiberEntry);  // taken by rpgemu_switch's ret
  for (int i = 0; i < 6; ++i) *--sp = 0;              // rbp rbx r12 r13 r14 r15
  f.sp = sp;
  f.done = false;
}

void RunBlock(Worker& w, const Job& j, int64_t b) {
  const int64_t gx = j.grid.x, gy = j.grid.y;
  blockIdx = uint3{static_cast<unsigned>(b % gx), static_cast<unsigned>((b / gx) % gy),
                   static_cast<unsigned>(b / (gx * gy))};
  blockDim = j.block;
  gridDim = j.grid;
  const size_t n = static_cast<size_t>(j.block.x) * j.block.y * j.block.z;
  EnsureFibers(w, n);
  if (w.smem.size() < j.smem) w.smem.resize(j.smem);
  if (j.smem > 0) std::memset(w.smem.data(), 0xFF, j.smem);
  for (size_t i = 0; i < n; ++i) {
    Fiber& f = w.fibers[i];
    ResetFiber(f);
    f.tid = uint3{static_cast<unsigned>(i % j.block.x), static_cast<unsigned>((i / j.block.x) % j.block.y),
                  static_cast<unsigned>(i / (static_cast<size_t>(j.block.x) * j.block.y))};
  }
  w.job = &j;
  size_t remaining = n;
  while (remaining > 0) {
    for (size_t i = 0; i < n; ++i) {
      Fiber& f = w.fibers[i];
      if (f.done) continue;
      threadIdx = f.tid;
      w.cur = &f;
      rpgemu_switch(&w.sched_sp, f.sp);
      if (f.done) --remaining;
    }
  }
  w.cur = nullptr;
  w.job = nullptr;
}

void DrainJob(Job& j) {
  Worker& w = t_worker;
  for (;;) {
    const int64_t b = j.next.fetch_add(1);
    if (b >= j.n_blocks) break;
    RunBlock(w, j, b);
  }
}

class Pool {
 public:
  Pool() {
    int n = static_cast<int>(std::thread::hardware_concurrency());
    if (const char* e = std::getenv("RPGEMU_THREADS")) n = std::atoi(e);
    if (n < 1) n = 1;
    for (int i = 1; i < n; ++i) threads_.emplace_back([this] { Loop(); });
  }
  void Run(Job& j) {
    if (threads_.empty() || j.n_blocks == 1) {
      DrainJob(j);
      return;
    }
    std::unique_lock<std::mutex> g(run_mu_);  // one launch at a time
    {
      std::lock_guard<std::mutex> l(mu_);
      job_ = &j;
      busy_ = static_cast<int>(threads_.size());
      ++gen_;
    }
    cv_.notify_all();
    DrainJob(j);
    std::unique_lock<std::mutex> l(mu_);
    done_cv_.wait(l, [this] { return busy_ == 0; });
    job_ = nullptr;
  }

 private:
  void Loop() {
    uint64_t seen = 0;
    for (;;) {
      Job* j;
      {
        std::unique_lock<std::mutex> l(mu_);
        cv_.wait(l, [&] { return gen_ != seen; });
        seen = gen_;
        j = job_;
      }
      DrainJob(*j);
      {
        std::lock_guard<std::mutex> l(mu_);
        if (--busy_ == 0) done_cv_.notify_all();
      }
    }
  }
  std::vector<std::thread> threads_;
  std::mutex mu_, run_mu_;
  std::condition_variable cv_, done_cv_;
  Job* job_ = nullptr;
  int busy_ = 0;
  uint64_t gen_ = 0;
};

Pool& ThePool() {
  static Pool* p = new Pool();  // never destroyed: its workers live until the process exits
  return *p;
}

cudaError_t Fail(cudaError_t e) {
  t_last_error = e;
  return e;
}

struct FakeHandle {
  int tag;
};

// Bytes added after every allocation (RPGEMU_EXACT=1: none).  The reference's
// RopeKernel has no bounds check (src/kernels_gpu.cu:598-621): when rows x
// heads x head_dim / 2 is not a multiple of its 256-thread blocks, the last
// block reads and writes one row past the end of the rotated buffer (the k
// buffer with two KV heads and an odd token count).  On a GPU that row lands
// in whatever memory follows; here it lands in this slack, so the in-bounds
// results are what the reference computes.  The exact mode lets an address
// sanitizer report such accesses.
size_t Slack() {
  static const size_t s = [] {
    const char* e = std::getenv("RPGEMU_EXACT");
    return (e != nullptr && e[0] == '1') ? size_t(0) : size_t(1) << 16;
  }();
  return s;
}

}  // namespace

extern "C" void rpgemu_barrier() {
  Worker& w = t_worker;
  if (w.cur == nullptr) return;  // host code outside a kernel
  rpgemu_switch(&w.cur->sp, w.sched_sp);
}

namespace rpgemu {

void* DynSmem() { return t_worker.smem.data(); }

cudaError_t LaunchImpl(dim3 grid, dim3 block, size_t smem_bytes, void (*body)(const void*), const void* ctx) {
  const int64_t nt = static_cast<int64_t>(block.x) * block.y * block.z;
  const int64_t nb = static_cast<int64_t>(grid.x) * grid.y * grid.z;
  if (nt <= 0 || nt > 1024 || nb <= 0 || grid.y > 65535 || grid.z > 65535 || smem_bytes > 227 * 1024) {
    return Fail(cudaErrorInvalidValue);
  }
  Job j;
  j.grid = grid;
  j.block = block;
  j.smem = smem_bytes;
  j.body = body;
  j.ctx = ctx;
  j.n_blocks = nb;
  ThePool().Run(j);
  return cudaSuccess;
}

}  // namespace rpgemu

const char* cudaGetErrorString(cudaError_t e) {
  switch (e) {
    case cudaSuccess: return "no error";
    case cudaErrorInvalidValue: return "invalid argument (emulated launch configuration)";
    case cudaErrorMemoryAllocation: return "out of memory (emulated)";
    case cudaErrorInvalidDevice: return "invalid device ordinal (emulated)";
    case cudaErrorNotSupported: return "operation not supported (emulated)";
    case cudaErrorStreamCaptureUnsupported: return "stream capture is not supported by the emulation";
    default: return "unknown emulated error";
  }
}
cudaError_t cudaGetLastError() {
  const cudaError_t e = t_last_error;
  t_last_error = cudaSuccess;
  return e;
}
cudaError_t cudaPeekAtLastError() { return t_last_error; }
cudaError_t cudaGetDeviceCount(int* n) {
  *n = 1;
  return cudaSuccess;
}
cudaError_t cudaGetDeviceProperties(cudaDeviceProp* p, int dev) {
  if (dev != 0) return Fail(cudaErrorInvalidDevice);
  std::memset(p, 0, sizeof(*p));
  std::snprintf(p->name, sizeof(p->name), "SIMT emulation on the host CPU");
  p->totalGlobalMem = size_t(64) << 30;
  p->sharedMemPerBlock = 48 * 1024;
  p->major = 10;
  p->minor = 0;
  p->multiProcessorCount = static_cast<int>(std::thread::hardware_concurrency());
  p->maxThreadsPerBlock = 1024;
  return cudaSuccess;
}
cudaError_t cudaSetDevice(int dev) { return dev == 0 ? cudaSuccess : Fail(cudaErrorInvalidDevice); }
cudaError_t cudaGetDevice(int* dev) {
  *dev = 0;
  return cudaSuccess;
}
cudaError_t cudaMemGetInfo(size_t* free_b, size_t* total_b) {
  const size_t pages = static_cast<size_t>(sysconf(_SC_PHYS_PAGES));
  const size_t avail = static_cast<size_t>(sysconf(_SC_AVPHYS_PAGES));
  const size_t ps = static_cast<size_t>(sysconf(_SC_PAGESIZE));
  *total_b = pages * ps;
  *free_b = avail * ps;
  return cudaSuccess;
}
cudaError_t cudaDriverGetVersion(int* v) {
  *v = 12090;
  return cudaSuccess;
}
cudaError_t cudaRuntimeGetVersion(int* v) {
  *v = 12090;
  return cudaSuccess;
}
cudaError_t cudaDeviceSynchronize() { return cudaSuccess; }

cudaError_t cudaMalloc(void** p, size_t bytes) {
  void* m = nullptr;
  if (bytes == 0 || posix_memalign(&m, 256, bytes + Slack()) != 0) return Fail(cudaErrorMemoryAllocation);
  std::memset(m, 0xFF, bytes + Slack());
  *p = m;
  return cudaSuccess;
}
cudaError_t cudaFree(void* p) {
  std::free(p);
  return cudaSuccess;
}
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind) {
  if (bytes > 0) std::memmove(dst, src, bytes);
  return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t) {
  return cudaMemcpy(dst, src, bytes, kind);
}
cudaError_t cudaMemset(void* dst, int value, size_t bytes) {
  std::memset(dst, value, bytes);
  return cudaSuccess;
}
cudaError_t cudaMemsetAsync(void* dst, int value, size_t bytes, cudaStream_t) { return cudaMemset(dst, value, bytes); }

cudaError_t cudaStreamCreate(cudaStream_t* s) {
  *s = reinterpret_cast<cudaStream_t>(new FakeHandle{1});
  return cudaSuccess;
}
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned) { return cudaStreamCreate(s); }
cudaError_t cudaStreamDestroy(cudaStream_t s) {
  delete reinterpret_cast<FakeHandle*>(s);
  return cudaSuccess;
}
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamIsCapturing(cudaStream_t, cudaStreamCaptureStatus* st) {
  *st = cudaStreamCaptureStatusNone;
  return cudaSuccess;
}
// Graph capture is refused without touching the sticky launch error, so the
// caller can take its per-step path.
cudaError_t cudaStreamBeginCapture(cudaStream_t, cudaStreamCaptureMode) { return cudaErrorStreamCaptureUnsupported; }
cudaError_t cudaStreamEndCapture(cudaStream_t, cudaGraph_t* g) {
  *g = nullptr;
  return cudaErrorStreamCaptureUnsupported;
}
cudaError_t cudaGraphInstantiateWithFlags(cudaGraphExec_t* e, cudaGraph_t, unsigned long long) {
  *e = nullptr;
  return cudaErrorNotSupported;
}
cudaError_t cudaGraphLaunch(cudaGraphExec_t, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t cudaGraphDestroy(cudaGraph_t) { return cudaSuccess; }
cudaError_t cudaGraphExecDestroy(cudaGraphExec_t) { return cudaSuccess; }
