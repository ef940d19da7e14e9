// SIMT emulation layer, device half.  TEST INFRASTRUCTURE ONLY (see
// cuda_runtime_api.h for what the layer is for).
//
// Kernel code compiles as plain C++: the execution-space qualifiers vanish,
// `__shared__` variables become thread_local statics (one worker thread runs
// one block at a time, so they are per block), `threadIdx` / `blockIdx` /
// `blockDim` / `gridDim` are thread_local values the scheduler sets before it
// resumes a thread's fiber, and `__syncthreads()` switches back to the
// scheduler, which resumes the next thread of the block.  A launch
// `K<<<g, b, sh, s>>>(args)` is rewritten by prep_cu.py into
// `::rpgemu::Launch(g, b, sh, s, &K, args)`: the arguments are evaluated once
// and every thread of every block calls K with them.  The intrinsics the
// reference uses are the IEEE operations they name (round-to-nearest multiply
// and subtract; the sources are compiled with -ffp-contract=off, so nothing is
// fused); library math (expf, sqrtf, ...) is the host C library's.
#ifndef RPG_ORACLE_EMU_CUDA_RUNTIME_H_
#define RPG_ORACLE_EMU_CUDA_RUNTIME_H_

#include <cmath>
#include <cstdint>
#include <cstring>
#include <tuple>
#include <utility>

#include "cuda_fp16.h"
#include "cuda_runtime_api.h"

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __noinline__
#define __launch_bounds__(...)
#define __shared__ static thread_local

extern thread_local uint3 threadIdx;
extern thread_local uint3 blockIdx;
extern thread_local dim3 blockDim;
extern thread_local dim3 gridDim;

extern "C" void rpgemu_barrier();

inline void __syncthreads() {
  asm volatile("" ::: "memory");
  rpgemu_barrier();
  asm volatile("" ::: "memory");
}

inline float __fmul_rn(float a, float b) { return a * b; }
inline float __fsub_rn(float a, float b) { return a - b; }
inline float __fadd_rn(float a, float b) { return a + b; }
inline unsigned __float_as_uint(float f) {
  unsigned u;
  std::memcpy(&u, &f, 4);
  return u;
}
inline float __uint_as_float(unsigned u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

namespace rpgemu {

// Dynamic shared memory of the block the calling worker runs.
void* DynSmem();

// Runs body(ctx) once per thread of every block of the grid.
cudaError_t LaunchImpl(dim3 grid, dim3 block, size_t smem_bytes, void (*body)(const void*), const void* ctx);

template <class... P, class... A>
void Launch(dim3 grid, dim3 block, size_t smem_bytes, cudaStream_t, void (*fn)(P...), A&&... a) {
  struct Ctx {
    void (*fn)(P...);
    std::tuple<std::decay_t<A>...> args;
  };
  const Ctx ctx{fn, std::tuple<std::decay_t<A>...>(std::forward<A>(a)...)};
  LaunchImpl(grid, block, smem_bytes,
             [](const void* c) {
               const Ctx* x = static_cast<const Ctx*>(c);
               std::apply(x->fn, x->args);
             },
             &ctx);
}

}  // namespace rpgemu

#endif  // RPG_ORACLE_EMU_CUDA_RUNTIME_H_
