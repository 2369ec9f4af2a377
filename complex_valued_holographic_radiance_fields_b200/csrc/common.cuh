// Shared helpers for the cvhrf CUDA sources: status plumbing and small math.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>
#include "../../include/cvhrf.h"

namespace cvhrf {

// Records the failing cudaError_t for cvhrf_last_cuda_error() (defined in capi.cu).
void set_last_cuda_error(int err);
// Adds n to the process-wide count of kernels this library has launched (capi.cu).
void count_launch(int n);

#define CVHRF_CUDA_TRY(expr)                                    \
  do {                                                          \
    cudaError_t _e = (expr);                                    \
    if (_e != cudaSuccess) {                                    \
      ::cvhrf::set_last_cuda_error((int)_e);                    \
      return CVHRF_ECUDA;                                       \
    }                                                           \
  } while (0)

#define CVHRF_LAUNCH_CHECK()        \
  do {                              \
    ::cvhrf::count_launch(1);       \
    CVHRF_CUDA_TRY(cudaGetLastError()); \
  } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
constexpr size_t align_up_c(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Carves 256-byte aligned sub-buffers out of a caller-provided workspace.
struct Carver {
  char* base;
  size_t cap;
  size_t used = 0;
  bool overflow = false;
  Carver(void* b, size_t c) : base((char*)b), cap(c) {}
  template <typename T>
  T* take(size_t count) {
    size_t off = align_up(used, 256);
    size_t bytes = count * sizeof(T);
    used = off + bytes;
    if (used > cap) { overflow = true; return nullptr; }
    return base ? reinterpret_cast<T*>(base + off) : nullptr;  // null base: size query only
  }
};

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }

// Asynchronous 8-byte global -> shared copy (sm_80+ cp.async), its group commit and wait.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

}  // namespace cvhrf
