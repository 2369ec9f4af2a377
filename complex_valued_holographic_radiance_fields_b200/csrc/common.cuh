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

// Complex arithmetic on the packed f32x2 datapath (sm_100): one instruction per complex
// add/sub (operand negation is free), two per complex product; each lane is an IEEE-rounded
// float operation.  The FFT butterflies use these.
__device__ __forceinline__ float2 padd(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 psub(float2 a, float2 b) { return __fadd2_rn(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ float2 pscale(float s, float2 a) { return __fmul2_rn(make_float2(s, s), a); }
// c + s a
__device__ __forceinline__ float2 pfma(float s, float2 a, float2 c) { return __ffma2_rn(make_float2(s, s), a, c); }
// a b (complex)
__device__ __forceinline__ float2 pmul(float2 a, float2 b) {
  return __ffma2_rn(make_float2(-a.y, a.y), make_float2(b.y, b.x), __fmul2_rn(make_float2(a.x, a.x), b));
}
// a conj(b)
__device__ __forceinline__ float2 pmulc(float2 a, float2 b) {
  return __ffma2_rn(make_float2(a.y, -a.y), make_float2(b.y, b.x), __fmul2_rn(make_float2(a.x, a.x), make_float2(b.x, -b.y)));
}

// Asynchronous 8-byte global -> shared copy (sm_80+ cp.async), its group commit and wait.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// ---- bulk asynchronous copies (TMA, this CTA only) completing on a shared-memory mbarrier ----
__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// makes an initialised mbarrier visible to the asynchronous (TMA) proxy
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// orders this thread's earlier generic-proxy shared-memory accesses before later
// asynchronous-proxy (TMA) accesses to the same memory
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
// global -> shared bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned)
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

}  // namespace cvhrf
