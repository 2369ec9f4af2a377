// L2 intensity loss of the training iteration, fused (train.py computes it with torch
// elementwise ops: loss = mean((|holo|^2 - target)^2) over C x S x S).
//
// Forward: one launch; blocks reduce grid-stride partial sums of r^2 (r = re^2 + im^2 -
// target) and the last block to finish sums the partials in a fixed order (deterministic)
// and writes loss = sum / n.  Backward: one elementwise launch,
//   dL/dholo = (g / n) * 2 r * 2 (re, im)     (g = upstream gradient, a device scalar)
// in torch's convention for complex inputs (d/dre + i d/dim).
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kLossThreads = 256;
constexpr int kLossMaxBlocks = 148 * 4;

__global__ void __launch_bounds__(kLossThreads) intensity_loss_kernel(const float4* __restrict__ holo2,
                                                                      const float2* __restrict__ target2, int npairs,
                                                                      const float* __restrict__ target, int n,
                                                                      float* __restrict__ partials,
                                                                      unsigned* __restrict__ done, float* loss) {
  __shared__ float sh[kLossThreads / 32];
  __shared__ bool last;
  float acc = 0.f;
  for (int i = blockIdx.x * kLossThreads + threadIdx.x; i < npairs; i += gridDim.x * kLossThreads) {
    const float4 h = holo2[i];
    const float2 t = target2[i];
    const float r0 = (h.x * h.x + h.y * h.y) - t.x;
    const float r1 = (h.z * h.z + h.w * h.w) - t.y;
    acc = fmaf(r0, r0, acc);
    acc = fmaf(r1, r1, acc);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && (n & 1)) {  // odd tail element
    const float2 h = reinterpret_cast<const float2*>(holo2)[n - 1];
    const float r = (h.x * h.x + h.y * h.y) - target[n - 1];
    acc = fmaf(r, r, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kLossThreads / 32; ++w) s += sh[w];
    partials[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < 32) {
    // the last block: lane l sums partials l, l + 32, ... in order, then a fixed shuffle tree
    __threadfence();
    double total = 0.0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += 32) total += (double)((volatile float*)partials)[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (threadIdx.x == 0) {
      *loss = (float)(total / (double)n);
      *done = 0u;  // ready for the next launch (also inside a replayed graph)
    }
  }
}

__global__ void __launch_bounds__(kLossThreads) intensity_loss_backward_kernel(const float2* __restrict__ holo,
                                                                               const float* __restrict__ target, int n,
                                                                               const float* __restrict__ grad_loss,
                                                                               float2* __restrict__ grad_holo) {
  const int i = blockIdx.x * kLossThreads + threadIdx.x;
  if (i >= n) return;
  const float g = *grad_loss / (float)n;
  const float2 h = holo[i];
  const float r = (h.x * h.x + h.y * h.y) - target[i];
  const float s = (g * 2.0f * r) * 2.0f;
  grad_holo[i] = make_float2(s * h.x, s * h.y);
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_intensity_loss_workspace_bytes(int n) {
  (void)n;
  return (kLossMaxBlocks + 64) * sizeof(float);
}

extern "C" int cvhrf_intensity_loss_init_workspace(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < cvhrf_intensity_loss_workspace_bytes(0)) return CVHRF_EWORKSPACE;
  CVHRF_CUDA_TRY(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream));
  return CVHRF_OK;
}

extern "C" int cvhrf_intensity_loss(const void* holo, const float* target, int n, float* loss, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!holo || !target || !loss || n < 1) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_intensity_loss_workspace_bytes(n)) return CVHRF_EWORKSPACE;
  if (((uintptr_t)holo & 15) || ((uintptr_t)target & 7)) return CVHRF_EINVAL;
  unsigned* done = (unsigned*)workspace;
  float* partials = (float*)workspace + 64;
  const int npairs = n / 2;
  int blocks = (npairs + kLossThreads - 1) / kLossThreads;
  blocks = blocks < 1 ? 1 : (blocks > kLossMaxBlocks ? kLossMaxBlocks : blocks);
  intensity_loss_kernel<<<blocks, kLossThreads, 0, (cudaStream_t)stream>>>(
      (const float4*)holo, (const float2*)target, npairs, target, n, partials, done, loss);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_intensity_loss_backward(const void* holo, const float* target, int n, const float* grad_loss,
                                             void* grad_holo, void* stream) {
  if (!holo || !target || !grad_loss || !grad_holo || n < 1) return CVHRF_EINVAL;
  intensity_loss_backward_kernel<<<(n + kLossThreads - 1) / kLossThreads, kLossThreads, 0, (cudaStream_t)stream>>>(
      (const float2*)holo, target, n, grad_loss, (float2*)grad_holo);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
