// The hologram -> SLM-field step of the training loss (train.py:280-283 with
// utils/propagator.py:612-620), fused:
//   phi = angle(h) mod 2 pi,  m = mean(phi) over all C x n values,  a = |h|
//   f[c] = a exp(i (phi - m) s_c)                  (s_c the propagator's phase scale)
// which torch runs as about fifteen elementwise and reduction launches forward and
// backward.  Forward: one reduction launch (deterministic: block partials summed in a
// fixed order by the last block) for m, one elementwise launch for f.  Backward, with G
// the incoming gradient (torch's convention for complex tensors, dL/dRe + i dL/dIm):
//   dtheta = Re(G) (-a sin t) + Im(G) (a cos t),  da = Re(G) cos t + Im(G) sin t
//   dphi = s_c dtheta - (1 / (C n)) sum_k s_k dtheta_k       (the mean couples all values)
//   dh = da h / a + dphi (-Im h + i Re h) / a^2               (zero where h = 0)
// one reduction launch for the sum and one elementwise launch.
#include <math.h>
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 148 * 4;
constexpr int kMaxChannels = 8;
constexpr float kTwoPi = 6.283185307179586f;

struct FieldArgs {
  int C;
  long long n;  // values per channel
  float scale[kMaxChannels];
};

__device__ __forceinline__ float wrapped_phase(float2 h) {
  const float p = atan2f(h.y, h.x);
  return p < 0.0f ? p + kTwoPi : p;  // torch.remainder(p, 2 pi) for p in [-pi, pi]
}

// mode 0: sum of wrapped phases; mode 1: sum of s_c dtheta (needs g, mean).
template <int MODE>
__global__ void __launch_bounds__(kThreads) field_reduce_kernel(const float2* __restrict__ holo,
                                                                const float2* __restrict__ g,
                                                                const float* __restrict__ mean, FieldArgs a,
                                                                float* __restrict__ partials,
                                                                unsigned* __restrict__ done, float* out) {
  __shared__ float sh[kThreads / 32];
  __shared__ bool last;
  const long long total = (long long)a.C * a.n;
  float acc = 0.f;
  const float m = MODE == 1 ? *mean : 0.0f;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < total; i += (long long)gridDim.x * kThreads) {
    const float2 h = holo[i];
    const float phi = wrapped_phase(h);
    if (MODE == 0) {
      acc += phi;
    } else {
      const float s = a.scale[(int)(i / a.n)];
      const float t = (phi - m) * s;
      float sn, cs;
      sincosf(t, &sn, &cs);
      const float amp = hypotf(h.x, h.y);
      const float2 gg = g[i];
      acc += s * (gg.x * (-amp * sn) + gg.y * (amp * cs));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) s += sh[w];
    partials[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x < 32) {
    __threadfence();
    double tot = 0.0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += 32) tot += (double)((volatile float*)partials)[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (threadIdx.x == 0) {
      *out = MODE == 0 ? (float)(tot / (double)total) : (float)tot;
      *done = 0u;  // ready for the next launch (also inside a replayed graph)
    }
  }
}

__global__ void __launch_bounds__(kThreads) field_forward_kernel(const float2* __restrict__ holo,
                                                                 const float* __restrict__ mean, FieldArgs a,
                                                                 float2* __restrict__ field) {
  const long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i >= (long long)a.C * a.n) return;
  const float2 h = holo[i];
  const float t = (wrapped_phase(h) - *mean) * a.scale[(int)(i / a.n)];
  float sn, cs;
  sincosf(t, &sn, &cs);
  const float amp = hypotf(h.x, h.y);
  field[i] = make_float2(amp * cs, amp * sn);
}

__global__ void __launch_bounds__(kThreads) field_backward_kernel(const float2* __restrict__ holo,
                                                                  const float2* __restrict__ g,
                                                                  const float* __restrict__ mean,
                                                                  const float* __restrict__ tsum, FieldArgs a,
                                                                  float2* __restrict__ grad) {
  const long long total = (long long)a.C * a.n;
  const long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i >= total) return;
  const float2 h = holo[i];
  const float s = a.scale[(int)(i / a.n)];
  const float t = (wrapped_phase(h) - *mean) * s;
  float sn, cs;
  sincosf(t, &sn, &cs);
  const float amp = hypotf(h.x, h.y);
  const float2 gg = g[i];
  if (amp == 0.0f) {
    grad[i] = make_float2(0.0f, 0.0f);
    return;
  }
  const float dtheta = gg.x * (-amp * sn) + gg.y * (amp * cs);
  const float da = gg.x * cs + gg.y * sn;
  const float dphi = s * dtheta - *tsum / (float)total;
  const float inv = 1.0f / amp;
  const float inv2 = inv * inv;
  grad[i] = make_float2(da * h.x * inv - dphi * h.y * inv2, da * h.y * inv + dphi * h.x * inv2);
}

bool make_args(int C, long long n, const float* phase_scale, FieldArgs& a) {
  if (C < 1 || C > kMaxChannels || n < 1) return false;
  a.C = C;
  a.n = n;
  for (int c = 0; c < kMaxChannels; ++c) a.scale[c] = c < C ? (phase_scale ? phase_scale[c] : 1.0f) : 0.0f;
  return true;
}

int grid_for(long long total) {
  long long b = (total + kThreads - 1) / kThreads;
  return (int)(b > kMaxBlocks ? kMaxBlocks : b);
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_hologram_field_workspace_bytes(void) { return (kMaxBlocks + 64) * sizeof(float); }

extern "C" int cvhrf_hologram_field_init_workspace(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < cvhrf_hologram_field_workspace_bytes()) return CVHRF_EWORKSPACE;
  CVHRF_CUDA_TRY(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream));
  return CVHRF_OK;
}

extern "C" int cvhrf_hologram_field(const void* holo, int C, long long n, const float* phase_scale, void* field,
                                    float* mean, void* workspace, size_t workspace_bytes, void* stream) {
  FieldArgs a;
  if (!holo || !field || !mean || !make_args(C, n, phase_scale, a)) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_hologram_field_workspace_bytes()) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const long long total = (long long)C * n;
  field_reduce_kernel<0><<<grid_for(total), kThreads, 0, st>>>((const float2*)holo, nullptr, nullptr, a,
                                                               (float*)workspace + 64, (unsigned*)workspace, mean);
  CVHRF_LAUNCH_CHECK();
  field_forward_kernel<<<(unsigned)((total + kThreads - 1) / kThreads), kThreads, 0, st>>>((const float2*)holo, mean,
                                                                                            a, (float2*)field);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_hologram_field_backward(const void* holo, int C, long long n, const float* phase_scale,
                                             const float* mean, const void* grad_field, void* grad_holo,
                                             void* workspace, size_t workspace_bytes, void* stream) {
  FieldArgs a;
  if (!holo || !mean || !grad_field || !grad_holo || !make_args(C, n, phase_scale, a)) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_hologram_field_workspace_bytes()) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const long long total = (long long)C * n;
  float* tsum = (float*)workspace + 32;
  field_reduce_kernel<1><<<grid_for(total), kThreads, 0, st>>>((const float2*)holo, (const float2*)grad_field, mean,
                                                               a, (float*)workspace + 64, (unsigned*)workspace, tsum);
  CVHRF_LAUNCH_CHECK();
  field_backward_kernel<<<(unsigned)((total + kThreads - 1) / kThreads), kThreads, 0, st>>>(
      (const float2*)holo, (const float2*)grad_field, mean, tsum, a, (float2*)grad_holo);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
