// Fused Adan (replaces utils/optimizer.py:288-484 Adan.step with _multi_tensor_adan
// :545-611 / _single_tensor_adan :487-542: about 17 torch foreach launches per group, the
// optimizer the reference's training script actually builds, optimizer.py:65).
//
// One launch updates every element of every group, in the reference's operation order
// and with the scalars torch receives (each formed in double on the host, then float):
//   g = clip * grad (written back, as grad.mul_ does)
//   d = neg_pre_grad + g              (0 on a group's first step: neg_pre_grad = -clip * grad)
//   m = m b1 + (1 - b1) g;  diff = diff b2 + (1 - b2) d;  d = d b2 + g;  v = v b3 + (1 - b3) d d
//   denom = sqrt(v) / sqrt(bc3) + eps
//   no_prox: p = p (1 - lr wd); p += (-s) m / denom; p += (-s_diff) diff / denom
//   else   : p += (-s) m / denom; p += (-s_diff) diff / denom; p = p / (1 + lr wd)
//   neg_pre_grad = -g                 (s = lr / bc1, s_diff = lr b2 / bc2)
// The optional global-norm clip factor min(max_norm / (||grad|| + eps), 1) is computed on
// the device by a deterministic two-level reduction (the reference reads it back to the host).
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kAdanMaxGroups = 16;
constexpr int kAdanThreads = 256;
constexpr int kAdanNormBlocks = 148 * 2;  // per group

struct AdanLaunch {
  int n;
  cvhrf_adan_group g[kAdanMaxGroups];
};

__global__ void __launch_bounds__(kAdanThreads) adan_kernel(AdanLaunch L, const float* __restrict__ clip_dev) {
  const cvhrf_adan_group& G = L.g[blockIdx.y];
  const float clip = clip_dev ? *clip_dev : 1.0f;
  const float b1 = G.beta1, b2 = G.beta2, b3 = G.beta3;
  for (long long i = (long long)blockIdx.x * kAdanThreads + threadIdx.x; i < G.n;
       i += (long long)gridDim.x * kAdanThreads) {
    const float g = G.grad[i] * clip;
    G.grad[i] = g;
    float d = G.first_step ? 0.0f : G.neg_pre_grad[i] + g;
    const float m = G.exp_avg[i] * b1 + G.one_minus_beta1 * g;
    const float diff = G.exp_avg_diff[i] * b2 + G.one_minus_beta2 * d;
    d = d * b2 + g;
    const float v = G.exp_avg_sq[i] * b3 + G.one_minus_beta3 * d * d;
    const float denom = sqrtf(v) / G.bias_correction3_sqrt + G.eps;
    float p = G.param[i];
    if (G.no_prox) {
      p = p * G.decay;
      p = p + (-G.step_size) * m / denom;
      p = p + (-G.step_size_diff) * diff / denom;
    } else {
      p = p + (-G.step_size) * m / denom;
      p = p + (-G.step_size_diff) * diff / denom;
      p = p / G.decay;
    }
    G.param[i] = p;
    G.exp_avg[i] = m;
    G.exp_avg_diff[i] = diff;
    G.exp_avg_sq[i] = v;
    G.neg_pre_grad[i] = -g;
  }
}

// partial sums of grad^2: partials[group * kAdanNormBlocks + block]; the last block to
// finish combines them in a fixed order and writes the clip factor
__global__ void __launch_bounds__(kAdanThreads) adan_clip_kernel(AdanLaunch L, float max_norm, float eps,
                                                                 double* __restrict__ partials,
                                                                 unsigned* __restrict__ done, float* clip_out) {
  __shared__ double sh[kAdanThreads / 32];
  __shared__ bool last;
  const cvhrf_adan_group& G = L.g[blockIdx.y];
  double acc = 0.0;
  for (long long i = (long long)blockIdx.x * kAdanThreads + threadIdx.x; i < G.n;
       i += (long long)gridDim.x * kAdanThreads) {
    const float g = G.grad[i];
    acc += (double)(g * g);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kAdanThreads / 32; ++w) s += sh[w];
    partials[blockIdx.y * gridDim.x + blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(done, 1u) == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    double total = 0.0;
    for (unsigned b = 0; b < gridDim.x * gridDim.y; ++b) total += ((volatile double*)partials)[b];
    const float norm = sqrtf((float)total);
    *clip_out = fminf(max_norm / (norm + eps), 1.0f);
    *done = 0u;
  }
}

bool fill(const cvhrf_adan_group* groups, int ngroups, AdanLaunch& L, long long& most) {
  if (!groups || ngroups < 0 || ngroups > kAdanMaxGroups) return false;
  L.n = 0;
  most = 0;
  for (int i = 0; i < ngroups; ++i) {
    const cvhrf_adan_group& g = groups[i];
    if (g.n < 0 || (g.n > 0 && (!g.param || !g.grad || !g.exp_avg || !g.exp_avg_sq || !g.exp_avg_diff ||
                                !g.neg_pre_grad)))
      return false;
    if (g.n == 0) continue;
    L.g[L.n++] = g;
    most = g.n > most ? g.n : most;
  }
  return true;
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" int cvhrf_adan(const cvhrf_adan_group* groups, int ngroups, const float* clip, void* stream) {
  AdanLaunch L{};
  long long most;
  if (!fill(groups, ngroups, L, most)) return CVHRF_EINVAL;
  if (L.n == 0) return CVHRF_OK;
  const long long bx = (most + kAdanThreads - 1) / kAdanThreads;
  dim3 grid((unsigned)(bx < 148 * 4 ? bx : 148 * 4), L.n);
  adan_kernel<<<grid, kAdanThreads, 0, (cudaStream_t)stream>>>(L, clip);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" size_t cvhrf_adan_clip_workspace_bytes(void) {
  return 256 + (size_t)kAdanMaxGroups * kAdanNormBlocks * sizeof(double);
}

extern "C" int cvhrf_adan_clip_init_workspace(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < cvhrf_adan_clip_workspace_bytes()) return CVHRF_EWORKSPACE;
  CVHRF_CUDA_TRY(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream));
  return CVHRF_OK;
}

extern "C" int cvhrf_adan_clip_factor(const cvhrf_adan_group* groups, int ngroups, float max_grad_norm, float eps,
                                      float* clip_out, void* workspace, size_t workspace_bytes, void* stream) {
  AdanLaunch L{};
  long long most;
  if (!fill(groups, ngroups, L, most) || !clip_out || !(max_grad_norm > 0.0f)) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_adan_clip_workspace_bytes()) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  if (L.n == 0) {
    const float one = 1.0f;
    CVHRF_CUDA_TRY(cudaMemcpyAsync(clip_out, &one, sizeof(float), cudaMemcpyHostToDevice, st));
    CVHRF_CUDA_TRY(cudaStreamSynchronize(st));  // the host source must outlive the copy
    return CVHRF_OK;
  }
  unsigned* done = (unsigned*)workspace;
  double* partials = (double*)((char*)workspace + 256);
  dim3 grid(kAdanNormBlocks, L.n);
  adan_clip_kernel<<<grid, kAdanThreads, 0, st>>>(L, max_grad_norm, eps, partials, done, clip_out);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
