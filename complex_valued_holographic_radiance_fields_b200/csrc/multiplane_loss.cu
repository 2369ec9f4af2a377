// Multiplane reconstruction loss, fused (train.py:293-304 with multiplane_loss_odak.__call__,
// utils/propagator.py:138-169, over every plane).
//
// Input: the K x C reconstructed plane fields f (complex64, S x S each, the output of the
// SLM -> plane propagation).  Per plane p, channel c and pixel (y, x) of the centred H x W
// crop (odak crop_center: rows S/2 - H/2 ...):
//   I = s_c |f|^2                 (s_c = sum over frames of the channel's laser power^2:
//                                  the frame loop of utils/propagator.py:612-634 summed by
//                                  train.py:293)
//   x = clamp(I, 0, 1)            (train.py:298)
//   loss += w0 (x - t)^2 + w1 (x m - t m)^2 + w2 (x t - t t)^2      (t target, m mask)
// and loss /= C H W: the sum over planes of the three torch MSE means of __call__.
// x is also written out (the clamped prediction the SSIM term reads).
//
// Forward: one launch; grid-stride partial sums, the last block to finish sums the block
// partials in a fixed order (deterministic).  Backward: one launch over the full S x S
// planes (zero outside the crop):
//   dL/dx = g (2 / n) (w0 (x - t) + w1 m (x m - t m) + w2 t (x t - t t)) + dpred
//   dL/dI = dL/dx where 0 <= I <= 1 (torch.clamp's gradient), else 0
//   dL/df = 2 s_c dL/dI f          (torch's convention for complex inputs)
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxBlocks = 148 * 4;
constexpr int kMaxChannels = 8;

struct LossGeom {
  int K, C, S, H, W, oy, ox;
  long long n;  // K C H W
  float w0, w1, w2;
  float scale[kMaxChannels];
};

__device__ __forceinline__ float term(float x, float t, float m, const LossGeom& g) {
  const float a = x - t;
  const float b = x * m - t * m;
  const float c = x * t - t * t;
  return g.w0 * (a * a) + g.w1 * (b * b) + g.w2 * (c * c);
}

__global__ void __launch_bounds__(kThreads) multiplane_loss_kernel(const float2* __restrict__ fields,
                                                                   const float* __restrict__ targets,
                                                                   const float* __restrict__ masks, LossGeom g,
                                                                   float* __restrict__ pred,
                                                                   float* __restrict__ partials,
                                                                   unsigned* __restrict__ done, float* loss) {
  __shared__ float sh[kThreads / 32];
  __shared__ bool last;
  float acc = 0.f;
  const long long HW = (long long)g.H * g.W;
  for (long long i = (long long)blockIdx.x * kThreads + threadIdx.x; i < g.n; i += (long long)gridDim.x * kThreads) {
    const long long pc = i / HW;
    const int r = (int)(i - pc * HW);
    const int y = r / g.W, x = r - y * g.W;
    const int c = (int)(pc % g.C);
    const float2 f = fields[(size_t)pc * g.S * g.S + (size_t)(y + g.oy) * g.S + (x + g.ox)];
    const float I = g.scale[c] * (f.x * f.x + f.y * f.y);
    const float v = fminf(fmaxf(I, 0.0f), 1.0f);
    pred[i] = v;
    acc += term(v, targets[i], masks[i], g);
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
    double total = 0.0;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += 32) total += (double)((volatile float*)partials)[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (threadIdx.x == 0) {
      *loss = (float)(total / (double)((long long)g.C * HW));
      *done = 0u;  // ready for the next launch (also inside a replayed graph)
    }
  }
}

__global__ void __launch_bounds__(kThreads) multiplane_loss_backward_kernel(
    const float2* __restrict__ fields, const float* __restrict__ targets, const float* __restrict__ masks, LossGeom g,
    const float* __restrict__ grad_loss, const float* __restrict__ grad_pred, float2* __restrict__ grad_fields) {
  const long long SS = (long long)g.S * g.S;
  const long long total = (long long)g.K * g.C * SS;
  const long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i >= total) return;
  const long long pc = i / SS;
  const int r = (int)(i - pc * SS);
  const int yy = r / g.S, xx = r - yy * g.S;
  const int y = yy - g.oy, x = xx - g.ox;
  float2 out = make_float2(0.0f, 0.0f);
  if (y >= 0 && y < g.H && x >= 0 && x < g.W) {
    const int c = (int)(pc % g.C);
    const float2 f = fields[i];
    const float s = g.scale[c];
    const float I = s * (f.x * f.x + f.y * f.y);
    if (I >= 0.0f && I <= 1.0f) {
      const long long j = pc * g.H * g.W + (long long)y * g.W + x;
      const float t = targets[j], m = masks[j];
      const float v = I;
      const float k = *grad_loss * (2.0f / (float)((long long)g.C * g.H * g.W));
      float d = k * (g.w0 * (v - t) + g.w1 * m * (v * m - t * m) + g.w2 * t * (v * t - t * t));
      if (grad_pred) d += grad_pred[j];
      const float q = 2.0f * s * d;
      out = make_float2(q * f.x, q * f.y);
    }
  }
  grad_fields[i] = out;
}

bool make_geom(int K, int C, int S, int H, int W, const float* channel_scale, const float* weights, LossGeom& g) {
  if (K < 1 || C < 1 || C > kMaxChannels || S < 1 || H < 1 || W < 1 || H > S || W > S || !weights) return false;
  g.K = K; g.C = C; g.S = S; g.H = H; g.W = W;
  g.oy = S / 2 - H / 2;
  g.ox = S / 2 - W / 2;
  if (g.oy + H > S || g.ox + W > S) return false;
  g.n = (long long)K * C * H * W;
  g.w0 = weights[0]; g.w1 = weights[1]; g.w2 = weights[2];
  for (int c = 0; c < kMaxChannels; ++c) g.scale[c] = (c < C) ? (channel_scale ? channel_scale[c] : 1.0f) : 0.0f;
  return true;
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_multiplane_loss_workspace_bytes(void) { return (kMaxBlocks + 64) * sizeof(float); }

extern "C" int cvhrf_multiplane_loss_init_workspace(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < cvhrf_multiplane_loss_workspace_bytes()) return CVHRF_EWORKSPACE;
  CVHRF_CUDA_TRY(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream));
  return CVHRF_OK;
}

extern "C" int cvhrf_multiplane_loss(const void* fields, int K, int C, int S, int H, int W,
                                     const float* channel_scale, const float* targets, const float* masks,
                                     const float* weights, float* pred, float* loss, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  LossGeom g;
  if (!fields || !targets || !masks || !pred || !loss || !make_geom(K, C, S, H, W, channel_scale, weights, g))
    return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_multiplane_loss_workspace_bytes()) return CVHRF_EWORKSPACE;
  unsigned* done = (unsigned*)workspace;
  float* partials = (float*)workspace + 64;
  long long blocks = (g.n + kThreads - 1) / kThreads;
  blocks = blocks > kMaxBlocks ? kMaxBlocks : blocks;
  multiplane_loss_kernel<<<(unsigned)blocks, kThreads, 0, (cudaStream_t)stream>>>(
      (const float2*)fields, targets, masks, g, pred, partials, done, loss);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_multiplane_loss_backward(const void* fields, int K, int C, int S, int H, int W,
                                              const float* channel_scale, const float* targets, const float* masks,
                                              const float* weights, const float* grad_loss, const float* grad_pred,
                                              void* grad_fields, void* stream) {
  LossGeom g;
  if (!fields || !targets || !masks || !grad_loss || !grad_fields ||
      !make_geom(K, C, S, H, W, channel_scale, weights, g))
    return CVHRF_EINVAL;
  const long long total = (long long)K * C * S * S;
  multiplane_loss_backward_kernel<<<(unsigned)((total + kThreads - 1) / kThreads), kThreads, 0,
                                    (cudaStream_t)stream>>>((const float2*)fields, targets, masks, g, grad_loss,
                                                            grad_pred, (float2*)grad_fields);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
