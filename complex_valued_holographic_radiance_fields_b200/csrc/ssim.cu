// Fused SSIM (replaces the reference's fusedssim / fusedssim_backward, conv.cu:935-1195,
// behind FusedSSIMMap / fast_ssim, cov3d_cuda/python_import.py:43-57, 449-454).
//
// SSIM per pixel and channel with an 11 x 11 Gaussian window (sigma 1.5) and zero
// padding outside the image:
//   mu1 = w * x, mu2 = w * y, s11 = w * x^2 - mu1^2, s22 = w * y^2 - mu2^2, s12 = w * xy - mu1 mu2
//   m = (2 mu1 mu2 + C1)(2 s12 + C2) / ((mu1^2 + mu2^2 + C1)(s11 + s22 + C2))
// The window is separable, so each 32 x 32 output tile does an 11-tap horizontal pass
// over its 42 staged rows and an 11-tap vertical pass (22 taps per quantity instead of
// the reference's 121).  The forward also stores, per pixel, the partial derivatives
// with respect to (mu1, s11, s12) in the form the backward needs:
//   P = dm/dmu1 - 2 mu1 dm/ds11 - mu2 dm/ds12,   Q = dm/ds11,   R = dm/ds12
// so that for an upstream gradient g (per pixel):
//   dL/dx = w * (g P) + 2 x (w * (g Q)) + y (w * (g R))        (w symmetric: w^T = w)
// and the backward is three separable convolutions.  The mean of the map (fast_ssim) is
// reduced in the same launch (deterministic two-level sum).
#include <math.h>
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kSsimTile = 32, kSsimHalo = 5, kSsimRows = kSsimTile + 2 * kSsimHalo;  // 42
constexpr int kSsimThreads = 256;
constexpr int kSsimMaxBlocks = 65535;

struct SsimWeights {
  float w[11];
};

__device__ __forceinline__ float pix(const float* img, int y, int x, int H, int W) {
  return (x >= 0 && x < W && y >= 0 && y < H) ? img[(size_t)y * W + x] : 0.0f;
}

// grid: (tiles x, tiles y, channels).  map may be null; partials: one float per block.
__global__ void __launch_bounds__(kSsimThreads) ssim_forward_kernel(const float* __restrict__ img1,
                                                                    const float* __restrict__ img2, int H, int W,
                                                                    float C1, float C2, SsimWeights wt,
                                                                    float* __restrict__ map, float* __restrict__ dP,
                                                                    float* __restrict__ dQ, float* __restrict__ dR,
                                                                    float* __restrict__ partials) {
  __shared__ float sx[kSsimRows][kSsimRows + 1], sy[kSsimRows][kSsimRows + 1];
  __shared__ float hq[5][kSsimRows][kSsimTile + 1];   // horizontal pass: x, y, xx, yy, xy
  __shared__ float red[kSsimThreads / 32];
  const int c = blockIdx.z;
  const size_t plane = (size_t)c * H * W;
  const float* a = img1 + plane;
  const float* b = img2 + plane;
  const int x0 = blockIdx.x * kSsimTile - kSsimHalo, y0 = blockIdx.y * kSsimTile - kSsimHalo;
  for (int e = threadIdx.x; e < kSsimRows * kSsimRows; e += kSsimThreads) {
    const int r = e / kSsimRows, q = e - r * kSsimRows;
    sx[r][q] = pix(a, y0 + r, x0 + q, H, W);
    sy[r][q] = pix(b, y0 + r, x0 + q, H, W);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kSsimRows * kSsimTile; e += kSsimThreads) {
    const int r = e / kSsimTile, q = e - r * kSsimTile;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f, s4 = 0.f;
#pragma unroll
    for (int k = 0; k < 11; ++k) {
      const float u = sx[r][q + k], v = sy[r][q + k], wk = wt.w[k];
      s0 = fmaf(wk, u, s0);
      s1 = fmaf(wk, v, s1);
      s2 = fmaf(wk, u * u, s2);
      s3 = fmaf(wk, v * v, s3);
      s4 = fmaf(wk, u * v, s4);
    }
    hq[0][r][q] = s0;
    hq[1][r][q] = s1;
    hq[2][r][q] = s2;
    hq[3][r][q] = s3;
    hq[4][r][q] = s4;
  }
  __syncthreads();
  float acc = 0.f;
  for (int e = threadIdx.x; e < kSsimTile * kSsimTile; e += kSsimThreads) {
    const int r = e / kSsimTile, q = e - r * kSsimTile;
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f, m4 = 0.f;
#pragma unroll
    for (int k = 0; k < 11; ++k) {
      const float wk = wt.w[k];
      m0 = fmaf(wk, hq[0][r + k][q], m0);
      m1 = fmaf(wk, hq[1][r + k][q], m1);
      m2 = fmaf(wk, hq[2][r + k][q], m2);
      m3 = fmaf(wk, hq[3][r + k][q], m3);
      m4 = fmaf(wk, hq[4][r + k][q], m4);
    }
    const int y = blockIdx.y * kSsimTile + r, x = blockIdx.x * kSsimTile + q;
    if (y >= H || x >= W) continue;
    const float mu1 = m0, mu2 = m1;
    const float s11 = m2 - mu1 * mu1, s22 = m3 - mu2 * mu2, s12 = m4 - mu1 * mu2;
    const float Cn = 2.0f * mu1 * mu2 + C1, Dn = 2.0f * s12 + C2;
    const float An = mu1 * mu1 + mu2 * mu2 + C1, Bn = s11 + s22 + C2;
    const float m = (Cn * Dn) / (An * Bn);
    const float dmu1 = (2.0f * mu2 * Dn) / (An * Bn) - (2.0f * mu1 * Cn * Dn) / (An * An * Bn);
    const float q11 = -(Cn * Dn) / (An * Bn * Bn);
    const float r12 = (2.0f * Cn) / (An * Bn);
    const size_t o = plane + (size_t)y * W + x;
    if (map) map[o] = m;
    dP[o] = dmu1 - 2.0f * mu1 * q11 - mu2 * r12;
    dQ[o] = q11;
    dR[o] = r12;
    acc += m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < kSsimThreads / 32; ++w) s += red[w];
    partials[((size_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x] = s;
  }
}

// mean of the map from the per-block partials (one block, fixed order)
__global__ void __launch_bounds__(1024) ssim_mean_kernel(const float* __restrict__ partials, int nparts, double inv_n,
                                                        float* __restrict__ out) {
  __shared__ double sh[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) acc += (double)partials[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < (int)(blockDim.x + 31) / 32; ++w) s += sh[w];
    *out = (float)(s * inv_n);
  }
}

// grad_img1 = w*(gP) + 2 x w*(gQ) + y w*(gR); g = dL_dmap[pixel] if dL_dmap, else *g_scalar * scale
__global__ void __launch_bounds__(kSsimThreads) ssim_backward_kernel(
    const float* __restrict__ img1, const float* __restrict__ img2, int H, int W, SsimWeights wt,
    const float* __restrict__ dP, const float* __restrict__ dQ, const float* __restrict__ dR,
    const float* __restrict__ dL_dmap, const float* __restrict__ g_scalar, float scale, float* __restrict__ grad) {
  __shared__ float sp[3][kSsimRows][kSsimRows + 1];
  __shared__ float hq[3][kSsimRows][kSsimTile + 1];
  const int c = blockIdx.z;
  const size_t plane = (size_t)c * H * W;
  const int x0 = blockIdx.x * kSsimTile - kSsimHalo, y0 = blockIdx.y * kSsimTile - kSsimHalo;
  const float gs = dL_dmap ? 1.0f : *g_scalar * scale;
  for (int e = threadIdx.x; e < kSsimRows * kSsimRows; e += kSsimThreads) {
    const int r = e / kSsimRows, q = e - r * kSsimRows;
    const int y = y0 + r, x = x0 + q;
    float p = 0.f, qq = 0.f, rr = 0.f;
    if (x >= 0 && x < W && y >= 0 && y < H) {
      const size_t o = plane + (size_t)y * W + x;
      const float g = dL_dmap ? dL_dmap[o] : 1.0f;
      p = g * dP[o];
      qq = g * dQ[o];
      rr = g * dR[o];
    }
    sp[0][r][q] = p;
    sp[1][r][q] = qq;
    sp[2][r][q] = rr;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kSsimRows * kSsimTile; e += kSsimThreads) {
    const int r = e / kSsimTile, q = e - r * kSsimTile;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < 11; ++k) {
      const float wk = wt.w[k];
      s0 = fmaf(wk, sp[0][r][q + k], s0);
      s1 = fmaf(wk, sp[1][r][q + k], s1);
      s2 = fmaf(wk, sp[2][r][q + k], s2);
    }
    hq[0][r][q] = s0;
    hq[1][r][q] = s1;
    hq[2][r][q] = s2;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kSsimTile * kSsimTile; e += kSsimThreads) {
    const int r = e / kSsimTile, q = e - r * kSsimTile;
    const int y = blockIdx.y * kSsimTile + r, x = blockIdx.x * kSsimTile + q;
    if (y >= H || x >= W) continue;
    float c0 = 0.f, c1 = 0.f, c2 = 0.f;
#pragma unroll
    for (int k = 0; k < 11; ++k) {
      const float wk = wt.w[k];
      c0 = fmaf(wk, hq[0][r + k][q], c0);
      c1 = fmaf(wk, hq[1][r + k][q], c1);
      c2 = fmaf(wk, hq[2][r + k][q], c2);
    }
    const size_t o = plane + (size_t)y * W + x;
    grad[o] = gs * (c0 + 2.0f * img1[o] * c1 + img2[o] * c2);
  }
}

SsimWeights gaussian_weights() {
  SsimWeights w;
  double g[11], s = 0.0;
  for (int i = 0; i < 11; ++i) {
    g[i] = exp(-((i - 5) * (i - 5)) / (2.0 * 1.5 * 1.5));
    s += g[i];
  }
  for (int i = 0; i < 11; ++i) w.w[i] = (float)(g[i] / s);
  return w;
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_ssim_workspace_bytes(int C, int H, int W) {
  if (C < 1 || H < 1 || W < 1) return 0;
  const size_t n = (size_t)C * H * W;
  const size_t blocks = (size_t)C * ((H + kSsimTile - 1) / kSsimTile) * ((W + kSsimTile - 1) / kSsimTile);
  return align_up(3 * n * sizeof(float), 256) + align_up(blocks * sizeof(float), 256);
}

extern "C" int cvhrf_ssim_forward(const float* img1, const float* img2, int C, int H, int W, float C1, float C2,
                                  float* map, float* mean, void* workspace, size_t workspace_bytes, void* stream) {
  if (!img1 || !img2 || C < 1 || H < 1 || W < 1 || (!map && !mean)) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_ssim_workspace_bytes(C, H, W)) return CVHRF_EWORKSPACE;
  const size_t n = (size_t)C * H * W;
  float* dP = (float*)workspace;
  float* dQ = dP + n;
  float* dR = dQ + n;
  float* partials = (float*)((char*)workspace + align_up(3 * n * sizeof(float), 256));
  dim3 grid((W + kSsimTile - 1) / kSsimTile, (H + kSsimTile - 1) / kSsimTile, C);
  if (grid.y > kSsimMaxBlocks || grid.z > kSsimMaxBlocks) return CVHRF_EUNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  ssim_forward_kernel<<<grid, kSsimThreads, 0, st>>>(img1, img2, H, W, C1, C2, gaussian_weights(), map, dP, dQ, dR,
                                                     partials);
  CVHRF_LAUNCH_CHECK();
  if (mean) {
    ssim_mean_kernel<<<1, 1024, 0, st>>>(partials, (int)(grid.x * grid.y * grid.z), 1.0 / (double)n, mean);
    CVHRF_LAUNCH_CHECK();
  }
  return CVHRF_OK;
}

extern "C" int cvhrf_ssim_backward(const float* img1, const float* img2, int C, int H, int W,
                                   const float* dL_dmap, const float* dL_dmean, float* grad_img1,
                                   const void* workspace, size_t workspace_bytes, void* stream) {
  if (!img1 || !img2 || !grad_img1 || C < 1 || H < 1 || W < 1 || (!dL_dmap == !dL_dmean)) return CVHRF_EINVAL;
  if (!workspace || workspace_bytes < cvhrf_ssim_workspace_bytes(C, H, W)) return CVHRF_EWORKSPACE;
  const size_t n = (size_t)C * H * W;
  const float* dP = (const float*)workspace;
  dim3 grid((W + kSsimTile - 1) / kSsimTile, (H + kSsimTile - 1) / kSsimTile, C);
  ssim_backward_kernel<<<grid, kSsimThreads, 0, (cudaStream_t)stream>>>(
      img1, img2, H, W, gaussian_weights(), dP, dP + n, dP + 2 * n, dL_dmap, dL_dmean, (float)(1.0 / (double)n),
      grad_img1);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
