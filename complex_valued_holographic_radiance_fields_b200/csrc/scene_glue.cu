// The caller's glue around the rasterizer, fused (replaces the torch
// ops of model.py:1365-1402 Scene.render and model.py:595-608 apply_activations):
//
//   forward : X_cam = X @ R + T; keep near < z < far; sort by depth; gather every
//             parameter in that order and activate it: scales = exp, quats = normalize
//             (eps 1e-12), phase = pre mod 2 pi (sign of the divisor), opacity =
//             sigmoid, plane probabilities = one-hot(argmax) (straight-through,
//             model.py:41-56).
//   backward: the matching chain rule scattered back to parameter rows: dX = dX_cam R^T,
//             dlog s = ds * s, normalize backward, mod passes through, sigmoid', and
//             the straight-through softmax(x / 0.001) * g (model.py:51-56).
//
// Plane ownership (cvhrf_scene_prepare_owned, for plane-parallel training): rows whose
// one-hot plane is not in the owned set are treated like rows outside (near, far): sorted
// last, and given depth z = near so that the rasterizer culls them.  With
// one-hot plane weights that is exact for the owned planes: such a row has weight 0 on
// every owned plane, so it neither renders there nor receives gradient there.
//
// Rows outside (near, far) are not dropped: they are sorted after every valid row (key
// 0xFFFFFFFF) and keep their out-of-range depth, so the rasterizer culls them (radius 0,
// no tiles, not visible) and their gradients come back as exact zeros.  This removes the
// host synchronisation torch.where(mask) needs to size the subset.
#include <math.h>
#include "scan_sort.cuh"

namespace cvhrf {
namespace {

__device__ __forceinline__ void cam_point(const float* X, const float* R, const float* T, float* c) {
#pragma unroll
  for (int j = 0; j < 3; ++j) c[j] = fmaf(X[2], R[6 + j], fmaf(X[1], R[3 + j], X[0] * R[j])) + T[j];
}

// ascending order of floats as unsigned keys
__device__ __forceinline__ uint32_t float_order_key(float z) {
  const uint32_t b = __float_as_uint(z);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// index of the largest plane logit, first one on ties (the one-hot of glue_gather_kernel)
__device__ __forceinline__ int argmax_plane(const float* logits, int K) {
  int best = 0;
  float bv = logits[0];
  for (int k = 1; k < K; ++k)
    if (logits[k] > bv) { bv = logits[k]; best = k; }
  return best;
}

__global__ void glue_keys_kernel(cvhrf_gaussians G, const float* __restrict__ R, const float* __restrict__ T,
                                 float near_plane, float far_plane, uint32_t owned_planes,
                                 uint32_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= G.N) return;
  float c[3];
  cam_point(G.means + 3 * r, R, T, c);
  bool valid = c[2] > near_plane && c[2] < far_plane;
  if (owned_planes != 0xFFFFFFFFu) valid = valid && ((owned_planes >> argmax_plane(G.pre_planes + r * G.K, G.K)) & 1u);
  uint32_t k = valid ? float_order_key(c[2]) : 0xFFFFFFFFu;
  if (valid && k == 0xFFFFFFFFu) k = 0xFFFFFFFEu;
  keys[r] = k;
  vals[r] = (uint32_t)r;
}

__global__ void glue_gather_kernel(cvhrf_gaussians G, const float* __restrict__ R, const float* __restrict__ T,
                                   const uint32_t* __restrict__ order, uint32_t owned_planes, float cull_z,
                                   float* cam, float* z, float* quats, float* scales, float* colours, float* phase,
                                   float* opac, float* planes) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= G.N) return;
  const int r = (int)order[s];
  float c[3];
  cam_point(G.means + 3 * r, R, T, c);
  const int best = argmax_plane(G.pre_planes + r * G.K, G.K);
  // a row of a plane this caller does not own is culled through its depth (z = near)
  if (owned_planes != 0xFFFFFFFFu && !((owned_planes >> best) & 1u)) c[2] = cull_z;
#pragma unroll
  for (int j = 0; j < 3; ++j) cam[3 * s + j] = c[j];
  z[s] = c[2];
  const float* q = G.pre_quats + 4 * r;
  const float nrm = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
#pragma unroll
  for (int j = 0; j < 4; ++j) quats[4 * s + j] = q[j] / nrm;
#pragma unroll
  for (int j = 0; j < 3; ++j) scales[3 * s + j] = expf(G.pre_scales[3 * r + j]);
  const float two_pi = (float)(2.0 * M_PI);
  for (int k = 0; k < G.C; ++k) {
    colours[s * G.C + k] = G.colours[r * G.C + k];
    float m = fmodf(G.pre_phase[r * G.C + k], two_pi);
    if (m != 0.0f && (m < 0.0f) != (two_pi < 0.0f)) m += two_pi;
    phase[s * G.C + k] = m;
  }
  opac[s] = 1.0f / (1.0f + expf(-G.pre_opac[r]));
  for (int k = 0; k < G.K; ++k) planes[s * G.K + k] = k == best ? 1.0f : 0.0f;
}

__global__ void glue_backward_kernel(cvhrf_gaussians G, const float* __restrict__ R,
                                     const uint32_t* __restrict__ order, const float* __restrict__ g_cam,
                                     const float* __restrict__ g_quats, const float* __restrict__ g_scales,
                                     const float* __restrict__ g_colours, const float* __restrict__ g_phase,
                                     const float* __restrict__ g_opac, const float* __restrict__ g_planes,
                                     float* d_means, float* d_quats, float* d_scales, float* d_colours,
                                     float* d_phase, float* d_opac, float* d_planes) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= G.N) return;
  const int r = (int)order[s];
  // X_cam = X R + T  ->  dX = dX_cam R^T
#pragma unroll
  for (int i = 0; i < 3; ++i)
    d_means[3 * r + i] = g_cam[3 * s] * R[3 * i] + g_cam[3 * s + 1] * R[3 * i + 1] + g_cam[3 * s + 2] * R[3 * i + 2];
  // normalize: q_hat = q / max(|q|, eps); dq = (g - q_hat (q_hat . g)) / |q|
  const float* q = G.pre_quats + 4 * r;
  const float nrm = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1e-12f);
  float qh[4], gq[4], dot = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qh[j] = q[j] / nrm;
    gq[j] = g_quats[4 * s + j];
    dot += qh[j] * gq[j];
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) d_quats[4 * r + j] = (gq[j] - qh[j] * dot) / nrm;
#pragma unroll
  for (int j = 0; j < 3; ++j) d_scales[3 * r + j] = g_scales[3 * s + j] * expf(G.pre_scales[3 * r + j]);
  for (int k = 0; k < G.C; ++k) {
    d_colours[r * G.C + k] = g_colours[s * G.C + k];
    d_phase[r * G.C + k] = g_phase[s * G.C + k];
  }
  const float sg = 1.0f / (1.0f + expf(-G.pre_opac[r]));
  d_opac[r] = g_opac[s] * sg * (1.0f - sg);
  // straight-through estimator: softmax(x / 0.001) * g
  float mx = -INFINITY;
  for (int k = 0; k < G.K; ++k) mx = fmaxf(mx, G.pre_planes[r * G.K + k] / 0.001f);
  float den = 0.f;
  for (int k = 0; k < G.K; ++k) den += expf(G.pre_planes[r * G.K + k] / 0.001f - mx);
  for (int k = 0; k < G.K; ++k)
    d_planes[r * G.K + k] = g_planes[s * G.K + k] * (expf(G.pre_planes[r * G.K + k] / 0.001f - mx) / den);
}

bool gaussians_ok(const cvhrf_gaussians* G) {
  return G && G->N >= 0 && G->K >= 1 && G->C >= 1 &&
         (G->N == 0 || (G->means && G->pre_quats && G->pre_scales && G->colours && G->pre_phase && G->pre_opac &&
                        G->pre_planes));
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_scene_workspace_bytes(int N) {
  if (N < 0) return 0;
  const size_t n = N > 0 ? N : 1;
  return 4 * align_up(n * sizeof(uint32_t), 256) + align_up(sort_scratch_words((int)n) * sizeof(uint32_t), 256);
}

extern "C" int cvhrf_scene_prepare_owned(const cvhrf_gaussians* G, const float* R, const float* T,
                                         float near_plane, float far_plane, uint32_t owned_planes, void* ws,
                                         size_t ws_bytes, int32_t* order, float* cam_means, float* z_vals,
                                         float* quats, float* scales, float* colours, float* phase,
                                         float* opacities, float* plane_probs, void* stream) {
  if (!gaussians_ok(G) || !R || !T) return CVHRF_EINVAL;
  const int N = G->N;
  if (N == 0) return CVHRF_OK;
  if (!order || !cam_means || !z_vals || !quats || !scales || !colours || !phase || !opacities || !plane_probs)
    return CVHRF_EINVAL;
  Carver cv(ws, ws_bytes);
  uint32_t* k0 = cv.take<uint32_t>(N);
  uint32_t* v0 = cv.take<uint32_t>(N);
  uint32_t* k1 = cv.take<uint32_t>(N);
  uint32_t* v1 = cv.take<uint32_t>(N);
  uint32_t* scr = cv.take<uint32_t>(sort_scratch_words(N));
  if (cv.overflow || !ws) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const int nb = (N + 255) / 256;
  glue_keys_kernel<<<nb, 256, 0, st>>>(*G, R, T, near_plane, far_plane, owned_planes, k0, v0);
  CVHRF_LAUNCH_CHECK();
  int alt = 0, rc;
  if ((rc = radix_sort_pairs(k0, v0, k1, v1, N, 0, 32, scr, st, &alt))) return rc;
  const uint32_t* ord = alt ? v1 : v0;
  CVHRF_CUDA_TRY(cudaMemcpyAsync(order, ord, N * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
  glue_gather_kernel<<<nb, 256, 0, st>>>(*G, R, T, ord, owned_planes, near_plane, cam_means, z_vals, quats, scales,
                                         colours, phase, opacities, plane_probs);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_scene_prepare(const cvhrf_gaussians* G, const float* R, const float* T, float near_plane,
                                   float far_plane, void* ws, size_t ws_bytes, int32_t* order, float* cam_means,
                                   float* z_vals, float* quats, float* scales, float* colours, float* phase,
                                   float* opacities, float* plane_probs, void* stream) {
  return cvhrf_scene_prepare_owned(G, R, T, near_plane, far_plane, 0xFFFFFFFFu, ws, ws_bytes, order, cam_means,
                                   z_vals, quats, scales, colours, phase, opacities, plane_probs, stream);
}

extern "C" int cvhrf_scene_backward(const cvhrf_gaussians* G, const float* R, const int32_t* order,
                                    const float* g_cam, const float* g_quats, const float* g_scales,
                                    const float* g_colours, const float* g_phase, const float* g_opacities,
                                    const float* g_plane_probs, float* d_means, float* d_pre_quats,
                                    float* d_pre_scales, float* d_colours, float* d_pre_phase, float* d_pre_opacities,
                                    float* d_pre_planes, void* stream) {
  if (!gaussians_ok(G) || !R) return CVHRF_EINVAL;
  const int N = G->N;
  if (N == 0) return CVHRF_OK;
  if (!order || !g_cam || !g_quats || !g_scales || !g_colours || !g_phase || !g_opacities || !g_plane_probs ||
      !d_means || !d_pre_quats || !d_pre_scales || !d_colours || !d_pre_phase || !d_pre_opacities || !d_pre_planes)
    return CVHRF_EINVAL;
  glue_backward_kernel<<<(N + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      *G, R, (const uint32_t*)order, g_cam, g_quats, g_scales, g_colours, g_phase, g_opacities, g_plane_probs,
      d_means, d_pre_quats, d_pre_scales, d_colours, d_pre_phase, d_pre_opacities, d_pre_planes);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
