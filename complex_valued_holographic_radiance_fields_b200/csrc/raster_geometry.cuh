// Per-Gaussian projection geometry of the wave rasterizer (forward and backward).
//
// Each function restates one reference kernel and keeps its arithmetic expression
// for expression (same operand order, same sub-expressions, default nvcc FMA
// contraction), because the tile binning downstream has to be bit-exact:
//   means2d          wave_rasterizer/forward.cu:297-330 (compute_means2d_kernel)
//   jacobian         wave_rasterizer/forward.cu:64-122  (compute_jacobian_kernel)
//   cov3d            wave_rasterizer/forward.cu:10-61   (compute_cov3d_cuda_kernel, GLM
//                    column-major products expanded term by term)
//   cov2d            wave_rasterizer/forward.cu:221-294 (four batched matmuls, each
//                    element accumulated as fma(a2,b2,fma(a1,b1,a0*b0)) -- the order the
//                    reference's cuBLAS batched GEMMs produce, verified bitwise on B200),
//                    then +0.3 on the diagonal (:125-136)
//   radius/rect      wave_rasterizer/forward_splat.cu:17-98 and auxiliary.h:95-112
// Backward:
//   means2d_bwd      wave_rasterizer/backward.cu:453-497
//   cov2d_bwd        wave_rasterizer/backward.cu:363-450 (five matmuls)
//   jacobian_bwd     wave_rasterizer/backward.cu:201-272
//   cov3d_bwd        wave_rasterizer/backward.cu:78-198 (no chain through quaternion
//                    normalisation, as in the reference)
#pragma once
#include "common.cuh"

namespace cvhrf {

constexpr int kTile = 16;                  // BLOCK_X = BLOCK_Y (config.h:16-17)
constexpr float kPlaneCutoff = 1e-6f;      // PLANE_PROBABILITY_CUTOFF (config.h:19)
constexpr float kMaxAlpha = 0.99f;         // MAX_ALPHA_VALUE (config.h:21)
constexpr int kMaxPlanes = 8;              // MAX_PLANES (config.h:23)
constexpr int kMaxChannels = 3;            // MAX_CHANNELS (config.h:22)

struct Camera {
  float fx, fy, px, py;
  float near_plane, far_plane;
  float half_tan_fov_x, half_tan_fov_y;   // 0.5f * width / fx (forward.cu:193-194)
  int W, H, grid_x, grid_y;
};

// matmul element of cuBLAS batched SGEMM with k = 3
__device__ __forceinline__ float dot3(float a0, float b0, float a1, float b1, float a2, float b2) {
  return __fmaf_rn(a2, b2, __fmaf_rn(a1, b1, __fmul_rn(a0, b0)));
}

__device__ __forceinline__ float2 means2d(float x, float y, float z, const Camera& cam) {
  if (z <= cam.near_plane || z >= cam.far_plane) return make_float2(1e6f, 1e6f);
  const float inv_z = 1.0f / z;
  const float px_div = -x * inv_z;
  const float py_div = -y * inv_z;
  return make_float2(cam.fx * px_div + cam.px, cam.fy * py_div + cam.py);
}

// J (2x3, row-major)
__device__ __forceinline__ void jacobian(float tx, float ty, float tz, const Camera& cam, float* J) {
  if (tz <= cam.near_plane || tz >= cam.far_plane) {
#pragma unroll
    for (int i = 0; i < 6; ++i) J[i] = 0.0f;
    return;
  }
  const float tz2 = tz * tz;
  const float lim_x = 1.3f * cam.half_tan_fov_x;
  const float lim_y = 1.3f * cam.half_tan_fov_y;
  const float tx_tz = tx / tz;
  const float ty_tz = ty / tz;
  const float clamped_tx_tz = fminf(fmaxf(tx_tz, -lim_x), lim_x);
  const float clamped_ty_tz = fminf(fmaxf(ty_tz, -lim_y), lim_y);
  const float clamped_tx = clamped_tx_tz * tz;
  const float clamped_ty = clamped_ty_tz * tz;
  J[0] = cam.fx / tz;
  J[1] = 0.0f;
  J[2] = -(cam.fx * clamped_tx) / tz2;
  J[3] = 0.0f;
  J[4] = cam.fy / tz;
  J[5] = -(cam.fy * clamped_ty) / tz2;
}

// Rotation matrix of a normalised quaternion in GLM column-major storage M[col][row]
// (forward.cu:36-40: glm::mat3 R(c0r0, c0r1, c0r2, c1r0, ...)).
__device__ __forceinline__ void quat_to_glm_rot(float r, float x, float y, float z, float M[3][3]) {
  M[0][0] = 1.f - 2.f * (y * y + z * z);
  M[0][1] = 2.f * (x * y - r * z);
  M[0][2] = 2.f * (x * z + r * y);
  M[1][0] = 2.f * (x * y + r * z);
  M[1][1] = 1.f - 2.f * (x * x + z * z);
  M[1][2] = 2.f * (y * z - r * x);
  M[2][0] = 2.f * (x * z - r * y);
  M[2][1] = 2.f * (y * z + r * x);
  M[2][2] = 1.f - 2.f * (x * x + y * y);
}

__device__ __forceinline__ void normalize_quat(const float* q, float& r, float& x, float& y, float& z) {
  r = q[0]; x = q[1]; y = q[2]; z = q[3];
  const float norm = sqrtf(r * r + x * x + y * y + z * z);
  r /= norm;
  x /= norm;
  y /= norm;
  z /= norm;
}

// GLM mat3 product (A*B)[c][r] = A[0][r]*B[c][0] + A[1][r]*B[c][1] + A[2][r]*B[c][2]
__device__ __forceinline__ void glm_mul(const float A[3][3], const float B[3][3], float Out[3][3]) {
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int r = 0; r < 3; ++r) Out[c][r] = A[0][r] * B[c][0] + A[1][r] * B[c][1] + A[2][r] * B[c][2];
}
__device__ __forceinline__ void glm_transpose(const float A[3][3], float Out[3][3]) {
#pragma unroll
  for (int c = 0; c < 3; ++c)
#pragma unroll
    for (int r = 0; r < 3; ++r) Out[c][r] = A[r][c];
}

// Sigma (3x3 row-major): out[i*3+j] = (SR^T SR)[i][j] with SR = S*R (GLM), S = diag(scale)
__device__ __forceinline__ void cov3d(const float* quat, const float* scale, float* out) {
  float r, x, y, z;
  normalize_quat(quat, r, x, y, z);
  float R[3][3], S[3][3] = {{scale[0], 0.f, 0.f}, {0.f, scale[1], 0.f}, {0.f, 0.f, scale[2]}};
  quat_to_glm_rot(r, x, y, z, R);
  float SR[3][3], SRt[3][3], Sig[3][3];
  glm_mul(S, R, SR);
  glm_transpose(SR, SRt);
  glm_mul(SRt, SR, Sig);
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) out[i * 3 + j] = Sig[i][j];
}

// cov2D = ((J W) Sigma) W^T J^T + 0.3 I, returned as (xx, xy, yx, yy); JW (2x3) also returned.
__device__ __forceinline__ float4 cov2d(const float* J, const float* Wm, const float* Sig, float* JW) {
  float B[6], Cm[6];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      JW[i * 3 + j] = dot3(J[i * 3 + 0], Wm[0 * 3 + j], J[i * 3 + 1], Wm[1 * 3 + j], J[i * 3 + 2], Wm[2 * 3 + j]);
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      B[i * 3 + j] = dot3(JW[i * 3 + 0], Sig[0 * 3 + j], JW[i * 3 + 1], Sig[1 * 3 + j], JW[i * 3 + 2], Sig[2 * 3 + j]);
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)  // (B W^T)[i][j] = sum_k B[i][k] W[j][k]
      Cm[i * 3 + j] = dot3(B[i * 3 + 0], Wm[j * 3 + 0], B[i * 3 + 1], Wm[j * 3 + 1], B[i * 3 + 2], Wm[j * 3 + 2]);
  float c[4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 2; ++j)  // (C J^T)[i][j] = sum_k C[i][k] J[j][k]
      c[i * 2 + j] = dot3(Cm[i * 3 + 0], J[j * 3 + 0], Cm[i * 3 + 1], J[j * 3 + 1], Cm[i * 3 + 2], J[j * 3 + 2]);
  c[0] += 0.3f;
  c[3] += 0.3f;
  return make_float4(c[0], c[1], c[2], c[3]);
}

// Radius of forward_splat.cu:41-85 (antialiasing on: +0.3 once more); 0 = culled.
__device__ __forceinline__ int splat_radius(float4 cov) {
  float cov_x = cov.x, cov_y = cov.y, cov_z = cov.z, cov_w = cov.w;
  float det_cov = cov_x * cov_w - cov_y * cov_z;
  if (fabsf(det_cov) < 1e-10f) return 0;
  const float reg_value = 0.3f;
  cov_x += reg_value;
  cov_w += reg_value;
  det_cov = cov_x * cov_w - cov_y * cov_z;
  const float det = det_cov;
  if (fabsf(det) < 1e-8f) return 0;
  const float mid = 0.5f * (cov_x + cov_w);
  const float disc = fmaxf(0.1f, mid * mid - det);
  const float lambda1 = mid + sqrtf(disc);
  const float lambda2 = mid - sqrtf(disc);
  const float radius_x = ceilf(3.0f * sqrtf(fmaxf(lambda1, lambda2)));
  return (int)radius_x;
}

// getRect (auxiliary.h:95-112) with CUDA's saturating float->uint conversions.
__device__ __forceinline__ void tile_rect(float2 p, int max_radius, int gx, int gy, uint2& rmin, uint2& rmax) {
  const int radius = max(1, max_radius);
  const uint32_t ux = (uint32_t)gx, uy = (uint32_t)gy;
  rmin.x = min(ux - 1, max(0u, __float2uint_rz((p.x - radius) / kTile)));
  rmin.y = min(uy - 1, max(0u, __float2uint_rz((p.y - radius) / kTile)));
  rmax.x = min(ux, max(1u, __float2uint_rz((p.x + radius + kTile - 1) / kTile)));
  rmax.y = min(uy, max(1u, __float2uint_rz((p.y + radius + kTile - 1) / kTile)));
  if (rmax.x <= rmin.x) rmax.x = min(ux, rmin.x + 1);
  if (rmax.y <= rmin.y) rmax.y = min(uy, rmin.y + 1);
}

// Depth sort key of duplicateWithKeysKernel (rasterizer_splat.cu:147-158).
__device__ __forceinline__ uint32_t depth_key(float depth) {
  uint32_t b = __float_as_uint(depth);
  return (b & 0x80000000u) == 0 ? (b | 0x80000000u) : (b & 0x7FFFFFFFu);
}

// ------------------------------------------------------------------ backward pieces
// Geometry backward of one Gaussian: d(cov2D) (xx, xy, yx, yy) and d(mean2D) ->
// d(cam_mean), d(quat), d(scale).
__device__ __forceinline__ void geometry_backward(const float* cm, const float* quat, const float* scale,
                                                  float2 dmean, const float* G2, const float* Wm, const Camera& cam,
                                                  float* dcam, float* dquat, float* dscale) {
  const float x = cm[0], y = cm[1], z = cm[2];
  // means2d backward (backward.cu:467-496)
  float g0 = 0.f, g1 = 0.f, g2 = 0.f;
  if (!(z <= cam.near_plane || z >= cam.far_plane)) {
    const float z2 = z * z;
    g0 = -cam.fx * dmean.x / z;
    g1 = -cam.fy * dmean.y / z;
    g2 = (cam.fx * x * dmean.x / z2) + (cam.fy * y * dmean.y / z2);
  }
  float J[6], Sig[9], JW[6];
  jacobian(x, y, z, cam, J);
  cov3d(quat, scale, Sig);
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      JW[i * 3 + j] = dot3(J[i * 3 + 0], Wm[0 * 3 + j], J[i * 3 + 1], Wm[1 * 3 + j], J[i * 3 + 2], Wm[2 * 3 + j]);
  // backward.cu:426-439
  float dC[6], dB[6], GJW[6], dS[9], dA[6], dJ[6];
  for (int i = 0; i < 2; ++i)
    for (int j = 0; j < 3; ++j) {
      dC[i * 3 + j] = G2[i * 2 + 0] * J[0 * 3 + j] + G2[i * 2 + 1] * J[1 * 3 + j];
      GJW[i * 3 + j] = G2[i * 2 + 0] * JW[0 * 3 + j] + G2[i * 2 + 1] * JW[1 * 3 + j];
    }
  for (int i = 0; i < 2; ++i)
    for (int j = 0; j < 3; ++j) dB[i * 3 + j] = dC[i * 3 + 0] * Wm[0 * 3 + j] + dC[i * 3 + 1] * Wm[1 * 3 + j] + dC[i * 3 + 2] * Wm[2 * 3 + j];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) dS[i * 3 + j] = JW[0 * 3 + i] * GJW[0 * 3 + j] + JW[1 * 3 + i] * GJW[1 * 3 + j];
  for (int i = 0; i < 2; ++i)
    for (int j = 0; j < 3; ++j)  // dB Sigma^T
      dA[i * 3 + j] = dB[i * 3 + 0] * Sig[j * 3 + 0] + dB[i * 3 + 1] * Sig[j * 3 + 1] + dB[i * 3 + 2] * Sig[j * 3 + 2];
  for (int i = 0; i < 2; ++i)
    for (int j = 0; j < 3; ++j)  // dA W^T
      dJ[i * 3 + j] = dA[i * 3 + 0] * Wm[j * 3 + 0] + dA[i * 3 + 1] * Wm[j * 3 + 1] + dA[i * 3 + 2] * Wm[j * 3 + 2];
  // jacobian backward (backward.cu:217-271)
  float h0 = 0.f, h1 = 0.f, h2 = 0.f;
  if (!(z <= cam.near_plane || z >= cam.far_plane)) {
    const float tz2 = z * z, tz3 = tz2 * z;
    const float lim_x = 1.3f * cam.half_tan_fov_x, lim_y = 1.3f * cam.half_tan_fov_y;
    const float tx_tz = x / z, ty_tz = y / z;
    const float xm = (tx_tz < -lim_x || tx_tz > lim_x) ? 0.0f : 1.0f;
    const float ym = (ty_tz < -lim_y || ty_tz > lim_y) ? 0.0f : 1.0f;
    const float dJ00_dtz = -cam.fx / tz2;
    const float dJ02_dtx = xm * (-cam.fx / tz2);
    const float dJ02_dtz = xm * (2.0f * cam.fx * x / tz3);
    const float dJ11_dtz = -cam.fy / tz2;
    const float dJ12_dty = ym * (-cam.fy / tz2);
    const float dJ12_dtz = ym * (2.0f * cam.fy * y / tz3);
    h0 = dJ[2] * dJ02_dtx;
    h1 = dJ[5] * dJ12_dty;
    h2 = dJ[0] * dJ00_dtz + dJ[2] * dJ02_dtz + dJ[4] * dJ11_dtz + dJ[5] * dJ12_dtz;
  }
  dcam[0] = g0 + h0;
  dcam[1] = g1 + h1;
  dcam[2] = g2 + h2;
  // cov3d backward (backward.cu:78-198), GLM storage M[col][row]
  float Gm[3][3];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) Gm[i][j] = dS[i * 3 + j];
  float r, qx, qy, qz;
  normalize_quat(quat, r, qx, qy, qz);
  float R[3][3];
  quat_to_glm_rot(r, qx, qy, qz, R);
  float dR[4][3][3] = {
      {{0.f, -2.f * qz, 2.f * qy}, {2.f * qz, 0.f, -2.f * qx}, {-2.f * qy, 2.f * qx, 0.f}},
      {{0.f, 2.f * qy, 2.f * qz}, {2.f * qy, -4.f * qx, -2.f * r}, {2.f * qz, 2.f * r, -4.f * qx}},
      {{-4.f * qy, 2.f * qx, 2.f * r}, {2.f * qx, 0.f, 2.f * qz}, {-2.f * r, 2.f * qz, -4.f * qy}},
      {{-4.f * qz, -2.f * r, 2.f * qx}, {2.f * r, -4.f * qz, 2.f * qy}, {2.f * qx, 2.f * qy, 0.f}}};
  float Rt[3][3], T1[3][3], T2[3][3];
  glm_transpose(R, Rt);
  for (int c = 0; c < 3; ++c)
    for (int rr = 0; rr < 3; ++rr) Rt[c][rr] *= 2.0f;
  glm_mul(Rt, Gm, T1);
  glm_mul(T1, R, T2);
  dscale[0] = T2[0][0] * scale[0];
  dscale[1] = T2[1][1] * scale[1];
  dscale[2] = T2[2][2] * scale[2];
  // SR[c][r] = s_r R[c][r]; S dR likewise
  for (int q = 0; q < 4; ++q) {
    float acc = 0.f;
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) {
        const float sdr_ij = scale[j] * dR[q][i][j], sdr_ji = scale[i] * dR[q][j][i];
        const float sr_ij = scale[j] * R[i][j], sr_ji = scale[i] * R[j][i];
        acc += Gm[i][j] * (sdr_ji * sr_ij + sr_ji * sdr_ij);
      }
    dquat[q] = acc;
  }
}

}  // namespace cvhrf
