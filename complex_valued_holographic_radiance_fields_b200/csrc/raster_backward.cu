// Complex-field tile rasterizer, backward (replaces rasterizer_splat.cu:551-684,
// backward_splat.cu:78-417 and the geometry backward of backward.cu).
//
// The reference accumulates every pixel's contribution with 2C+8 global atomicAdds
// per (pixel, Gaussian).  Here the backward is atomic-free and deterministic:
//   1. render_backward_kernel: one CTA per tile replays the tile's list back to
//      front (same per-pixel arithmetic as renderBackwardTileKernel), reduces each
//      Gaussian's per-pixel contributions across the CTA (warp reduce-scatter, then
//      across warps in shared memory) and writes ONE record per (tile, Gaussian)
//      pair into that pair's emission slot.  A Gaussian's slots are contiguous.
//   2. gaussian_grad_kernel: one thread per Gaussian sums its records and chains
//      d(mean2D), d(cov2D) through the projection (means2d, cov2d, jacobian, cov3d
//      backward) to the camera-space mean, quaternion and scale.
// Record layout (VR = 6 + K + 2C floats): dmean.x, dmean.y, dcov_xx, dcov_xy,
// dcov_yy, dopacity, dplane[K], dcolour[C], dphase[C].
#include "raster_ws.cuh"

namespace cvhrf {

namespace {

constexpr int kRedV = 16;  // padded length of the per-Gaussian vector that is reduced

// Sum v[0..15] over the warp; afterwards every even lane l holds the total of index (l >> 1).
__device__ __forceinline__ float warp_reduce_scatter16(float (&v)[kRedV]) {
  const int lane = threadIdx.x & 31;
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = hi ? v[i] : v[i + 8];
      const float keep = hi ? v[i + 8] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = hi ? v[i] : v[i + 4];
      const float keep = hi ? v[i + 4] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = hi ? v[i] : v[i + 2];
      const float keep = hi ? v[i + 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// Per-Gaussian constants of the backward pixel loop, computed once per batch with the
// reference's expressions (backward_splat.cu:194-206, 283-292), so the per-pixel
// arithmetic is unchanged; plus a conservative bounding box of the region where
// alpha >= 1/255 can hold (outside it the reference `continue`s, :218).
struct BwdG {
  float mx, my, opacity, ex;      // mean, opacity, box half-width
  float cx, cy, cz, ey;           // conic_x, conic_y, conic_z, box half-height
  float A, B, Cc, D;              // d cov / d conic coefficients
  float E, G;                     // (A..G: see render_backward_kernel)
  int ok;                         // det != 0 and the box is non-empty
};

template <int KG, int C>
__global__ void __launch_bounds__(256) render_backward_kernel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const uint32_t* __restrict__ slot_sorted,
    const float4* __restrict__ rec0, const float4* __restrict__ cov2d, const float* __restrict__ colours,
    const float* __restrict__ phase, const float* __restrict__ plane_probs, const float* __restrict__ final_T,
    const int32_t* __restrict__ n_contrib, const float2* __restrict__ grad_field, int K, int W, int H, int gx,
    int p0, int accumulate, float* __restrict__ records) {
  constexpr int NW = 8;
  static_assert(6 + KG + 2 * C <= kRedV, "reduction vector too long");
  __shared__ uint32_t s_slot[256];
  __shared__ BwdG s_g[256];
  __shared__ float s_w[KG][256];
  __shared__ float s_col[C][256];
  __shared__ float2 s_cs[C][256];
  __shared__ float s_part[NW][32][kRedV];

  const int VR = 6 + K + 2 * C;
  const int tile = blockIdx.x;
  const int tx = tile % gx, ty = tile / gx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int px = tx * kTile + (threadIdx.x & 15), py = ty * kTile + (threadIdx.x >> 4);
  const bool inside = px < W && py < H;
  const float pxf = (float)px, pyf = (float)py;
  const int2 range = ranges[tile];
  const int n = range.y - range.x;
  if (n <= 0) return;
  const size_t HW = (size_t)H * W, pix = inside ? (size_t)py * W + px : 0;
  const float ddelx_dx = 0.5f * W, ddely_dy = 0.5f * H;

  float T[KG], last_alpha[KG];
  int last[KG];
  float2 dL[KG][C], acc_rec[KG][C], last_col[KG][C];
  int max_last = 0;
#pragma unroll
  for (int kk = 0; kk < KG; ++kk) {
    const int p = p0 + kk;
    const bool pv = inside && p < K;
    T[kk] = pv ? final_T[p * HW + pix] : 0.f;
    last[kk] = pv ? n_contrib[p * HW + pix] : 0;
    max_last = max(max_last, last[kk]);
    last_alpha[kk] = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      dL[kk][c] = pv ? grad_field[(size_t)(p * C + c) * HW + pix] : make_float2(0.f, 0.f);
      acc_rec[kk][c] = make_float2(0.f, 0.f);
      last_col[kk][c] = make_float2(0.f, 0.f);
    }
  }
  // positions >= the CTA's largest last-contributor index are skipped by every pixel
  __shared__ int s_maxlast;
  if (threadIdx.x == 0) s_maxlast = 0;
  __syncthreads();
  atomicMax(&s_maxlast, max_last);
  __syncthreads();
  const int n_eff = min(n, s_maxlast);

  for (int end = n_eff; end > 0; end -= 256) {
    const int cnt = min(256, end);
    __syncthreads();
    if ((int)threadIdx.x < cnt) {
      const int i = range.x + end - 1 - threadIdx.x;
      const int gi = point_list[i];
      s_slot[threadIdx.x] = slot_sorted[i];
      const float4 r0 = rec0[gi];
      const float4 cov = cov2d[gi];
      float wmax = 0.f;
#pragma unroll
      for (int kk = 0; kk < KG; ++kk) {
        const float w = (p0 + kk < K) ? plane_probs[gi * K + p0 + kk] : 0.f;
        s_w[kk][threadIdx.x] = w;
        if (w >= kPlaneCutoff) wmax = fmaxf(wmax, w);
      }
      BwdG g;
      g.mx = r0.x;
      g.my = r0.y;
      g.opacity = r0.z;
      const float det = cov.x * cov.w - cov.y * cov.z;
      const float det_inv = 1.0f / det;
      g.cx = cov.w * det_inv;
      g.cy = -cov.y * det_inv;
      g.cz = cov.x * det_inv;
      g.A = (cov.w * det_inv * det_inv) * cov.w;
      g.B = (-cov.y * det_inv * det_inv) * (-cov.y);
      g.Cc = (cov.w * det_inv * det_inv) * (-cov.y);
      g.D = -det_inv;
      g.E = (-cov.y * det_inv * det_inv) * cov.x;
      g.G = (cov.x * det_inv * det_inv) * cov.x;
      // alpha >= 1/255 needs d^T conic d <= 2 ln(255 opacity w); box of that ellipse, padded
      const float tau = logf(255.0f * r0.z * wmax);
      g.ok = (det != 0.0f) && (tau > 0.0f) && (wmax > 0.0f);
      const float t2 = 2.0f * fmaxf(tau, 0.0f) * 1.01f;
      g.ex = sqrtf(t2 * fabsf(cov.x)) * 1.01f + 0.05f;
      g.ey = sqrtf(t2 * fabsf(cov.w)) * 1.01f + 0.05f;
      s_g[threadIdx.x] = g;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        s_col[c][threadIdx.x] = colours[gi * C + c];
        float sn, cs;
        __sincosf(phase[gi * C + c], &sn, &cs);
        s_cs[c][threadIdx.x] = make_float2(cs, sn);
      }
    }
    __syncthreads();
    for (int jb = 0; jb < cnt; jb += 32) {
      const int nj = min(32, cnt - jb);
      for (int jl = 0; jl < nj; ++jl) {
        const int jj = jb + jl;
        const int pos = end - 1 - jj;  // 0-based position in the tile list
        const BwdG& g = s_g[jj];
        const float2 d = {g.mx - pxf, g.my - pyf};
        const bool near_px = inside && g.ok && pos < max_last && fabsf(d.x) <= g.ex && fabsf(d.y) <= g.ey;
        if (!__any_sync(0xffffffffu, near_px)) {
          if (lane < kRedV) s_part[warp][jl][lane] = 0.f;
          continue;
        }
        float v[kRedV];
#pragma unroll
        for (int i = 0; i < kRedV; ++i) v[i] = 0.f;
        if (near_px) {
          const float opacity = g.opacity;
          const float conic_x = g.cx, conic_y = g.cy, conic_z = g.cz;
          const float power = -0.5f * (conic_x * d.x * d.x + conic_z * d.y * d.y) - conic_y * d.x * d.y;
          if (power <= 0.0f) {
            const float G = expf(power);
#pragma unroll
            for (int kk = 0; kk < KG; ++kk) {
              const float plane_prob = s_w[kk][jj];
              if (pos >= last[kk] || plane_prob < kPlaneCutoff) continue;
              const float alpha = min(0.99f, opacity * G * plane_prob);
              if (alpha < 1.0f / 255.0f) continue;
              T[kk] = T[kk] / (1.0f - alpha);
              const float dchannel_dcolor = alpha * T[kk];
              float dL_dalpha = 0.0f;
#pragma unroll
              for (int c = 0; c < C; ++c) {
                const float color = s_col[c][jj];
                const float2 cs = s_cs[c][jj];
                const float color_real = color * cs.x;
                const float color_imag = color * cs.y;
                acc_rec[kk][c].x = last_alpha[kk] * last_col[kk][c].x + (1.0f - last_alpha[kk]) * acc_rec[kk][c].x;
                acc_rec[kk][c].y = last_alpha[kk] * last_col[kk][c].y + (1.0f - last_alpha[kk]) * acc_rec[kk][c].y;
                last_col[kk][c] = make_float2(color_real, color_imag);
                const float dre = dL[kk][c].x, dim = dL[kk][c].y;
                dL_dalpha += (color_real - acc_rec[kk][c].x) * dre;
                dL_dalpha += (color_imag - acc_rec[kk][c].y) * dim;
                v[6 + KG + c] += dchannel_dcolor * (cs.x * dre + cs.y * dim);
                v[6 + KG + C + c] += dchannel_dcolor * color * (-cs.y * dre + cs.x * dim);
              }
              dL_dalpha *= T[kk];
              last_alpha[kk] = alpha;
              const float dL_dG = opacity * plane_prob * dL_dalpha;
              const float gdx = G * d.x;
              const float gdy = G * d.y;
              const float dG_ddelx = -gdx * conic_x - gdy * conic_y;
              const float dG_ddely = -gdy * conic_z - gdx * conic_y;
              v[0] += dL_dG * dG_ddelx * ddelx_dx;
              v[1] += dL_dG * dG_ddely * ddely_dy;
              const float dL_dconic_x = -0.5f * gdx * d.x * dL_dG;
              const float dL_dconic_y = -0.5f * gdx * d.y * dL_dG;
              const float dL_dconic_z = -0.5f * gdy * d.y * dL_dG;
              v[2] += dL_dconic_x * g.A + dL_dconic_z * g.B;
              v[3] += dL_dconic_x * g.Cc + dL_dconic_y * g.D + dL_dconic_z * g.E;
              v[4] += dL_dconic_x * g.B + dL_dconic_z * g.G;
              v[5] += G * plane_prob * dL_dalpha;
              v[6 + kk] += opacity * G * dL_dalpha;
            }
          }
        }
        const float tot = warp_reduce_scatter16(v);
        if ((lane & 1) == 0) s_part[warp][jl][lane >> 1] = tot;
      }
      __syncthreads();
      const int V = 6 + KG + 2 * C;
      for (int e = threadIdx.x; e < nj * kRedV; e += blockDim.x) {
        const int jl = e / kRedV, idx = e - jl * kRedV;
        if (idx >= V) continue;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) s += s_part[w][jl][idx];
        int ri;
        if (idx < 6) ri = idx;
        else if (idx < 6 + KG) { const int p = p0 + idx - 6; if (p >= K) continue; ri = 6 + p; }
        else ri = 6 + K + (idx - 6 - KG);
        float* dst = records + (size_t)s_slot[jb + jl] * VR + ri;
        if (accumulate && (idx < 6 || idx >= 6 + KG)) s += *dst;
        *dst = s;
      }
      __syncthreads();
    }
  }
  // pairs past the CTA's last contributor get zero records
  if (n_eff < n) {
    const int V = VR;
    for (int e = threadIdx.x; e < (n - n_eff) * V; e += blockDim.x) {
      const int q = e / V, ri = e - q * V;
      const bool mine = ri < 6 || ri >= 6 + K || (ri - 6 >= p0 && ri - 6 < p0 + KG);
      if (!mine) continue;
      float* dst = records + (size_t)slot_sorted[range.x + n_eff + q] * VR + ri;
      if (!(accumulate && (ri < 6 || ri >= 6 + K))) *dst = 0.f;
    }
  }
}

__global__ void __launch_bounds__(128) gaussian_grad_kernel(cvhrf_raster_scene s, Camera cam, GeomWs g,
                                                            const float* __restrict__ records, float* gcam,
                                                            float* gz, float* gq, float* gs, float* gcol,
                                                            float* gph, float* gop, float* gpl) {
  const int si = blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= s.N) return;
  const int K = s.K, C = s.C, VR = 6 + K + 2 * C;
  const uint32_t gi = g.order[si];
  const uint32_t a = si == 0 ? 0u : g.offsets[si - 1], b = g.offsets[si];
  float r[6 + kMaxPlanes + 2 * kMaxChannels];
  for (int i = 0; i < VR; ++i) r[i] = 0.f;
  for (uint32_t k = a; k < b; ++k) {
    const float* rec = records + (size_t)k * VR;
    for (int i = 0; i < VR; ++i) r[i] += rec[i];
  }
  float dcam[3] = {0.f, 0.f, 0.f}, dq[4] = {0.f, 0.f, 0.f, 0.f}, ds[3] = {0.f, 0.f, 0.f};
  if (b > a) {
    float Wm[9];
    for (int k = 0; k < 9; ++k) Wm[k] = __ldg(&s.view_matrix[k]);
    const float G2[4] = {r[2], r[3], r[3], r[4]};
    geometry_backward(s.cam_means + 3 * gi, s.quats + 4 * gi, s.scales + 3 * gi, make_float2(r[0], r[1]), G2, Wm,
                      cam, dcam, dq, ds);
  }
  for (int k = 0; k < 3; ++k) gcam[3 * gi + k] = dcam[k];
  for (int k = 0; k < 4; ++k) gq[4 * gi + k] = dq[k];
  for (int k = 0; k < 3; ++k) gs[3 * gi + k] = ds[k];
  gz[gi] = 0.f;
  gop[gi] = r[5];
  for (int p = 0; p < K; ++p) gpl[gi * K + p] = r[6 + p];
  for (int c = 0; c < C; ++c) {
    gcol[gi * C + c] = r[6 + K + c];
    gph[gi * C + c] = r[6 + K + C + c];
  }
}

template <int KG>
void launch_bwd_kg(int C, dim3 grid, cudaStream_t st, const int2* ranges, const int32_t* pl, const uint32_t* slot,
                   const GeomWs& g, const cvhrf_raster_scene& s, const float* fT, const int32_t* nc,
                   const float2* gf, int gx, int p0, int accumulate, float* rec) {
#define CVHRF_BWD(CC)                                                                                          \
  render_backward_kernel<KG, CC><<<grid, 256, 0, st>>>(ranges, pl, slot, g.rec0, g.cov2d, s.colours, s.phase,   \
                                                       s.plane_probs, fT, nc, gf, s.K, s.W, s.H, gx, p0,        \
                                                       accumulate, rec)
  switch (C) {
    case 1: CVHRF_BWD(1); break;
    case 2: CVHRF_BWD(2); break;
    default: CVHRF_BWD(3); break;
  }
#undef CVHRF_BWD
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_raster_backward_workspace_bytes(int num_pairs, int K, int C) {
  if (num_pairs < 0 || K < 1 || C < 1) return 0;
  const size_t n = num_pairs > 0 ? num_pairs : 1;
  return align_up(n * (6 + K + 2 * C) * sizeof(float), 256);
}

extern "C" int cvhrf_raster_backward(const cvhrf_raster_scene* scene, const void* geom_ws, size_t geom_bytes,
                                     const void* bin_ws, size_t bin_bytes, int num_pairs, const void* grad_field,
                                     const float* final_Ts, const int32_t* n_contrib, const int32_t* point_list,
                                     const int32_t* ranges, void* bwd_ws, size_t bwd_bytes, float* grad_cam_means, float* grad_z_vals,
                                     float* grad_quats, float* grad_scales, float* grad_colours, float* grad_phase,
                                     float* grad_opacities, float* grad_plane_probs, void* stream) {
  if (!scene_ok(scene) || num_pairs < 0 || !grad_field || !final_Ts || !n_contrib || !ranges) return CVHRF_EINVAL;
  if (num_pairs > 0 && !point_list) return CVHRF_EINVAL;
  const cvhrf_raster_scene& s = *scene;
  if (s.N > 0 && !(grad_cam_means && grad_z_vals && grad_quats && grad_scales && grad_colours && grad_phase &&
                   grad_opacities && grad_plane_probs))
    return CVHRF_EINVAL;
  if (s.N == 0) return CVHRF_OK;
  GeomWs g = carve_geom(const_cast<void*>(geom_ws), geom_bytes, s.N, s.C);
  if (g.bytes == 0 || !geom_ws) return CVHRF_EWORKSPACE;
  BinWs b = carve_bin(const_cast<void*>(bin_ws), bin_bytes, num_pairs);
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  if (!bwd_ws || bwd_bytes < cvhrf_raster_backward_workspace_bytes(num_pairs, s.K, s.C)) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const Camera cam = make_camera(s);
  float* rec = (float*)bwd_ws;
  if (num_pairs > 0) {
    const int T = cam.grid_x * cam.grid_y;
    dim3 grid(T);
    const int32_t* pl = point_list;
    const int KG = s.K <= 4 ? s.K : 4;
    for (int p0 = 0; p0 < s.K; p0 += KG) {
      const int acc = p0 > 0 ? 1 : 0;
      switch (KG) {
        case 1: launch_bwd_kg<1>(s.C, grid, st, (const int2*)ranges, pl, b.slot, g, s, final_Ts, n_contrib, (const float2*)grad_field, cam.grid_x, p0, acc, rec); break;
        case 2: launch_bwd_kg<2>(s.C, grid, st, (const int2*)ranges, pl, b.slot, g, s, final_Ts, n_contrib, (const float2*)grad_field, cam.grid_x, p0, acc, rec); break;
        case 3: launch_bwd_kg<3>(s.C, grid, st, (const int2*)ranges, pl, b.slot, g, s, final_Ts, n_contrib, (const float2*)grad_field, cam.grid_x, p0, acc, rec); break;
        default: launch_bwd_kg<4>(s.C, grid, st, (const int2*)ranges, pl, b.slot, g, s, final_Ts, n_contrib, (const float2*)grad_field, cam.grid_x, p0, acc, rec); break;
      }
      CVHRF_LAUNCH_CHECK();
    }
  }
  gaussian_grad_kernel<<<(s.N + 127) / 128, 128, 0, st>>>(s, cam, g, rec, grad_cam_means, grad_z_vals, grad_quats,
                                                          grad_scales, grad_colours, grad_phase, grad_opacities,
                                                          grad_plane_probs);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

