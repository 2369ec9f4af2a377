// Complex-field tile rasterizer, forward (replaces rasterizer_splat.cu:325-548,
// forward.cu geometry kernels and forward_splat.cu).
//
// Phase 1 (geometry): one fused kernel per Gaussian computes visibility, the 2D mean,
// the 2D covariance, radius, tile count, render constants and the depth sort key;
// a stable radix sort orders Gaussians by depth key; a scan of tile counts in that
// order gives each Gaussian's contiguous slot range for its (tile, Gaussian) pairs.
// Phase 2 (render): pairs are emitted in (depth, index) order and stably sorted by
// tile, which reproduces the reference's (tile | depth) 64-bit key order exactly;
// then one CTA per 16x16 tile composites all K planes in a single pass over the
// tile's Gaussian list (the reference makes one pass per plane).
#include "raster_ws.cuh"

namespace cvhrf {

namespace {

__global__ void __launch_bounds__(256) preprocess_kernel(cvhrf_raster_scene s, Camera cam, GeomWs g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= s.N) return;
  float Wm[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) Wm[k] = __ldg(&s.view_matrix[k]);
  const float x = s.cam_means[3 * i], y = s.cam_means[3 * i + 1], zc = s.cam_means[3 * i + 2];
  // visibility: the intended test of checkFrustum/in_frustum (rasterizer_splat.cu:42-62,
  // auxiliary.h:196-221) on the camera-space depth: z > 0.2 and near < z < far
  g.vis[i] = (zc > 0.2f && zc > cam.near_plane && zc < cam.far_plane) ? 1u : 0u;
  const float2 m2 = means2d(x, y, zc, cam);
  float J[6], Sig[9], JW[6];
  jacobian(x, y, zc, cam, J);
  cov3d(s.quats + 4 * i, s.scales + 3 * i, Sig);
  const float4 cov = cov2d(J, Wm, Sig, JW);
  g.means2d[i] = m2;
  g.cov2d[i] = cov;
  // preprocessGaussiansKernel (forward_splat.cu:17-98) on z_vals
  const float z = s.z_vals[i];
  int radius = 0;
  uint32_t tiles = 0;
  if (!(z <= cam.near_plane || z >= cam.far_plane)) {
    radius = splat_radius(cov);
    if (radius != 0) {
      uint2 rmin, rmax;
      tile_rect(m2, radius, cam.grid_x, cam.grid_y, rmin, rmax);
      tiles = (rmax.y - rmin.y) * (rmax.x - rmin.x);
    }
  }
  g.radii[i] = radius;
  g.tiles[i] = tiles;
  g.key[i] = tiles > 0 ? depth_key(z) : 0xFFFFFFFFu;
  g.order[i] = (uint32_t)i;
  // render constants, computed as renderTileKernel does per pair (forward_splat.cu:200-216)
  const float det = cov.x * cov.w - cov.y * cov.z;
  const float det_inv = 1.0f / det;
  g.conic[i] = make_float4(cov.w * det_inv, -cov.y * det_inv, -cov.z * det_inv, cov.x * det_inv);
  g.rec0[i] = make_float4(m2.x, m2.y, s.opacities[i], 0.f);
  for (int c = 0; c < s.C; ++c) {
    float sn, cs;
    __sincosf(s.phase[i * s.C + c], &sn, &cs);
    const float col = s.colours[i * s.C + c];
    g.cp[(size_t)i * s.C + c] = make_float2(col * cs, col * sn);
  }
}

__global__ void gather_tiles_kernel(const uint32_t* __restrict__ order, const uint32_t* __restrict__ tiles,
                                    uint32_t* __restrict__ out, int N) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < N) out[i] = tiles[order[i]];
}

__global__ void counts_kernel(const uint32_t* offsets, const uint32_t* vis_scan, int N, int32_t* counts) {
  counts[0] = N > 0 ? (int32_t)offsets[N - 1] : 0;
  counts[1] = N > 0 ? (int32_t)vis_scan[N - 1] : 0;
}

__global__ void __launch_bounds__(256) emit_pairs_kernel(GeomWs g, Camera cam, int N, BinWs b, uint32_t cap,
                                                         int32_t* overflow) {
  const int si = blockIdx.x * blockDim.x + threadIdx.x;
  if (si >= N) return;
  const uint32_t gi = g.order[si];
  const uint32_t n = g.tiles[gi];
  if (n == 0) return;
  uint32_t slot = si == 0 ? 0u : g.offsets[si - 1];
  if (slot + n > cap) {  // more pairs than the caller's capacity: flag it, emit nothing
    if (overflow) *overflow = 1;
    return;
  }
  uint2 rmin, rmax;
  tile_rect(g.means2d[gi], g.radii[gi], cam.grid_x, cam.grid_y, rmin, rmax);
  for (uint32_t ty = rmin.y; ty < rmax.y; ++ty)
    for (uint32_t tx = rmin.x; tx < rmax.x; ++tx) {
      b.tkey[slot] = ty * (uint32_t)cam.grid_x + tx;
      b.slot[slot] = slot;
      b.gauss[slot] = gi;
      ++slot;
    }
}

__global__ void clear_ranges_kernel(int2* ranges, int T) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < T) ranges[i] = make_int2(0, 0);
}

__global__ void ranges_kernel(const uint32_t* __restrict__ tkey, const uint32_t* __restrict__ slot,
                              const uint32_t* __restrict__ gauss, int n, int2* ranges, int32_t* point_list,
                              const int32_t* __restrict__ n_dev) {
  if (n_dev) n = min(n, *n_dev);
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t t = tkey[i];
  point_list[i] = (int32_t)gauss[slot[i]];
  if (i == 0 || tkey[i - 1] != t) ranges[t].x = i;
  if (i == n - 1 || tkey[i + 1] != t) ranges[t].y = i + 1;
}

__global__ void capacity_count_kernel(const int32_t* counts, int cap, int32_t* eff, int32_t* overflow) {
  const int n = counts[0];
  const bool fits = n <= cap;
  *eff = fits ? n : 0;
  if (!fits) *overflow = 1;
}

__global__ void visible_mask_kernel(const float* __restrict__ cam_means, int N, float near_plane, float far_plane,
                                    uint8_t* __restrict__ mask) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const float zc = cam_means[3 * i + 2];
  mask[i] = (zc > 0.2f && zc > near_plane && zc < far_plane) ? 1 : 0;
}

__global__ void visible_kernel(const float* __restrict__ cam_means, const uint32_t* __restrict__ vis_scan, int N,
                               float near_plane, float far_plane, int64_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const float zc = cam_means[3 * i + 2];
  if (zc > 0.2f && zc > near_plane && zc < far_plane) out[vis_scan[i] - 1] = i;
}

// renderTileKernel (forward_splat.cu:101-289), all K planes in one pass.
//
// 128 threads per 16x16 tile; each thread owns two horizontally adjacent pixels and
// evaluates both with packed f32x2 arithmetic (sm_100 FFMA2/FMUL2/FADD2).  Every lane
// of a packed operation is an ordinary IEEE-rounded float operation, so each pixel
// sees the reference's arithmetic: power = -0.5 (dx (i00 dx + i10 dy) + dy (i01 dx +
// i11 dy)), G = expf(power), alpha = min(0.99, (o G) w), T' = T (1 - alpha), done when
// T' < 1e-4, last = 1-based position of the last contributor.  A pixel that is done or
// outside the image contributes through a zero weight (acc + 0 * c == acc).
template <int K, int C>
__global__ void __launch_bounds__(128) render_forward_kernel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float4* __restrict__ rec0,
    const float4* __restrict__ conic, const float2* __restrict__ cp, const float* __restrict__ plane_probs,
    int W, int H, int gx, float2* __restrict__ field, float* __restrict__ final_T, int32_t* __restrict__ n_contrib) {
  constexpr int NB = 128;  // Gaussians staged per batch
  __shared__ float2 s_m[NB];       // mean
  __shared__ float2 s_o[NB];       // (opacity, -)
  __shared__ float4 s_c0[NB];      // (i00, i00, i01, i01)
  __shared__ float4 s_c1[NB];      // (i10, i10, i11, i11)
  __shared__ float s_w[K][NB];
  __shared__ int s_pm[NB];           // planes with weight >= 1e-6 (bit p)
  __shared__ float2 s_cp[C][NB];
  const int tile = blockIdx.x;
  const int tx = tile % gx, ty = tile / gx;
  const int lx = (threadIdx.x & 7) * 2, ly = threadIdx.x >> 3;
  const int px = tx * kTile + lx, py = ty * kTile + ly;
  const bool in0 = px < W && py < H, in1 = px + 1 < W && py < H;
  const float2 npx = make_float2(-(float)px, -(float)(px + 1));
  const float pyf = (float)py;
  const int2 range = ranges[tile];
  const int n = range.y - range.x;

  float2 T[K];
  int last0[K], last1[K];
  bool done0[K], done1[K];
  float2 acc0[K][C], acc1[K][C];
#pragma unroll
  for (int p = 0; p < K; ++p) {
    T[p] = make_float2(1.0f, 1.0f);
    last0[p] = last1[p] = 0;
    done0[p] = !in0;
    done1[p] = !in1;
#pragma unroll
    for (int c = 0; c < C; ++c) acc0[p][c] = acc1[p][c] = make_float2(0.f, 0.f);
  }
  bool alldone = !in0 && !in1;

  for (int base = 0; base < n; base += NB) {
    if (__syncthreads_and(alldone)) break;
    {
      const int j = base + threadIdx.x;
      if (j < n) {
        const int gi = point_list[range.x + j];
        const float4 r0 = rec0[gi];
        const float4 cn = conic[gi];
        s_m[threadIdx.x] = make_float2(r0.x, r0.y);
        s_o[threadIdx.x] = make_float2(r0.z, r0.z);
        s_c0[threadIdx.x] = make_float4(cn.x, cn.x, cn.y, cn.y);
        s_c1[threadIdx.x] = make_float4(cn.z, cn.z, cn.w, cn.w);
        int pm = 0;
#pragma unroll
        for (int p = 0; p < K; ++p) {
          const float w = plane_probs[gi * K + p];
          s_w[p][threadIdx.x] = w;
          pm |= (w >= kPlaneCutoff) ? (1 << p) : 0;
        }
        s_pm[threadIdx.x] = pm;
#pragma unroll
        for (int c = 0; c < C; ++c) s_cp[c][threadIdx.x] = cp[gi * C + c];
      }
    }
    __syncthreads();
    const int cnt = min(NB, n - base);
    for (int jj = 0; jj < cnt && !alldone; ++jj) {
      const float2 m = s_m[jj];
      const float2 dx = __fadd2_rn(make_float2(m.x, m.x), npx);
      const float dys = m.y - pyf;
      const float2 dy = make_float2(dys, dys);
      const float4 c0 = s_c0[jj], c1 = s_c1[jj];
      const float2 u = __ffma2_rn(make_float2(c0.x, c0.y), dx, __fmul2_rn(make_float2(c1.x, c1.y), dy));
      const float2 v = __ffma2_rn(make_float2(c0.z, c0.w), dx, __fmul2_rn(make_float2(c1.z, c1.w), dy));
      const float2 power = __fmul2_rn(make_float2(-0.5f, -0.5f), __ffma2_rn(dx, u, __fmul2_rn(dy, v)));
      const bool ok0 = power.x <= 0.0f, ok1 = power.y <= 0.0f;
      if (!ok0 && !ok1) continue;
      const int pm = s_pm[jj];
      if (pm == 0) continue;
      const float2 og = __fmul2_rn(s_o[jj], make_float2(expf(power.x), expf(power.y)));
      const int pos = base + jj + 1;
      bool flip = false;
#pragma unroll
      for (int p = 0; p < K; ++p) {
        if (pm & (1 << p)) {
          const float w = s_w[p][jj];
          const bool a0 = ok0 && !done0[p], a1 = ok1 && !done1[p];
          if (a0 || a1) {
            const float2 aw = __fmul2_rn(og, make_float2(w, w));
            const float2 alpha = make_float2(fminf(kMaxAlpha, aw.x), fminf(kMaxAlpha, aw.y));
            const float2 test = __fmul2_rn(T[p], __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(-alpha.x, -alpha.y)));
            const float2 wt = __fmul2_rn(alpha, T[p]);
            const float2 wt0 = make_float2(a0 ? wt.x : 0.f, a0 ? wt.x : 0.f);
            const float2 wt1 = make_float2(a1 ? wt.y : 0.f, a1 ? wt.y : 0.f);
#pragma unroll
            for (int c = 0; c < C; ++c) {
              const float2 col = s_cp[c][jj];
              acc0[p][c] = __ffma2_rn(wt0, col, acc0[p][c]);
              acc1[p][c] = __ffma2_rn(wt1, col, acc1[p][c]);
            }
            if (a0) { T[p].x = test.x; last0[p] = pos; if (test.x < 0.0001f) { done0[p] = true; flip = true; } }
            if (a1) { T[p].y = test.y; last1[p] = pos; if (test.y < 0.0001f) { done1[p] = true; flip = true; } }
          }
        }
      }
      if (flip) {
        bool all = true;
#pragma unroll
        for (int p = 0; p < K; ++p) all = all && done0[p] && done1[p];
        alldone = all;
      }
    }
  }
  const size_t HW = (size_t)H * W, pix = (size_t)py * W + px;
#pragma unroll
  for (int p = 0; p < K; ++p) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
      if (in0) field[(p * C + c) * HW + pix] = acc0[p][c];
      if (in1) field[(p * C + c) * HW + pix + 1] = acc1[p][c];
    }
    if (in0) { final_T[p * HW + pix] = T[p].x; n_contrib[p * HW + pix] = last0[p]; }
    if (in1) { final_T[p * HW + pix + 1] = T[p].y; n_contrib[p * HW + pix + 1] = last1[p]; }
  }
}

template <int K>
int launch_render_k(int C, dim3 grid, cudaStream_t st, const int2* ranges, const int32_t* pl, const GeomWs& g,
                    const float* pp, int W, int H, int gx, float2* field, float* fT, int32_t* nc) {
  switch (C) {
    case 1: render_forward_kernel<K, 1><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, W, H, gx, field, fT, nc); break;
    case 2: render_forward_kernel<K, 2><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, W, H, gx, field, fT, nc); break;
    default: render_forward_kernel<K, 3><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, W, H, gx, field, fT, nc); break;
  }
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_raster_geometry_workspace_bytes(int N, int K, int C) {
  (void)K;
  if (N < 0 || C < 1) return 0;
  return carve_geom(nullptr, (size_t)-1, N > 0 ? N : 1, C).bytes + 256;
}

static GeomWs carve_geom_checked(void* ws, size_t bytes, int N, int C, bool& ok) {
  GeomWs g = carve_geom(ws, bytes, N > 0 ? N : 1, C);
  ok = g.bytes != 0 && ws != nullptr;
  return g;
}

extern "C" int cvhrf_raster_forward_geometry(const cvhrf_raster_scene* scene, void* geom_ws, size_t geom_bytes,
                                             int32_t* counts_dev, void* stream) {
  if (!scene_ok(scene) || !counts_dev) return CVHRF_EINVAL;
  const cvhrf_raster_scene& s = *scene;
  bool ok;
  GeomWs g = carve_geom_checked(geom_ws, geom_bytes, s.N, s.C, ok);
  if (!ok) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const Camera cam = make_camera(s);
  const int N = s.N;
  if (N > 0) {
    const int nb = (N + 255) / 256;
    preprocess_kernel<<<nb, 256, 0, st>>>(s, cam, g);
    CVHRF_LAUNCH_CHECK();
    int alt = 0, rc;
    // callers usually pass Gaussians already in depth order (Scene.render sorts them):
    // then the 4 sort passes are skipped on the device
    if ((rc = keys_sorted_flag(g.key, N, g.sorted, st))) return rc;
    if ((rc = radix_sort_pairs(g.key, g.order, g.key_alt, g.order_alt, N, 0, 32, g.scratch, st, &alt, g.sorted)))
      return rc;
    if (alt) {  // 4 passes of 8 bits always end in the primary buffers; kept for safety
      CVHRF_CUDA_TRY(cudaMemcpyAsync(g.order, g.order_alt, N * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    }
    gather_tiles_kernel<<<nb, 256, 0, st>>>(g.order, g.tiles, g.offsets, N);
    CVHRF_LAUNCH_CHECK();
    if ((rc = inclusive_scan_u32(g.offsets, g.offsets, N, g.scratch, st))) return rc;
    if ((rc = inclusive_scan_u32(g.vis, g.vis, N, g.scratch, st))) return rc;
  }
  counts_kernel<<<1, 1, 0, st>>>(g.offsets, g.vis, N, counts_dev);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" size_t cvhrf_raster_binning_workspace_bytes(int N, int num_pairs, int W, int H) {
  (void)N; (void)W; (void)H;
  if (num_pairs < 0) return 0;
  return carve_bin(nullptr, (size_t)-1, num_pairs).bytes + 256;
}

extern "C" int cvhrf_raster_forward_render(const cvhrf_raster_scene* scene, const void* geom_ws, size_t geom_bytes,
                                           int num_pairs, int num_visible, void* bin_ws, size_t bin_bytes,
                                           void* field, float* final_Ts, int32_t* n_contrib, int32_t* point_list,
                                           int32_t* ranges, int64_t* visible_indices, void* stream) {
  if (!scene_ok(scene) || num_pairs < 0 || num_visible < 0 || !field || !final_Ts || !n_contrib || !ranges)
    return CVHRF_EINVAL;
  if ((num_pairs > 0 && !point_list) || (num_visible > 0 && !visible_indices)) return CVHRF_EINVAL;
  const cvhrf_raster_scene& s = *scene;
  bool ok;
  GeomWs g = carve_geom_checked(const_cast<void*>(geom_ws), geom_bytes, s.N, s.C, ok);
  if (!ok) return CVHRF_EWORKSPACE;
  BinWs b = carve_bin(bin_ws, bin_bytes, num_pairs);
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const Camera cam = make_camera(s);
  const int T = cam.grid_x * cam.grid_y;
  int rc;
  clear_ranges_kernel<<<(T + 255) / 256, 256, 0, st>>>((int2*)ranges, T);
  CVHRF_LAUNCH_CHECK();
  if (num_pairs > 0) {
    emit_pairs_kernel<<<(s.N + 255) / 256, 256, 0, st>>>(g, cam, s.N, b, (uint32_t)num_pairs, nullptr);
    CVHRF_LAUNCH_CHECK();
    int alt = 0;
    if ((rc = radix_sort_pairs(b.tkey, b.slot, b.tkey_alt, b.slot_alt, num_pairs, 0, tile_bits(T), b.scratch, st,
                               &alt)))
      return rc;
    if (alt) {  // keep the sorted result in the primary buffers (the backward reads b.slot)
      CVHRF_CUDA_TRY(cudaMemcpyAsync(b.tkey, b.tkey_alt, num_pairs * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
      CVHRF_CUDA_TRY(cudaMemcpyAsync(b.slot, b.slot_alt, num_pairs * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    }
    ranges_kernel<<<(num_pairs + 255) / 256, 256, 0, st>>>(b.tkey, b.slot, b.gauss, num_pairs, (int2*)ranges,
                                                           point_list, nullptr);
    CVHRF_LAUNCH_CHECK();
  }
  if (num_visible > 0) {
    visible_kernel<<<(s.N + 255) / 256, 256, 0, st>>>(s.cam_means, g.vis, s.N, s.near_plane, s.far_plane,
                                                      visible_indices);
    CVHRF_LAUNCH_CHECK();
  }
  dim3 grid(T);
  const int2* rg = (const int2*)ranges;
  float2* f = (float2*)field;
  switch (s.K) {
    case 1: return launch_render_k<1>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 2: return launch_render_k<2>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 3: return launch_render_k<3>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 4: return launch_render_k<4>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 5: return launch_render_k<5>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 6: return launch_render_k<6>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 7: return launch_render_k<7>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    default: return launch_render_k<8>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
  }
}

// Same as cvhrf_raster_forward_render without the host round trip: the pair count stays in
// counts_dev[0] (written by cvhrf_raster_forward_geometry), buffers are sized for
// pairs_capacity, and *overflow is set when the count exceeds it (outputs then invalid).
extern "C" int cvhrf_raster_forward_render_capacity(const cvhrf_raster_scene* scene, const void* geom_ws,
                                                    size_t geom_bytes, const int32_t* counts_dev, int pairs_capacity,
                                                    void* bin_ws, size_t bin_bytes, void* field, float* final_Ts,
                                                    int32_t* n_contrib, int32_t* point_list, int32_t* ranges,
                                                    uint8_t* visible_mask, int32_t* overflow, void* stream) {
  const int num_pairs = pairs_capacity;
  if (!scene_ok(scene) || num_pairs < 1 || !counts_dev || !field || !final_Ts || !n_contrib || !ranges ||
      !point_list || !overflow || (scene->N > 0 && !visible_mask))
    return CVHRF_EINVAL;
  const cvhrf_raster_scene& s = *scene;
  bool ok;
  GeomWs g = carve_geom_checked(const_cast<void*>(geom_ws), geom_bytes, s.N, s.C, ok);
  if (!ok) return CVHRF_EWORKSPACE;
  BinWs b = carve_bin(bin_ws, bin_bytes, num_pairs);
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const Camera cam = make_camera(s);
  const int T = cam.grid_x * cam.grid_y;
  int rc;
  clear_ranges_kernel<<<(T + 255) / 256, 256, 0, st>>>((int2*)ranges, T);
  CVHRF_LAUNCH_CHECK();
  capacity_count_kernel<<<1, 1, 0, st>>>(counts_dev, num_pairs, b.eff, overflow);
  CVHRF_LAUNCH_CHECK();
  if (num_pairs > 0) {
    emit_pairs_kernel<<<(s.N + 255) / 256, 256, 0, st>>>(g, cam, s.N, b, (uint32_t)num_pairs, overflow);
    CVHRF_LAUNCH_CHECK();
    int alt = 0;
    if ((rc = radix_sort_pairs(b.tkey, b.slot, b.tkey_alt, b.slot_alt, num_pairs, 0, tile_bits(T), b.scratch, st,
                               &alt, nullptr, b.eff)))
      return rc;
    if (alt) {  // keep the sorted result in the primary buffers (the backward reads b.slot)
      CVHRF_CUDA_TRY(cudaMemcpyAsync(b.tkey, b.tkey_alt, num_pairs * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
      CVHRF_CUDA_TRY(cudaMemcpyAsync(b.slot, b.slot_alt, num_pairs * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st));
    }
    ranges_kernel<<<(num_pairs + 255) / 256, 256, 0, st>>>(b.tkey, b.slot, b.gauss, num_pairs, (int2*)ranges,
                                                           point_list, b.eff);
    CVHRF_LAUNCH_CHECK();
  }
  if (s.N > 0) {
    visible_mask_kernel<<<(s.N + 255) / 256, 256, 0, st>>>(s.cam_means, s.N, s.near_plane, s.far_plane,
                                                           visible_mask);
    CVHRF_LAUNCH_CHECK();
  }
  dim3 grid(T);
  const int2* rg = (const int2*)ranges;
  float2* f = (float2*)field;
  switch (s.K) {
    case 1: return launch_render_k<1>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 2: return launch_render_k<2>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 3: return launch_render_k<3>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 4: return launch_render_k<4>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 5: return launch_render_k<5>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 6: return launch_render_k<6>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    case 7: return launch_render_k<7>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
    default: return launch_render_k<8>(s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts, n_contrib);
  }
}
