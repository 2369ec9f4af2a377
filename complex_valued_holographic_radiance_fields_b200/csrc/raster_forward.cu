// Complex-field tile rasterizer, forward (replaces rasterizer_splat.cu:325-548,
// forward.cu geometry kernels and forward_splat.cu).
//
// Phase 1 (geometry): one fused kernel per Gaussian computes visibility, the 2D mean,
// the 2D covariance, radius, tile count, render constants and the depth sort key;
// a stable radix sort orders Gaussians by depth key; a scan of tile counts in that
// order gives each Gaussian's contiguous slot range for its (tile, Gaussian) pairs.
// Phase 2 (render): pairs are emitted in (depth, index) order and stably sorted by
// tile, which reproduces the reference's (tile | depth) 64-bit key order exactly;
// then one CTA per 16x16 tile composites the K planes one after another, each over the
// tile's Gaussians of that plane (compacted on chip from the depth-ordered list).
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

// Pairs are written by whole warps: lane j computes Gaussian j's tile rectangle, then the
// warp writes each of the 32 Gaussians' (tile key, Gaussian) pairs with consecutive lanes
// on consecutive slots.  The pair's slot is its index, so no slot array is written: the
// tile sort's first pass takes index values (radix_sort_pairs with v0 == nullptr).
__global__ void __launch_bounds__(256) emit_pairs_kernel(GeomWs g, Camera cam, int N, BinWs b, uint32_t cap,
                                                         int32_t* overflow) {
  const int si = blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  uint32_t n = 0, slot = 0, gi = 0;
  uint2 rmin = make_uint2(0, 0), rmax = make_uint2(0, 0);
  if (si < N) {
    gi = g.order[si];
    n = g.tiles[gi];
    if (n) {
      slot = si == 0 ? 0u : g.offsets[si - 1];
      if (slot + n > cap) {  // more pairs than the caller's capacity: flag it, emit nothing
        if (overflow) *overflow = 1;
        n = 0;
      } else {
        tile_rect(g.means2d[gi], g.radii[gi], cam.grid_x, cam.grid_y, rmin, rmax);
      }
    }
  }
  unsigned todo = __ballot_sync(0xffffffffu, n != 0);
  while (todo) {
    const int j = __ffs(todo) - 1;
    todo &= todo - 1;
    const uint32_t nj = __shfl_sync(0xffffffffu, n, j);
    const uint32_t sj = __shfl_sync(0xffffffffu, slot, j);
    const uint32_t gj = __shfl_sync(0xffffffffu, gi, j);
    const uint32_t x0 = __shfl_sync(0xffffffffu, rmin.x, j), y0 = __shfl_sync(0xffffffffu, rmin.y, j);
    const uint32_t w = __shfl_sync(0xffffffffu, rmax.x, j) - x0;
    for (uint32_t t = lane; t < nj; t += 32) {
      const uint32_t ty = t / w, tx = t - ty * w;
      b.tkey[sj + t] = (y0 + ty) * (uint32_t)cam.grid_x + x0 + tx;
      b.gauss[sj + t] = gj;
    }
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
// Block -> tile map for the render kernels: tiles by decreasing list length (1024 buckets
// of 8 list entries, the longest bucket first; order inside a bucket is arbitrary), so the
// longest tiles start first and the last wave holds short ones.  Every tile's output is
// independent of the order.
__global__ void __launch_bounds__(1024) tile_order_kernel(const int2* __restrict__ ranges, int T,
                                                          int32_t* __restrict__ order) {
  constexpr int NBK = 1024;
  __shared__ int cnt[NBK];
  __shared__ uint32_t sh[33];
  cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int w = ranges[t].y - ranges[t].x;
    atomicAdd(&cnt[NBK - 1 - min(w >> 3, NBK - 1)], 1);   // bucket 0 = longest
  }
  __syncthreads();
  {  // exclusive scan of the 1024 bucket counts (warp scans, then over the 32 warp totals)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = cnt[threadIdx.x];
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += y;
    }
    if (lane == 31) sh[warp] = (uint32_t)inc;
    __syncthreads();
    if (warp == 0) {
      int w = (int)sh[lane], wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += y;
      }
      sh[lane] = (uint32_t)(wi - w);
    }
    __syncthreads();
    cnt[threadIdx.x] = (int)sh[warp] + inc - c;
  }
  __syncthreads();
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const int w = ranges[t].y - ranges[t].x;
    order[atomicAdd(&cnt[NBK - 1 - min(w >> 3, NBK - 1)], 1)] = t;
  }
}

// One CTA of 128 threads per 16x16 tile; each thread owns two horizontally adjacent pixels
// as a packed f32x2 pair (sm_100 FFMA2/FMUL2/FADD2; every lane of a packed operation is an
// ordinary IEEE-rounded float operation) and each warp an 8 x 8 quadrant.  The planes are
// composited one after another: for plane p the CTA walks the tile's depth-ordered list in
// batches of 128, keeps (ballot compaction, order preserved) only the Gaussians whose
// plane-p weight is >= the cutoff, and front-to-back blends them.  Per pixel this is
// exactly the reference's chain: power = -0.5 (dx (i00 dx + i10 dy) + dy (i01 dx + i11 dy)),
// skip if power > 0, G = expf(power), alpha = min(0.99, (o G) w), the pixel takes
// colour * alpha * T, T' = T (1 - alpha), last = 1-based list position, and stops once
// T' < 1e-4.  "Stopped" is the same as T < 1e-4 (T starts at 1 and changes only through
// a contribution), so a stopped or off-image pixel just gets alpha = 0: then T (1 - 0) == T
// and acc + 0 * c == acc exactly.  A warp whose 64 pixels have all stopped skips the rest
// of the plane, and the CTA leaves the plane when all 256 have.

// ln(2^-26) - 0.1: with power < kFarLog - ln(opacity w), alpha = min(0.99, opacity expf(power) w)
// stays below 2^-26 even with expf's rounding, so 1 - alpha rounds to 1.0f
constexpr float kFarLog = -18.0218f - 0.1f;

template <int C>
__global__ void __launch_bounds__(128) render_forward_kernel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float4* __restrict__ rec0,
    const float4* __restrict__ conic, const float2* __restrict__ cp, const float* __restrict__ plane_probs, int K,
    int W, int H, int gx, float2* __restrict__ field, float* __restrict__ final_T, int32_t* __restrict__ n_contrib,
    const int32_t* __restrict__ tile_order) {
  constexpr int NT = 128, NB = 128, NW = 4;
  static_assert(NB == NT, "one staged Gaussian per thread");
  __shared__ float4 s_mo[NB];      // (mx, mx, my, list position)
  __shared__ float4 s_c0[NB];      // (i00, i00, i01, i01)
  __shared__ float4 s_c1[NB];      // (i10, i10, i11, i11)
  __shared__ float4 s_ow[NB];      // (o, o, w, w)
  __shared__ float s_far[NB];      // power below which alpha < 2^-26 (the far-field skip)
  __shared__ float4 s_col[C][NB];  // (re, re, im, im)
  __shared__ int s_cnt[NW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile = tile_order ? tile_order[blockIdx.x] : (int)blockIdx.x;
  const int tx = tile % gx, ty = tile / gx;
  const int px = tx * kTile + (warp & 1) * 8 + (lane & 3) * 2, py = ty * kTile + (warp >> 1) * 8 + (lane >> 2);
  const bool rowin = py < H;
  const float2 npx = make_float2(-(float)px, -(float)(px + 1));
  const float pyf = (float)py;
  const int2 range = ranges[tile];
  const int n = range.y - range.x;
  const size_t HW = (size_t)H * W, pix = (size_t)py * W + px;

  for (int p = 0; p < K; ++p) {
    // off-image pixels start "stopped" (T = 0 < 1e-4) and are never written
    float2 T = make_float2(rowin && px < W ? 1.f : 0.f, rowin && px + 1 < W ? 1.f : 0.f);
    int last0 = 0, last1 = 0;
    float2 re[C], im[C];
#pragma unroll
    for (int c = 0; c < C; ++c) re[c] = im[c] = make_float2(0.f, 0.f);

    for (int base = 0; base < n; base += NB) {
      const bool mine_done = T.x < 1e-4f && T.y < 1e-4f;
      if (__syncthreads_and(mine_done)) break;
      // stage: keep this batch's plane-p Gaussians, in list order
      const int j = base + tid;
      bool keep = false;
      int gi = 0;
      if (j < n) {
        gi = point_list[range.x + j];
        keep = plane_probs[(size_t)gi * K + p] >= kPlaneCutoff;
      }
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      if (lane == 0) s_cnt[warp] = __popc(bal);
      __syncthreads();
      int off = 0, cnt = 0;
#pragma unroll
      for (int w2 = 0; w2 < NW; ++w2) {
        off += w2 < warp ? s_cnt[w2] : 0;
        cnt += s_cnt[w2];
      }
      if (keep) {
        const int o = off + __popc(bal & ((1u << lane) - 1u));
        const float4 r0 = rec0[gi];
        const float4 cn = conic[gi];
        const float w = plane_probs[(size_t)gi * K + p];
        s_mo[o] = make_float4(r0.x, r0.x, r0.y, __int_as_float(j + 1));
        s_c0[o] = make_float4(cn.x, cn.x, cn.y, cn.y);
        s_c1[o] = make_float4(cn.z, cn.z, cn.w, cn.w);
        s_ow[o] = make_float4(r0.z, r0.z, w, w);
        s_far[o] = kFarLog - logf(r0.z * w);
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const float2 v = cp[(size_t)gi * C + c];
          s_col[c][o] = make_float4(v.x, v.x, v.y, v.y);
        }
      }
      __syncthreads();
      // a warp whose 64 pixels have all stopped skips the batch (it only adds exact zeros)
      if (__all_sync(0xffffffffu, mine_done)) continue;
      for (int jj = 0; jj < cnt; ++jj) {
        if ((jj & 31) == 31 && __all_sync(0xffffffffu, T.x < 1e-4f && T.y < 1e-4f)) break;
        const float4 mo = s_mo[jj];
        const float4 k0 = s_c0[jj], k1 = s_c1[jj];
        const float dys = mo.z - pyf;
        const float2 dy = make_float2(dys, dys);
        const float2 dx = __fadd2_rn(make_float2(mo.x, mo.y), npx);
        const float2 u = __ffma2_rn(make_float2(k0.x, k0.y), dx, __fmul2_rn(make_float2(k1.x, k1.y), dy));
        const float2 v = __ffma2_rn(make_float2(k0.z, k0.w), dx, __fmul2_rn(make_float2(k1.z, k1.w), dy));
        const float2 power = __fmul2_rn(make_float2(-0.5f, -0.5f), __ffma2_rn(dx, u, __fmul2_rn(dy, v)));
        const bool a0 = power.x <= 0.f && !(T.x < 1e-4f), a1 = power.y <= 0.f && !(T.y < 1e-4f);
        const int pos = __float_as_int(mo.w);
        if (!__any_sync(0xffffffffu, fmaxf(power.x, power.y) >= s_far[jj])) {
          // far field for the whole warp: alpha < 2^-26 at every pixel, so T (1 - alpha) == T
          // exactly and the colour term is below float resolution; only the last-contributor
          // index moves (the reference counts every Gaussian with power <= 0)
          last0 = a0 ? pos : last0;
          last1 = a1 ? pos : last1;
          continue;
        }
        const float4 ow = s_ow[jj];
        const float2 aw = __fmul2_rn(__fmul2_rn(make_float2(ow.x, ow.y), make_float2(expf(power.x), expf(power.y))),
                                     make_float2(ow.z, ow.w));
        const float2 alpha = make_float2(a0 ? fminf(kMaxAlpha, aw.x) : 0.f, a1 ? fminf(kMaxAlpha, aw.y) : 0.f);
        const float2 wt = __fmul2_rn(alpha, T);
        T = __fmul2_rn(T, __fadd2_rn(make_float2(1.f, 1.f), make_float2(-alpha.x, -alpha.y)));
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const float4 col = s_col[c][jj];
          re[c] = __ffma2_rn(wt, make_float2(col.x, col.y), re[c]);
          im[c] = __ffma2_rn(wt, make_float2(col.z, col.w), im[c]);
        }
        last0 = a0 ? pos : last0;
        last1 = a1 ? pos : last1;
      }
    }
    if (rowin) {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        float2* out = field + (size_t)(p * C + c) * HW + pix;
        if (px < W) out[0] = make_float2(re[c].x, im[c].x);
        if (px + 1 < W) out[1] = make_float2(re[c].y, im[c].y);
      }
      if (px < W) {
        final_T[p * HW + pix] = T.x;
        n_contrib[p * HW + pix] = last0;
      }
      if (px + 1 < W) {
        final_T[p * HW + pix + 1] = T.y;
        n_contrib[p * HW + pix + 1] = last1;
      }
    }
    __syncthreads();   // s_* are restaged by the next plane
  }
}

int launch_render(int K, int C, dim3 grid, cudaStream_t st, const int2* ranges, const int32_t* pl, const GeomWs& g,
                  const float* pp, int W, int H, int gx, float2* field, float* fT, int32_t* nc, const int32_t* order) {
  switch (C) {
    case 1: render_forward_kernel<1><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
    case 2: render_forward_kernel<2><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
    default: render_forward_kernel<3><<<grid, 128, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
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
  (void)N;
  if (num_pairs < 0 || W < 1 || H < 1) return 0;
  const int T = ((W + kTile - 1) / kTile) * ((H + kTile - 1) / kTile);
  return carve_bin(nullptr, (size_t)-1, num_pairs, T).bytes + 256;
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
  const Camera cam = make_camera(s);
  const int T = cam.grid_x * cam.grid_y;
  BinWs b = carve_bin(bin_ws, bin_bytes, num_pairs, T);
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  clear_ranges_kernel<<<(T + 255) / 256, 256, 0, st>>>((int2*)ranges, T);
  CVHRF_LAUNCH_CHECK();
  if (num_pairs > 0) {
    emit_pairs_kernel<<<(s.N + 255) / 256, 256, 0, st>>>(g, cam, s.N, b, (uint32_t)num_pairs, nullptr);
    CVHRF_LAUNCH_CHECK();
    int alt = 0;
    if ((rc = radix_sort_pairs(b.tkey, b.slot, b.tkey_alt, b.slot_alt, num_pairs, 0, tile_bits(T), b.scratch, st,
                               &alt, nullptr, nullptr, true)))
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
  tile_order_kernel<<<1, 1024, 0, st>>>((const int2*)ranges, T, b.tile_order);
  CVHRF_LAUNCH_CHECK();
  dim3 grid(T);
  const int2* rg = (const int2*)ranges;
  float2* f = (float2*)field;
  return launch_render(s.K, s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts,
                       n_contrib, b.tile_order);
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
  const Camera cam = make_camera(s);
  const int T = cam.grid_x * cam.grid_y;
  BinWs b = carve_bin(bin_ws, bin_bytes, num_pairs, T);
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
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
                               &alt, nullptr, b.eff, true)))
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
  tile_order_kernel<<<1, 1024, 0, st>>>((const int2*)ranges, T, b.tile_order);
  CVHRF_LAUNCH_CHECK();
  dim3 grid(T);
  const int2* rg = (const int2*)ranges;
  float2* f = (float2*)field;
  return launch_render(s.K, s.C, grid, st, rg, point_list, g, s.plane_probs, s.W, s.H, cam.grid_x, f, final_Ts,
                       n_contrib, b.tile_order);
}
