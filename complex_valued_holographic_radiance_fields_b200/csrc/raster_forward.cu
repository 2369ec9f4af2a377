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

// One CTA of 64 threads per 16x16 tile; each thread owns four horizontally adjacent
// pixels as two packed f32x2 pairs (sm_100 FFMA2/FMUL2/FADD2; every lane of a packed
// operation is an ordinary IEEE-rounded float operation).  The planes are composited
// one after another: for plane p the CTA walks the tile's depth-ordered list in batches
// of 128, keeps (ballot compaction, order preserved) only the Gaussians whose plane-p
// weight is >= the cutoff, and front-to-back blends them.  Per pixel this is exactly the
// reference's chain: power = -0.5 (dx (i00 dx + i10 dy) + dy (i01 dx + i11 dy)),
// skip if power > 0, G = expf(power), alpha = min(0.99, (o G) w), the pixel takes
// colour * alpha * T, T' = T (1 - alpha), last = 1-based list position, and stops once
// T' < 1e-4.  "Stopped" is the same as T < 1e-4 (T starts at 1 and changes only
// through a contribution), so a stopped or off-image pixel just gets alpha = 0: then
// T (1 - 0) == T and acc + 0 * c == acc exactly.  A plane ends early when every pixel
// of the tile has stopped in it.
// ln(2^-26) - 0.1: with power < kFarLog - ln(opacity w), alpha = min(0.99, opacity expf(power) w)
// stays below 2^-26 even with expf's rounding, so 1 - alpha rounds to 1.0f
constexpr float kFarLog = -18.0218f - 0.1f;

template <int C>
__global__ void __launch_bounds__(64) render_forward_kernel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const float4* __restrict__ rec0,
    const float4* __restrict__ conic, const float2* __restrict__ cp, const float* __restrict__ plane_probs, int K,
    int W, int H, int gx, float2* __restrict__ field, float* __restrict__ final_T, int32_t* __restrict__ n_contrib,
    const int32_t* __restrict__ tile_order) {
  constexpr int NT = 64, NB = 128;
  __shared__ float4 s_mo[NB];      // (mx, mx, my, list position)
  __shared__ float4 s_c0[NB];      // (i00, i00, i01, i01)
  __shared__ float4 s_c1[NB];      // (i10, i10, i11, i11)
  __shared__ float4 s_ow[NB];      // (o, o, w, w)
  __shared__ float s_far[NB];      // power below which alpha < 2^-26 (see the far-field skip)
  __shared__ float4 s_col[C][NB];  // (re, re, im, im)
  __shared__ int s_cnt[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tile = tile_order ? tile_order[blockIdx.x] : (int)blockIdx.x;
  const int tx = tile % gx, ty = tile / gx;
  const int px = tx * kTile + (tid & 3) * 4, py = ty * kTile + (tid >> 2);
  const bool rowin = py < H;
  const float2 npxA = make_float2(-(float)px, -(float)(px + 1));
  const float2 npxB = make_float2(-(float)(px + 2), -(float)(px + 3));
  const float pyf = (float)py;
  const int2 range = ranges[tile];
  const int n = range.y - range.x;
  const size_t HW = (size_t)H * W, pix = (size_t)py * W + px;

  for (int p = 0; p < K; ++p) {
    // off-image pixels start "stopped" (T = 0 < 1e-4) and are never written
    float2 TA = make_float2(rowin && px < W ? 1.f : 0.f, rowin && px + 1 < W ? 1.f : 0.f);
    float2 TB = make_float2(rowin && px + 2 < W ? 1.f : 0.f, rowin && px + 3 < W ? 1.f : 0.f);
    int lA0 = 0, lA1 = 0, lB0 = 0, lB1 = 0;
    float2 reA[C], imA[C], reB[C], imB[C];
#pragma unroll
    for (int c = 0; c < C; ++c) reA[c] = imA[c] = reB[c] = imB[c] = make_float2(0.f, 0.f);

    for (int base = 0; base < n; base += NB) {
      const bool mine_done = TA.x < 1e-4f && TA.y < 1e-4f && TB.x < 1e-4f && TB.y < 1e-4f;
      if (__syncthreads_and(mine_done)) break;
      // stage: keep this batch's plane-p Gaussians, in list order
      int gi[2];
      bool keep[2];
      unsigned bal[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int j = base + r * NT + tid;
        keep[r] = false;
        gi[r] = 0;
        if (j < n) {
          gi[r] = point_list[range.x + j];
          keep[r] = plane_probs[(size_t)gi[r] * K + p] >= kPlaneCutoff;
        }
        bal[r] = __ballot_sync(0xffffffffu, keep[r]);
        if (lane == 0) s_cnt[r * 2 + warp] = __popc(bal[r]);
      }
      __syncthreads();
      const int c0 = s_cnt[0], c1 = s_cnt[1], c2 = s_cnt[2], c3 = s_cnt[3];
      const unsigned lt = (1u << lane) - 1u;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        if (keep[r]) {
          const int seg = r * 2 + warp;
          const int off = (seg > 0 ? c0 : 0) + (seg > 1 ? c1 : 0) + (seg > 2 ? c2 : 0) + __popc(bal[r] & lt);
          const int g = gi[r];
          const float4 r0 = rec0[g];
          const float4 cn = conic[g];
          const float w = plane_probs[(size_t)g * K + p];
          s_mo[off] = make_float4(r0.x, r0.x, r0.y, __int_as_float(base + r * NT + tid + 1));
          s_c0[off] = make_float4(cn.x, cn.x, cn.y, cn.y);
          s_c1[off] = make_float4(cn.z, cn.z, cn.w, cn.w);
          s_ow[off] = make_float4(r0.z, r0.z, w, w);
          s_far[off] = kFarLog - logf(r0.z * w);
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const float2 v = cp[(size_t)g * C + c];
            s_col[c][off] = make_float4(v.x, v.x, v.y, v.y);
          }
        }
      }
      __syncthreads();
      const int cnt = c0 + c1 + c2 + c3;
      // a warp whose 128 pixels have all stopped skips the batch (it only adds exact zeros)
      if (__all_sync(0xffffffffu, mine_done)) continue;
      for (int jj = 0; jj < cnt; ++jj) {
        if ((jj & 31) == 31 && __all_sync(0xffffffffu, TA.x < 1e-4f && TA.y < 1e-4f && TB.x < 1e-4f && TB.y < 1e-4f))
          break;
        const float4 mo = s_mo[jj];
        const float4 k0 = s_c0[jj], k1 = s_c1[jj];
        const float2 mx = make_float2(mo.x, mo.y);
        const float dys = mo.z - pyf;
        const float2 dy = make_float2(dys, dys);
        const float2 t1 = __fmul2_rn(make_float2(k1.x, k1.y), dy);
        const float2 t2 = __fmul2_rn(make_float2(k1.z, k1.w), dy);
        const float2 dxA = __fadd2_rn(mx, npxA), dxB = __fadd2_rn(mx, npxB);
        const float2 uA = __ffma2_rn(make_float2(k0.x, k0.y), dxA, t1);
        const float2 vA = __ffma2_rn(make_float2(k0.z, k0.w), dxA, t2);
        const float2 uB = __ffma2_rn(make_float2(k0.x, k0.y), dxB, t1);
        const float2 vB = __ffma2_rn(make_float2(k0.z, k0.w), dxB, t2);
        const float2 nh = make_float2(-0.5f, -0.5f);
        const float2 pA = __fmul2_rn(nh, __ffma2_rn(dxA, uA, __fmul2_rn(dy, vA)));
        const float2 pB = __fmul2_rn(nh, __ffma2_rn(dxB, uB, __fmul2_rn(dy, vB)));
        const bool aA0 = pA.x <= 0.f && !(TA.x < 1e-4f), aA1 = pA.y <= 0.f && !(TA.y < 1e-4f);
        const bool aB0 = pB.x <= 0.f && !(TB.x < 1e-4f), aB1 = pB.y <= 0.f && !(TB.y < 1e-4f);
        if (!__any_sync(0xffffffffu, fmaxf(fmaxf(pA.x, pA.y), fmaxf(pB.x, pB.y)) >= s_far[jj])) {
          // far field for the whole warp: alpha < 2^-26 at every pixel, so T (1 - alpha) == T
          // exactly and the colour term is below float resolution; only the last-contributor
          // index moves (the reference counts every Gaussian with power <= 0)
          const int pos = __float_as_int(mo.w);
          lA0 = aA0 ? pos : lA0;
          lA1 = aA1 ? pos : lA1;
          lB0 = aB0 ? pos : lB0;
          lB1 = aB1 ? pos : lB1;
          continue;
        }
        const float4 ow = s_ow[jj];
        const float2 o2 = make_float2(ow.x, ow.y), w2 = make_float2(ow.z, ow.w);
        const float2 awA = __fmul2_rn(__fmul2_rn(o2, make_float2(expf(pA.x), expf(pA.y))), w2);
        const float2 awB = __fmul2_rn(__fmul2_rn(o2, make_float2(expf(pB.x), expf(pB.y))), w2);
        const float2 alA = make_float2(aA0 ? fminf(kMaxAlpha, awA.x) : 0.f, aA1 ? fminf(kMaxAlpha, awA.y) : 0.f);
        const float2 alB = make_float2(aB0 ? fminf(kMaxAlpha, awB.x) : 0.f, aB1 ? fminf(kMaxAlpha, awB.y) : 0.f);
        const float2 one = make_float2(1.f, 1.f);
        const float2 wtA = __fmul2_rn(alA, TA), wtB = __fmul2_rn(alB, TB);
        TA = __fmul2_rn(TA, __fadd2_rn(one, make_float2(-alA.x, -alA.y)));
        TB = __fmul2_rn(TB, __fadd2_rn(one, make_float2(-alB.x, -alB.y)));
#pragma unroll
        for (int c = 0; c < C; ++c) {
          const float4 col = s_col[c][jj];
          const float2 cr = make_float2(col.x, col.y), ci = make_float2(col.z, col.w);
          reA[c] = __ffma2_rn(wtA, cr, reA[c]);
          imA[c] = __ffma2_rn(wtA, ci, imA[c]);
          reB[c] = __ffma2_rn(wtB, cr, reB[c]);
          imB[c] = __ffma2_rn(wtB, ci, imB[c]);
        }
        const int pos = __float_as_int(mo.w);
        lA0 = aA0 ? pos : lA0;
        lA1 = aA1 ? pos : lA1;
        lB0 = aB0 ? pos : lB0;
        lB1 = aB1 ? pos : lB1;
      }
    }
    if (rowin) {
      const float Tv[4] = {TA.x, TA.y, TB.x, TB.y};
      const int lv[4] = {lA0, lA1, lB0, lB1};
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const float re[4] = {reA[c].x, reA[c].y, reB[c].x, reB[c].y};
        const float im[4] = {imA[c].x, imA[c].y, imB[c].x, imB[c].y};
        float2* out = field + (size_t)(p * C + c) * HW + pix;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (px + q < W) out[q] = make_float2(re[q], im[q]);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (px + q < W) {
          final_T[p * HW + pix + q] = Tv[q];
          n_contrib[p * HW + pix + q] = lv[q];
        }
      }
    }
    __syncthreads();   // s_* are restaged by the next plane
  }
}

int launch_render(int K, int C, dim3 grid, cudaStream_t st, const int2* ranges, const int32_t* pl, const GeomWs& g,
                  const float* pp, int W, int H, int gx, float2* field, float* fT, int32_t* nc, const int32_t* order) {
  switch (C) {
    case 1: render_forward_kernel<1><<<grid, 64, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
    case 2: render_forward_kernel<2><<<grid, 64, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
    default: render_forward_kernel<3><<<grid, 64, 0, st>>>(ranges, pl, g.rec0, g.conic, g.cp, pp, K, W, H, gx, field, fT, nc, order); break;
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
