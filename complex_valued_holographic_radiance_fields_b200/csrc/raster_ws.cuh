// Workspace layouts shared by the rasterizer forward and backward.
#pragma once
#include "common.cuh"
#include "raster_geometry.cuh"
#include "scan_sort.cuh"

namespace cvhrf {

// Per-Gaussian state, written by the forward geometry phase and read again by the
// render and backward phases (the reference keeps the equivalent on a process-wide
// singleton, rasterizer_splat.cu:395-398; here it lives in the caller's workspace).
struct GeomWs {
  float2* means2d;     // N
  float4* cov2d;       // N   (with the +0.3 of add_diagonal_offset_kernel)
  float4* rec0;        // N   (mean.x, mean.y, opacity, 0)
  float4* conic;       // N   (inv00, inv01, inv10, inv11) as renderTileKernel computes them
  float2* cp;          // N*C (colour * cos(phase), colour * sin(phase))
  int* radii;          // N
  uint32_t* tiles;     // N   tiles touched
  uint32_t* key;       // N   depth key (sorted in place)
  uint32_t* order;     // N   Gaussian index in depth order (sorted in place)
  uint32_t* key_alt;   // N   ping-pong
  uint32_t* order_alt; // N
  uint32_t* offsets;   // N   inclusive scan of tiles in depth order
  uint32_t* vis;       // N   visibility flag, then its inclusive scan
  uint32_t* scratch;   // scan / sort scratch
  int* sorted;         // 1: depth keys already in order (the depth sort is skipped)
  size_t bytes;
};

inline GeomWs carve_geom(void* base, size_t cap, int N, int C) {
  Carver cv(base, cap);
  GeomWs g;
  g.means2d = cv.take<float2>(N);
  g.cov2d = cv.take<float4>(N);
  g.rec0 = cv.take<float4>(N);
  g.conic = cv.take<float4>(N);
  g.cp = cv.take<float2>((size_t)N * C);
  g.radii = cv.take<int>(N);
  g.tiles = cv.take<uint32_t>(N);
  g.key = cv.take<uint32_t>(N);
  g.order = cv.take<uint32_t>(N);
  g.key_alt = cv.take<uint32_t>(N);
  g.order_alt = cv.take<uint32_t>(N);
  g.offsets = cv.take<uint32_t>(N);
  g.vis = cv.take<uint32_t>(N);
  const size_t sw = sort_scratch_words(N) > scan_scratch_words(N) ? sort_scratch_words(N) : scan_scratch_words(N);
  g.scratch = cv.take<uint32_t>(sw);
  g.sorted = cv.take<int>(1);
  g.bytes = cv.overflow ? 0 : cv.used;
  return g;
}

// Per-pair state of the binning phase.
struct BinWs {
  uint32_t* tkey;      // pairs: tile id (sorted)
  uint32_t* slot;      // pairs: emission slot (sorted) -> per-pair gradient record index
  uint32_t* tkey_alt;
  uint32_t* slot_alt;
  uint32_t* gauss;     // pairs: Gaussian index of each emission slot
  uint32_t* scratch;
  int32_t* eff;        // capacity mode: pair count if it fits the capacity, else 0
  int32_t* tile_order; // tiles by decreasing list length: the render kernels' block -> tile map
  size_t bytes;
};

inline BinWs carve_bin(void* base, size_t cap, int pairs, int tiles) {
  Carver cv(base, cap);
  const int n = pairs > 0 ? pairs : 1;
  BinWs b;
  b.tkey = cv.take<uint32_t>(n);
  b.slot = cv.take<uint32_t>(n);
  b.tkey_alt = cv.take<uint32_t>(n);
  b.slot_alt = cv.take<uint32_t>(n);
  b.gauss = cv.take<uint32_t>(n);
  b.scratch = cv.take<uint32_t>(sort_scratch_words(n));
  b.eff = cv.take<int32_t>(1);
  b.tile_order = cv.take<int32_t>(tiles > 0 ? tiles : 1);
  b.bytes = cv.overflow ? 0 : cv.used;
  return b;
}

inline Camera make_camera(const cvhrf_raster_scene& s) {
  Camera c;
  c.fx = s.fx;
  c.fy = s.fy;
  c.px = s.px;
  c.py = s.py;
  c.near_plane = s.near_plane;
  c.far_plane = s.far_plane;
  c.half_tan_fov_x = 0.5f * s.W / s.fx;
  c.half_tan_fov_y = 0.5f * s.H / s.fy;
  c.W = s.W;
  c.H = s.H;
  c.grid_x = (s.W + kTile - 1) / kTile;
  c.grid_y = (s.H + kTile - 1) / kTile;
  return c;
}

inline bool scene_ok(const cvhrf_raster_scene* s) {
  return s && s->N >= 0 && s->K >= 1 && s->K <= kMaxPlanes && s->C >= 1 && s->C <= kMaxChannels && s->W >= 1 &&
         s->H >= 1 && (s->N == 0 || (s->cam_means && s->z_vals && s->quats && s->scales && s->colours && s->phase &&
                                     s->opacities && s->plane_probs && s->view_matrix));
}

// Bits needed for tile ids 0..T-1 (getHigherMsb of rasterizer_splat.cu:25-38 gives an
// upper bound of the same sort range; any range covering all ids sorts identically).
inline int tile_bits(int T) {
  int b = 0;
  while ((1 << b) < T) ++b;
  return b < 1 ? 1 : b;
}

}  // namespace cvhrf
