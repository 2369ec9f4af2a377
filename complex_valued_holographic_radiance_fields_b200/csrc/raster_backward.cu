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
// Record layout (6 + K + 2C floats, padded to a multiple of 4 so records are float4
// aligned): dmean.x, dmean.y, dcov_xx, dcov_xy, dcov_yy, dopacity, dplane[K], dcolour[C],
// dphase[C].
#include "raster_ws.cuh"

namespace cvhrf {

#ifdef CVHRF_BWD_STATS
// debugging counters (not built into the library): kept Gaussians, warp iterations,
// active warp iterations, candidate pixels, contributing pixels
__device__ unsigned long long g_bwd_stats[8];
#endif

namespace {

constexpr int kRedV = 12;  // length of the per-Gaussian vector that is reduced

// floats per (tile, Gaussian) record: 6 + K + 2C rounded up to a multiple of 4
__host__ __device__ __forceinline__ int record_stride(int K, int C) { return (6 + K + 2 * C + 3) & ~3; }

// Sum v[0..11] over the warp (reduce-scatter: each exchange hands half of a lane's live
// sums to its partner).  Afterwards the total of index 3i + j (i < 4, j < 3) is held by
// lane 8i + {0, 4, 2}[j] (reduce12_slot gives the index a lane holds, or -1).  13 shuffles
// for 12 sums.
__device__ __forceinline__ float warp_reduce_scatter12(float (&v)[kRedV]) {
  const int lane = threadIdx.x & 31;
  {  // 12 -> 6
    const bool hi = lane & 16;
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      const float send = hi ? v[i] : v[i + 6];
      const float keep = hi ? v[i + 6] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {  // 6 -> 3
    const bool hi = lane & 8;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float send = hi ? v[i] : v[i + 3];
      const float keep = hi ? v[i + 3] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  // lane (bits 4, 3 = b) now holds sums 6 b4 + 3 b3 + (0..2) over its 8-lane group
  {  // 3 -> 2 (the third sum rides along)
    const bool hi = lane & 4;
    const float send = hi ? v[0] : v[1];
    const float keep = hi ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    v[2] += __shfl_xor_sync(0xffffffffu, v[2], 4);
  }
  {  // 2 -> 1
    const bool hi = lane & 2;
    const float send = hi ? v[0] : v[2];
    const float keep = hi ? v[2] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}
__device__ __forceinline__ int reduce12_slot(int lane) {
  if ((lane & 1) || (lane & 6) == 6) return -1;
  const int j = (lane & 2) ? 2 : ((lane & 4) ? 1 : 0);
  return 3 * (lane >> 3) + j;
}

// Per-Gaussian constants of the backward pixel loop, computed once per batch with the
// reference's expressions (backward_splat.cu:194-206, 283-292), plus a conservative
// bounding box of the region where alpha >= 1/255 can hold (outside it the reference
// `continue`s, :218).
struct BwdG {
  float mx, my, opacity, ex;      // mean, opacity, box half-width
  float cx, cy, cz, ey;           // conic_x, conic_y, conic_z, box half-height
  float A, B, Cc, D;              // d cov / d conic coefficients
  float E, G;
  float tau;                      // ln(255 opacity w): alpha >= 1/255 needs power >= -tau
};

// Per-thread state of one plane's back-to-front replay for a horizontal pixel pair
// (backward_splat.cu:133-148), packed per component: .x = left pixel, .y = right pixel.
// The reference keeps the colour accumulated behind the current Gaussian, acc_c, and
// uses it only in dL/dalpha = sum_c (cp_c - acc_c) . dL_c (real dot product of the
// complex components).  Only Q = sum_c acc_c . dL_c is therefore kept: with
// P = sum_c cp_c . dL_c, dL/dalpha = P - Q and the update acc_c' = alpha cp_c +
// (1 - alpha) acc_c becomes Q' = alpha P + (1 - alpha) Q.  (The reference applies the
// update lazily at the next contributor; applying it right away gives the same values.)
template <int C>
struct PairState {
  float2 T;                       // transmittance
  int last0, last1;               // n_contrib: positions >= last are skipped
  float2 dre[C], dim[C];          // dL/dpixel (real, imaginary)
  float2 Q;                       // sum_c acc_c . dL_c
};

// Number of per-pixel sums reduced over the CTA for one Gaussian.  The reference's
// per-pixel gradient terms (backward_splat.cu:236-300) are linear in
//   gd = G dL/dalpha   (dL/dalpha already scaled by T)   and   dch = alpha T
// times quantities that are either per-pixel (offset d, dL) or per-Gaussian, so the CTA
// reduces
//   S0 = sum gd, S1 = sum gd dx, S2 = sum gd dy, S3 = sum gd dx dx, S4 = sum gd dx dy,
//   S5 = sum gd dy dy, X_c = sum dch re(dL_c), Y_c = sum dch im(dL_c)
// and applies the per-Gaussian factors once per (tile, Gaussian): with ow = opacity w,
//   dmean = -ddel * ow (conic . (S1, S2)),  dconic = -0.5 ow (S3, S4, S5),
//   dopacity = w S0,  dplane = opacity S0,
//   dcolour_c = cos X_c + sin Y_c,  dphase_c = -im(cp_c) X_c + re(cp_c) Y_c.
template <int C>
constexpr int red_len() { return 6 + 2 * C; }

// One pixel pair, one Gaussian: renderBackwardTileKernel's per-pixel arithmetic
// (:184-300) for both pixels at once; r[] receives the pair's share of the sums above.
// A pixel that does not contribute (masked, power > 0, alpha < 1/255) gets alpha = 0 and
// gd = 0, which leaves its state unchanged exactly (T / 1, 0 P + 1 Q) and adds exact zeros.
// power = -0.5 (conic_x dx^2 + conic_z dy^2) - conic_y dx dy for the pixel pair
__device__ __forceinline__ float2 pair_power(const float4 con, float2 dx, float dy) {
  const float2 cx2 = make_float2(con.x, con.x);
  const float czdd = con.z * dy * dy;
  const float ncydy = -(con.y * dy);
  const float2 quad = __ffma2_rn(__fmul2_rn(cx2, dx), dx, make_float2(czdd, czdd));
  return __ffma2_rn(make_float2(-0.5f, -0.5f), quad, __fmul2_rn(make_float2(ncydy, ncydy), dx));
}

template <int C>
__device__ __forceinline__ void bwd_pair(PairState<C>& st, const float4 con, float w, float2 dx, float dy,
                                         float2 power, bool n0, bool n1, const float2* cpx, float* r) {
  // con = (conic_x, conic_y, conic_z, opacity); power = pair_power(con, dx, dy)
  const float2 dy2 = make_float2(dy, dy);
  // __expf: the gradients are compared at 1e-4, and ex2.approx is within a few ulp
  const float2 G = make_float2(__expf(power.x), __expf(power.y));
  const float2 aw = __fmul2_rn(__fmul2_rn(make_float2(con.w, con.w), G), make_float2(w, w));
  const float al0 = fminf(0.99f, aw.x), al1 = fminf(0.99f, aw.y);
  const bool a0 = n0 && power.x <= 0.0f && al0 >= 1.0f / 255.0f;
  const bool a1 = n1 && power.y <= 0.0f && al1 >= 1.0f / 255.0f;
#ifdef CVHRF_BWD_STATS
  {
    const unsigned cand = __popc(__ballot_sync(0xffffffffu, n0)) + __popc(__ballot_sync(0xffffffffu, n1));
    const unsigned act = __popc(__ballot_sync(0xffffffffu, a0)) + __popc(__ballot_sync(0xffffffffu, a1));
    if ((threadIdx.x & 31) == 0) {
      atomicAdd(&g_bwd_stats[3], (unsigned long long)cand);
      atomicAdd(&g_bwd_stats[4], (unsigned long long)act);
    }
  }
#endif
  const float2 al = make_float2(a0 ? al0 : 0.f, a1 ? al1 : 0.f);
  const float2 om = make_float2(1.0f - al.x, 1.0f - al.y);
  st.T = make_float2(__fdividef(st.T.x, om.x), __fdividef(st.T.y, om.y));
  const float2 dch = __fmul2_rn(al, st.T);
  float2 P = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    P = __ffma2_rn(make_float2(cpx[c].x, cpx[c].x), st.dre[c], P);
    P = __ffma2_rn(make_float2(cpx[c].y, cpx[c].y), st.dim[c], P);
    const float2 X = __fmul2_rn(dch, st.dre[c]), Y = __fmul2_rn(dch, st.dim[c]);
    r[6 + c] = X.x + X.y;
    r[6 + C + c] = Y.x + Y.y;
  }
  const float2 dLda = __fmul2_rn(__fadd2_rn(P, make_float2(-st.Q.x, -st.Q.y)), st.T);
  st.Q = __ffma2_rn(al, P, __fmul2_rn(om, st.Q));
  const float2 gd = make_float2(a0 ? G.x * dLda.x : 0.f, a1 ? G.y * dLda.y : 0.f);
  const float2 gdx = __fmul2_rn(gd, dx), gdy = __fmul2_rn(gd, dy2);
  const float2 gdxx = __fmul2_rn(gdx, dx), gdxy = __fmul2_rn(gdx, dy2), gdyy = __fmul2_rn(gdy, dy2);
  r[0] = gd.x + gd.y;
  r[1] = gdx.x + gdx.y;
  r[2] = gdy.x + gdy.y;
  r[3] = gdxx.x + gdxx.y;
  r[4] = gdxy.x + gdxy.y;
  r[5] = gdyy.x + gdyy.y;
}

// One CTA per 16x16 tile, 128 threads x 2 horizontally adjacent pixels (each warp an 8 x 8
// quadrant, which keeps the per-warp footprint test tight), one pass per
// plane.  Each pass stages the tile list back to front in batches, keeps only the
// Gaussians that can contribute on this plane inside this tile (plane weight >= 1e-6,
// alpha >= 1/255 box meets the tile, position below the tile's largest n_contrib), and
// for each of those reduces the per-pixel sums over the CTA and adds the pair's share
// into its record (records start at zero; each pass adds its plane's share).
template <int C>
__global__ void __launch_bounds__(128, 6) render_backward_kernel(
    const int2* __restrict__ ranges, const int32_t* __restrict__ point_list, const uint32_t* __restrict__ slot_sorted,
    const float4* __restrict__ rec0, const float4* __restrict__ cov2d, const float* __restrict__ colours,
    const float* __restrict__ phase, const float* __restrict__ plane_probs, const float* __restrict__ final_T,
    const int32_t* __restrict__ n_contrib, const float2* __restrict__ grad_field, int K, int W, int H, int gx,
    float* __restrict__ records, const int32_t* __restrict__ tile_order) {
  constexpr int NB = 128, NW = 4, RL = red_len<C>(), RP = RL;
  static_assert(RL <= 12, "reduction vector too long");
  __shared__ uint32_t s_slot[NB];
  __shared__ float4 s_geo[NB];      // (mean x, mean y, box half-width, box half-height): the footprint test
  __shared__ float4 s_wq[NB];       // (plane weight, list position, -ln(255 opacity weight), Gaussian) (ints as bits)
  __shared__ float4 s_con[NB];      // (conic x, conic y, conic z, opacity): the pixel arithmetic
  __shared__ float4 s_coefA[NB];    // (A, B, Cc, D) and
  __shared__ float2 s_coefB[NB];    // (E, G): d cov / d conic, used once per (tile, Gaussian)
  __shared__ float2 s_cpx[C][NB];   // colour * e^{i phase}
  __shared__ float s_part[NW][NB][RP];
  __shared__ int s_wcnt[NW];
  __shared__ int s_maxlast;

  const int VR = record_stride(K, C);
  const int tile = tile_order[blockIdx.x];
  const int tx = tile % gx, ty = tile / gx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int px = tx * kTile + (warp & 1) * 8 + (lane & 3) * 2, py = ty * kTile + (warp >> 1) * 8 + (lane >> 2);
  const bool in0 = px < W && py < H, in1 = px + 1 < W && py < H;
  const float2 npx = make_float2(-(float)px, -(float)(px + 1));
  const float pyf = (float)py;
  const int2 range = ranges[tile];
  const int n = range.y - range.x;
  if (n <= 0) return;
  const size_t HW = (size_t)H * W;
  const size_t pix0 = in0 ? (size_t)py * W + px : 0, pix1 = in1 ? (size_t)py * W + px + 1 : 0;
  const float ddelx_dx = 0.5f * W, ddely_dy = 0.5f * H;
  const float tx0 = (float)(tx * kTile), tx1 = (float)(tx * kTile + kTile - 1);
  const float ty0 = (float)(ty * kTile), ty1 = (float)(ty * kTile + kTile - 1);
  const unsigned lt = (1u << lane) - 1u;
  const int slot12 = reduce12_slot(lane);

  for (int p = 0; p < K; ++p) {
    PairState<C> st;
    st.T = make_float2(in0 ? final_T[p * HW + pix0] : 0.f, in1 ? final_T[p * HW + pix1] : 0.f);
    st.last0 = in0 ? n_contrib[p * HW + pix0] : 0;
    st.last1 = in1 ? n_contrib[p * HW + pix1] : 0;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const float2 g0 = in0 ? grad_field[(size_t)(p * C + c) * HW + pix0] : make_float2(0.f, 0.f);
      const float2 g1 = in1 ? grad_field[(size_t)(p * C + c) * HW + pix1] : make_float2(0.f, 0.f);
      st.dre[c] = make_float2(g0.x, g1.x);
      st.dim[c] = make_float2(g0.y, g1.y);
    }
    st.Q = make_float2(0.f, 0.f);
    __syncthreads();
    if (threadIdx.x == 0) s_maxlast = 0;
    __syncthreads();
    atomicMax(&s_maxlast, max(st.last0, st.last1));
    __syncthreads();
    const int n_eff = min(n, s_maxlast);

    for (int end = n_eff; end > 0; end -= NB) {
      const int cnt = min(NB, end);
      // ---- stage and compact this batch (order kept: back to front) ----
      bool keep = false;
      BwdG g;
      float w = 0.f;
      int gi = 0, pos = 0;
      if ((int)threadIdx.x < cnt) {
        pos = end - 1 - threadIdx.x;
        gi = point_list[range.x + pos];
        w = plane_probs[gi * K + p];
        if (w >= kPlaneCutoff) {
          const float4 r0 = rec0[gi];
          const float4 cov = cov2d[gi];
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
          // alpha >= 1/255 needs d^T conic d <= 2 ln(255 opacity w): padded box of that ellipse
          const float tau = logf(255.0f * r0.z * w);
          g.tau = tau;
          const float t2 = 2.0f * fmaxf(tau, 0.0f) * 1.01f;
          g.ex = sqrtf(t2 * fabsf(cov.x)) * 1.01f + 0.05f;
          g.ey = sqrtf(t2 * fabsf(cov.w)) * 1.01f + 0.05f;
          keep = det != 0.0f && tau > 0.0f && g.mx + g.ex >= tx0 && g.mx - g.ex <= tx1 && g.my + g.ey >= ty0 &&
                 g.my - g.ey <= ty1;
        }
      }
      const unsigned bal = __ballot_sync(0xffffffffu, keep);
      __syncthreads();  // previous batch fully consumed
      if (lane == 0) s_wcnt[warp] = __popc(bal);
      __syncthreads();
      int off = 0, total = 0;
#pragma unroll
      for (int w2 = 0; w2 < NW; ++w2) {
        off += w2 < warp ? s_wcnt[w2] : 0;
        total += s_wcnt[w2];
      }
      if (keep) {
        const int idx = off + __popc(bal & lt);
        s_slot[idx] = slot_sorted[range.x + pos];
        s_geo[idx] = make_float4(g.mx, g.my, g.ex, g.ey);
        s_wq[idx] = make_float4(w, __int_as_float(pos), -g.tau - 1e-3f, __int_as_float(gi));
        s_con[idx] = make_float4(g.cx, g.cy, g.cz, g.opacity);
        s_coefA[idx] = make_float4(g.A, g.B, g.Cc, g.D);
        s_coefB[idx] = make_float2(g.E, g.G);
#pragma unroll
        for (int c = 0; c < C; ++c) {
          float sn, cs;
          __sincosf(phase[gi * C + c], &sn, &cs);
          const float col = colours[gi * C + c];
          s_cpx[c][idx] = make_float2(col * cs, col * sn);
        }
      }
      __syncthreads();
      // ---- each warp replays all kept Gaussians over its 8 x 8 pixels ----
#ifdef CVHRF_BWD_STATS
      if (threadIdx.x == 0) atomicAdd(&g_bwd_stats[0], (unsigned long long)total);
      if (lane == 0) atomicAdd(&g_bwd_stats[1], (unsigned long long)total);
#endif
      for (int jj = 0; jj < total; ++jj) {
        const float4 geo = s_geo[jj];
        const float4 wq = s_wq[jj];
        const int q = __float_as_int(wq.y);
        const float2 dx = __fadd2_rn(make_float2(geo.x, geo.x), npx);
        const float dy = geo.y - pyf;
        const bool ny = fabsf(dy) <= geo.w;
        const bool n0 = in0 && q < st.last0 && ny && fabsf(dx.x) <= geo.z;
        const bool n1 = in1 && q < st.last1 && ny && fabsf(dx.y) <= geo.z;
        if (!__any_sync(0xffffffffu, n0 || n1)) {
          if (lane < RL) s_part[warp][jj][lane] = 0.f;
          continue;
        }
        // second, exact-footprint vote: alpha >= 1/255 needs power >= -ln(255 opacity w);
        // the bound carries a 1e-3 margin, so no contributing pixel is dropped (the exact
        // test is bwd_pair's)
        const float4 con = s_con[jj];
        const float2 power = pair_power(con, dx, dy);
        const bool c0 = n0 && power.x >= wq.z && power.x <= 0.0f;
        const bool c1 = n1 && power.y >= wq.z && power.y <= 0.0f;
        if (!__any_sync(0xffffffffu, c0 || c1)) {
          if (lane < RL) s_part[warp][jj][lane] = 0.f;
          continue;
        }
#ifdef CVHRF_BWD_STATS
        if (lane == 0) atomicAdd(&g_bwd_stats[2], 1ull);
#endif
        float v[kRedV];
        float2 cpx[C];
#pragma unroll
        for (int c = 0; c < C; ++c) cpx[c] = s_cpx[c][jj];
        bwd_pair<C>(st, con, wq.x, dx, dy, power, c0, c1, cpx, v);
#pragma unroll
        for (int i = RL; i < 12; ++i) v[i] = 0.f;
        const float tot = warp_reduce_scatter12(v);
        if (slot12 >= 0 && slot12 < RL) s_part[warp][jj][slot12] = tot;
      }
      __syncthreads();
      // ---- the pair's record share: the warps' sums, per-Gaussian factors applied once ----
      const int VO = 7 + 2 * C;
      for (int e = threadIdx.x; e < total * VO; e += blockDim.x) {
        const int j = e / VO, idx = e - j * VO;
        float S[RL];
#pragma unroll
        for (int k = 0; k < 6; ++k) S[k] = s_part[0][j][k] + s_part[1][j][k] + s_part[2][j][k] + s_part[3][j][k];
        const float4 con = s_con[j];
        const float4 ca = s_coefA[j];
        const float2 cb = s_coefB[j];
        const float ww = s_wq[j].x;
        const float ow = con.w * ww;
        float val;
        if (idx == 0) val = -ddelx_dx * ow * (con.x * S[1] + con.y * S[2]);
        else if (idx == 1) val = -ddely_dy * ow * (con.z * S[2] + con.y * S[1]);
        else if (idx <= 4) {
          const float dcx = -0.5f * ow * S[3], dcy = -0.5f * ow * S[4], dcz = -0.5f * ow * S[5];
          val = idx == 2 ? dcx * ca.x + dcz * ca.y
              : idx == 3 ? dcx * ca.z + dcy * ca.w + dcz * cb.x
                         : dcx * ca.y + dcz * cb.y;
        } else if (idx == 5) val = ww * S[0];
        else if (idx == 6) val = con.w * S[0];
        else {
          const int c = idx < 7 + C ? idx - 7 : idx - 7 - C;
          const float X = s_part[0][j][6 + c] + s_part[1][j][6 + c] + s_part[2][j][6 + c] + s_part[3][j][6 + c];
          const float Y = s_part[0][j][6 + C + c] + s_part[1][j][6 + C + c] + s_part[2][j][6 + C + c] +
                          s_part[3][j][6 + C + c];
          if (idx < 7 + C) {
            // cos / sin of the phase recomputed here (same call as at staging) instead of kept
            float sn, cs;
            __sincosf(phase[__float_as_int(s_wq[j].w) * C + c], &sn, &cs);
            val = cs * X + sn * Y;
          } else {
            const float2 cp = s_cpx[c][j];
            val = -cp.y * X + cp.x * Y;
          }
        }
        const int ri = idx < 6 ? idx : (idx == 6 ? 6 + p : 6 + K + (idx - 7));
        // a reduction without return (red.global.add): the record's earlier planes were
        // added batches ago by this block, so the order of additions is the plane order
        atomicAdd(records + (size_t)s_slot[j] * VR + ri, val);
      }
    }
  }
}

// One CTA per 128 consecutive Gaussians (depth order).  Phase 1 sums each Gaussian's
// contiguous records with coalesced loads (a half-warp per Gaussian when a record has
// <= 16 floats, a warp otherwise; lane = record component).  Phase 2: one thread per
// Gaussian chains the sums through the projection.
constexpr int kGradBlock = 128;    // Gaussians per CTA
constexpr int kGradThreads = 128;  // threads per CTA: 32 half-warps sum the records, 128 threads chain
constexpr int kRecMax = (6 + kMaxPlanes + 2 * kMaxChannels + 3) & ~3;

__global__ void __launch_bounds__(kGradThreads) gaussian_grad_kernel(cvhrf_raster_scene s, Camera cam, GeomWs g,
                                                                   const float* __restrict__ records, float* gcam,
                                                                   float* gz, float* gq, float* gs, float* gcol,
                                                                   float* gph, float* gop, float* gpl,
                                                                   uint32_t max_slot) {
  __shared__ float s_r[kGradBlock][kRecMax + 1];
  const int K = s.K, C = s.C, VR = record_stride(K, C);
  const int s0 = blockIdx.x * kGradBlock;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // 8 lanes per Gaussian, lane q sums components 4q .. 4q + 3 with float4 loads
  const int sub = lane >> 3, q = lane & 7;
  for (int lg = warp * 4 + sub; lg < kGradBlock; lg += (kGradThreads / 32) * 4) {
    const int si = s0 + lg;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (si < s.N && 4 * q < VR) {
      // records exist for slots < max_slot (the pair capacity in capacity mode)
      const uint32_t a = min(si == 0 ? 0u : g.offsets[si - 1], max_slot), b = min(g.offsets[si], max_slot);
      const float4* rec = reinterpret_cast<const float4*>(records + (size_t)a * VR) + q;
      const int step = VR >> 2;
#pragma unroll 4
      for (uint32_t k = a; k < b; ++k, rec += step) {
        const float4 v = *rec;
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
    }
    if (4 * q < VR) {
      s_r[lg][4 * q] = acc.x;
      s_r[lg][4 * q + 1] = acc.y;
      s_r[lg][4 * q + 2] = acc.z;
      s_r[lg][4 * q + 3] = acc.w;
    }
  }
  __syncthreads();
  const int si = s0 + threadIdx.x;
  if (threadIdx.x >= kGradBlock || si >= s.N) return;
  const float* r = s_r[threadIdx.x];
  const uint32_t gi = g.order[si];
  const uint32_t a = min(si == 0 ? 0u : g.offsets[si - 1], max_slot), b = min(g.offsets[si], max_slot);
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

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

#ifdef CVHRF_BWD_STATS
extern "C" void cvhrf_debug_bwd_stats(unsigned long long* out) {
  cudaMemcpyFromSymbol(out, g_bwd_stats, sizeof(g_bwd_stats));
  const unsigned long long z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  cudaMemcpyToSymbol(g_bwd_stats, z, sizeof(z));
}
#endif

extern "C" size_t cvhrf_raster_backward_workspace_bytes(int num_pairs, int K, int C) {
  if (num_pairs < 0 || K < 1 || C < 1) return 0;
  const size_t n = num_pairs > 0 ? num_pairs : 1;
  return align_up(n * record_stride(K, C) * sizeof(float), 256);
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
  BinWs b = carve_bin(const_cast<void*>(bin_ws), bin_bytes, num_pairs,
                      ((s.W + kTile - 1) / kTile) * ((s.H + kTile - 1) / kTile));
  if (b.bytes == 0 || !bin_ws) return CVHRF_EWORKSPACE;
  if (!bwd_ws || bwd_bytes < cvhrf_raster_backward_workspace_bytes(num_pairs, s.K, s.C)) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const Camera cam = make_camera(s);
  float* rec = (float*)bwd_ws;
  if (num_pairs > 0) {
    const int T = cam.grid_x * cam.grid_y;
    dim3 grid(T);
    const int32_t* pl = point_list;
    CVHRF_CUDA_TRY(cudaMemsetAsync(rec, 0, (size_t)num_pairs * record_stride(s.K, s.C) * sizeof(float), st));
    const int2* rg = (const int2*)ranges;
    const float2* gf = (const float2*)grad_field;
    // six 37 KB CTAs per SM need the full shared-memory carve-out (set once, before any capture)
    static const bool carve = [] {
      cudaFuncSetAttribute(render_backward_kernel<1>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      cudaFuncSetAttribute(render_backward_kernel<2>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      cudaFuncSetAttribute(render_backward_kernel<3>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
      return true;
    }();
    (void)carve;
#define CVHRF_BWD(CC)                                                                                       \
  render_backward_kernel<CC><<<grid, 128, 0, st>>>(rg, pl, b.slot, g.rec0, g.cov2d, s.colours, s.phase,      \
                                                   s.plane_probs, final_Ts, n_contrib, gf, s.K, s.W, s.H,    \
                                                   cam.grid_x, rec, b.tile_order)
    switch (s.C) {
      case 1: CVHRF_BWD(1); break;
      case 2: CVHRF_BWD(2); break;
      default: CVHRF_BWD(3); break;
    }
#undef CVHRF_BWD
    CVHRF_LAUNCH_CHECK();
  }
  gaussian_grad_kernel<<<(s.N + kGradBlock - 1) / kGradBlock, kGradThreads, 0, st>>>(s, cam, g, rec, grad_cam_means, grad_z_vals, grad_quats,
                                                          grad_scales, grad_colours, grad_phase, grad_opacities,
                                                          grad_plane_probs, (uint32_t)num_pairs);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

