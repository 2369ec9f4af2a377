/*
 * CPU restatement of the reference wave rasterizer (forward + backward).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libcvhrf's rasterizer kernels and the
 * timed CPU baseline of bench.py.  Scalar C, one thread, float32 arithmetic with no
 * FMA contraction (built with -ffp-contract=off); tile loops run on OpenMP threads, so values agree with the GPU to
 * rounding, not bit for bit; integer outputs (pair list, ranges) agree exactly
 * unless a radius or tile bound lands within one ulp of an integer.
 *
 * Follows, function by function (paths inside the reference project):
 *   geometry      cuda_prop/cov3d_cuda/wave_rasterizer/forward.cu:10-61 (cov3d, GLM
 *                 products), :64-122 (Jacobian, 1.3x fov clamp), :221-294 (cov2D =
 *                 J W Sigma W^T J^T + 0.3 I), :297-330 (2D means)
 *   visibility    rasterizer_splat.cu:42-62 + auxiliary.h:196-221, with the intended
 *                 camera-space depth (the reference reads a 3x3 matrix as 4x4)
 *   preprocess    forward_splat.cu:17-98 (radius from Sigma2D + 0.3 again), getRect
 *                 auxiliary.h:95-112
 *   binning       rasterizer_splat.cu:114-201 (keys = tile << 32 | depth bits with the
 *                 sign bit set, stable radix sort, tile ranges)
 *   render        forward_splat.cu:101-289 (front to back, one pass per plane,
 *                 n_contrib = 1-based position of the last contributor); every pixel
 *                 of an edge tile sees the whole list (the reference leaves part of
 *                 its shared-memory batch unloaded there)
 *   backward      backward_splat.cu:78-307 (back to front replay, alpha < 1/255
 *                 skipped, dmean scaled by 0.5 W / 0.5 H) and backward.cu:78-497
 *                 (cov2d / Jacobian / cov3d / means2d backward)
 */
#include <math.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TILE 16
#define PLANE_CUTOFF 1e-6f
#define MAX_ALPHA 0.99f

typedef struct {
  int N, K, C, W, H;
  float fx, fy, px, py, near_plane, far_plane;
  const float *cam, *z, *quats, *scales, *colours, *phase, *opac, *planes, *view;
} Scene;

static void means2d(const Scene* s, int i, float* m) {
  const float x = s->cam[3 * i], y = s->cam[3 * i + 1], z = s->cam[3 * i + 2];
  if (z <= s->near_plane || z >= s->far_plane) { m[0] = m[1] = 1e6f; return; }
  const float inv_z = 1.0f / z;
  m[0] = s->fx * (-x * inv_z) + s->px;
  m[1] = s->fy * (-y * inv_z) + s->py;
}

static void jacobian(const Scene* s, int i, float* J) {
  const float tx = s->cam[3 * i], ty = s->cam[3 * i + 1], tz = s->cam[3 * i + 2];
  memset(J, 0, 6 * sizeof(float));
  if (tz <= s->near_plane || tz >= s->far_plane) return;
  const float tz2 = tz * tz;
  const float lim_x = 1.3f * (0.5f * s->W / s->fx), lim_y = 1.3f * (0.5f * s->H / s->fy);
  const float cx = fminf(fmaxf(tx / tz, -lim_x), lim_x) * tz;
  const float cy = fminf(fmaxf(ty / tz, -lim_y), lim_y) * tz;
  J[0] = s->fx / tz;
  J[2] = -(s->fx * cx) / tz2;
  J[4] = s->fy / tz;
  J[5] = -(s->fy * cy) / tz2;
}

/* GLM column-major M[col][row] */
static void glm_mul(float A[3][3], float B[3][3], float O[3][3]) {
  for (int c = 0; c < 3; ++c)
    for (int r = 0; r < 3; ++r) O[c][r] = A[0][r] * B[c][0] + A[1][r] * B[c][1] + A[2][r] * B[c][2];
}

static void quat_rot(const float* q, float* rr, float R[3][3]) {
  float r = q[0], x = q[1], y = q[2], z = q[3];
  const float n = sqrtf(r * r + x * x + y * y + z * z);
  r /= n; x /= n; y /= n; z /= n;
  rr[0] = r; rr[1] = x; rr[2] = y; rr[3] = z;
  R[0][0] = 1.f - 2.f * (y * y + z * z); R[0][1] = 2.f * (x * y - r * z); R[0][2] = 2.f * (x * z + r * y);
  R[1][0] = 2.f * (x * y + r * z); R[1][1] = 1.f - 2.f * (x * x + z * z); R[1][2] = 2.f * (y * z - r * x);
  R[2][0] = 2.f * (x * z - r * y); R[2][1] = 2.f * (y * z + r * x); R[2][2] = 1.f - 2.f * (x * x + y * y);
}

static void cov3d(const float* q, const float* sc, float* out) {
  float R[3][3], rr[4], S[3][3] = {{sc[0], 0, 0}, {0, sc[1], 0}, {0, 0, sc[2]}}, SR[3][3], SRt[3][3], Sg[3][3];
  quat_rot(q, rr, R);
  glm_mul(S, R, SR);
  for (int c = 0; c < 3; ++c)
    for (int r = 0; r < 3; ++r) SRt[c][r] = SR[r][c];
  glm_mul(SRt, SR, Sg);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) out[i * 3 + j] = Sg[i][j];
}

static void matmul(const float* A, const float* B, float* O, int n, int k, int m) {
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < m; ++j) {
      float a = 0.f;
      for (int t = 0; t < k; ++t) a += A[i * k + t] * B[t * m + j];
      O[i * m + j] = a;
    }
}
static void transpose(const float* A, float* O, int n, int m) {
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < m; ++j) O[j * n + i] = A[i * m + j];
}

static void cov2d(const Scene* s, int i, float* c, float* J, float* Sig, float* JW) {
  float B[6], Cm[6], Wt[9], Jt[6];
  jacobian(s, i, J);
  cov3d(s->quats + 4 * i, s->scales + 3 * i, Sig);
  matmul(J, s->view, JW, 2, 3, 3);
  matmul(JW, Sig, B, 2, 3, 3);
  transpose(s->view, Wt, 3, 3);
  matmul(B, Wt, Cm, 2, 3, 3);
  transpose(J, Jt, 2, 3);
  matmul(Cm, Jt, c, 2, 3, 2);
  c[0] += 0.3f;
  c[3] += 0.3f;
}

static int splat_radius(const float* cov) {
  float cx = cov[0], cy = cov[1], cz = cov[2], cw = cov[3];
  float det = cx * cw - cy * cz;
  if (fabsf(det) < 1e-10f) return 0;
  cx += 0.3f; cw += 0.3f;
  det = cx * cw - cy * cz;
  if (fabsf(det) < 1e-8f) return 0;
  const float mid = 0.5f * (cx + cw);
  const float disc = fmaxf(0.1f, mid * mid - det);
  const float l1 = mid + sqrtf(disc), l2 = mid - sqrtf(disc);
  const float r = ceilf(3.0f * sqrtf(fmaxf(l1, l2)));
  return r != r ? 0 : (int)r;
}

static uint32_t f2u_sat(float v) { return (v != v || v <= 0.f) ? 0u : (v >= 4294967040.f ? 0xFFFFFFFFu : (uint32_t)v); }

static void tile_rect(const float* p, int maxr, int gx, int gy, uint32_t* r) {
  const int radius = maxr > 1 ? maxr : 1;
  uint32_t x0 = f2u_sat((p[0] - radius) / TILE), y0 = f2u_sat((p[1] - radius) / TILE);
  uint32_t x1 = f2u_sat((p[0] + radius + TILE - 1) / TILE), y1 = f2u_sat((p[1] + radius + TILE - 1) / TILE);
  x0 = x0 < (uint32_t)gx - 1 ? x0 : (uint32_t)gx - 1;
  y0 = y0 < (uint32_t)gy - 1 ? y0 : (uint32_t)gy - 1;
  x1 = x1 > 1 ? x1 : 1; x1 = x1 < (uint32_t)gx ? x1 : (uint32_t)gx;
  y1 = y1 > 1 ? y1 : 1; y1 = y1 < (uint32_t)gy ? y1 : (uint32_t)gy;
  if (x1 <= x0) x1 = x0 + 1 < (uint32_t)gx ? x0 + 1 : (uint32_t)gx;
  if (y1 <= y0) y1 = y0 + 1 < (uint32_t)gy ? y0 + 1 : (uint32_t)gy;
  r[0] = x0; r[1] = y0; r[2] = x1; r[3] = y1;
}

typedef struct { uint64_t key; uint32_t val; uint32_t seq; } Pair;
static int cmp_pair(const void* a, const void* b) {
  const Pair *p = (const Pair*)a, *q = (const Pair*)b;
  if (p->key != q->key) return p->key < q->key ? -1 : 1;
  return p->seq < q->seq ? -1 : (p->seq > q->seq);
}

/* Forward.  field: K*C*H*W*2 floats (re, im).  Returns the number of pairs, or
 * -(needed) if point_list_cap is too small (nothing else is then valid). */
int ora_raster_forward(int N, int K, int C, int W, int H, float fx, float fy, float px, float py, float near_plane,
                       float far_plane, const float* cam, const float* z, const float* quats, const float* scales,
                       const float* colours, const float* phase, const float* opac, const float* planes,
                       const float* view, float* field, float* final_T, int32_t* n_contrib, int32_t* point_list,
                       int point_list_cap, int32_t* ranges, uint8_t* visible, float* means_out, float* cov_out) {
  Scene s = {N, K, C, W, H, fx, fy, px, py, near_plane, far_plane, cam, z, quats, scales, colours, phase, opac, planes, view};
  const int gx = (W + TILE - 1) / TILE, gy = (H + TILE - 1) / TILE, T = gx * gy;
  float* m2 = (float*)malloc(sizeof(float) * 2 * (N + 1));
  float* cv = (float*)malloc(sizeof(float) * 4 * (N + 1));
  int* rad = (int*)malloc(sizeof(int) * (N + 1));
  long total = 0;
#pragma omp parallel for reduction(+ : total) schedule(static)
  for (int i = 0; i < N; ++i) {
    const float zc = cam[3 * i + 2];
    visible[i] = (zc > 0.2f && zc > near_plane && zc < far_plane);
    float J[6], Sig[9], JW[6];
    means2d(&s, i, m2 + 2 * i);
    cov2d(&s, i, cv + 4 * i, J, Sig, JW);
    rad[i] = 0;
    if (!(z[i] <= near_plane || z[i] >= far_plane)) rad[i] = splat_radius(cv + 4 * i);
    if (rad[i] > 0) {
      uint32_t r[4];
      tile_rect(m2 + 2 * i, rad[i], gx, gy, r);
      total += (long)(r[2] - r[0]) * (r[3] - r[1]);
    }
  }
  if (means_out) memcpy(means_out, m2, sizeof(float) * 2 * N);
  if (cov_out) memcpy(cov_out, cv, sizeof(float) * 4 * N);
  if (total > point_list_cap) { free(m2); free(cv); free(rad); return (int)-total; }
  Pair* pr = (Pair*)malloc(sizeof(Pair) * (total + 1));
  long k = 0;
  for (int i = 0; i < N; ++i) {
    if (rad[i] <= 0) continue;
    uint32_t r[4];
    tile_rect(m2 + 2 * i, rad[i], gx, gy, r);
    uint32_t db;
    memcpy(&db, &z[i], 4);
    db = (db & 0x80000000u) == 0 ? (db | 0x80000000u) : (db & 0x7FFFFFFFu);
    for (uint32_t y = r[1]; y < r[3]; ++y)
      for (uint32_t x = r[0]; x < r[2]; ++x) {
        pr[k].key = ((uint64_t)(y * gx + x) << 32) | db;
        pr[k].val = (uint32_t)i;
        pr[k].seq = (uint32_t)k;
        ++k;
      }
  }
  qsort(pr, total, sizeof(Pair), cmp_pair);  /* (key, emission order): the stable order */
  memset(ranges, 0, sizeof(int32_t) * 2 * T);
  for (long i = 0; i < total; ++i) {
    point_list[i] = (int32_t)pr[i].val;
    const uint32_t t = (uint32_t)(pr[i].key >> 32);
    if (i == 0 || (uint32_t)(pr[i - 1].key >> 32) != t) ranges[2 * t] = (int32_t)i;
    if (i == total - 1 || (uint32_t)(pr[i + 1].key >> 32) != t) ranges[2 * t + 1] = (int32_t)(i + 1);
  }
  free(pr);
  const size_t HW = (size_t)H * W;
  for (size_t i = 0; i < (size_t)K * C * HW * 2; ++i) field[i] = 0.f;
  for (size_t i = 0; i < (size_t)K * HW; ++i) { final_T[i] = 1.f; n_contrib[i] = 0; }
#pragma omp parallel for schedule(dynamic, 4)
  for (int t = 0; t < T; ++t) {
    const int a = ranges[2 * t], b = ranges[2 * t + 1];
    if (b <= a) continue;
    const int tx = t % gx, ty = t / gx;
    for (int py_ = ty * TILE; py_ < ty * TILE + TILE && py_ < H; ++py_)
      for (int px_ = tx * TILE; px_ < tx * TILE + TILE && px_ < W; ++px_) {
        const size_t pix = (size_t)py_ * W + px_;
        for (int p = 0; p < K; ++p) {
          float Tr = 1.f;
          int last = 0;
          float acc[6] = {0, 0, 0, 0, 0, 0};
          for (int j = a; j < b; ++j) {
            const int g = point_list[j];
            if (z[g] <= near_plane || z[g] >= far_plane) continue;
            const float w = planes[g * K + p];
            if (w < PLANE_CUTOFF) continue;
            const float dx = m2[2 * g] - (float)px_, dy = m2[2 * g + 1] - (float)py_;
            const float* c4 = cv + 4 * g;
            const float det = c4[0] * c4[3] - c4[1] * c4[2];
            const float di = 1.0f / det;
            const float i00 = c4[3] * di, i01 = -c4[1] * di, i10 = -c4[2] * di, i11 = c4[0] * di;
            const float power = -0.5f * (dx * (i00 * dx + i10 * dy) + dy * (i01 * dx + i11 * dy));
            if (power > 0.0f) continue;
            const float alpha = fminf(MAX_ALPHA, opac[g] * expf(power) * w);
            const float test_T = Tr * (1.0f - alpha);
            for (int c = 0; c < C; ++c) {
              const float sc = colours[g * C + c] * alpha * Tr;
              acc[2 * c] += sc * cosf(phase[g * C + c]);
              acc[2 * c + 1] += sc * sinf(phase[g * C + c]);
            }
            Tr = test_T;
            last = j - a + 1;
            if (test_T < 0.0001f) break;
          }
          for (int c = 0; c < C; ++c) {
            field[2 * ((p * C + c) * HW + pix)] = acc[2 * c];
            field[2 * ((p * C + c) * HW + pix) + 1] = acc[2 * c + 1];
          }
          final_T[p * HW + pix] = Tr;
          n_contrib[p * HW + pix] = last;
        }
      }
  }
  free(m2); free(cv); free(rad);
  return (int)total;
}

/* Backward.  grad_field: K*C*H*W*2.  Outputs dense gradients (grad_z stays 0). */
void ora_raster_backward(int N, int K, int C, int W, int H, float fx, float fy, float px, float py, float near_plane,
                         float far_plane, const float* cam, const float* z, const float* quats, const float* scales,
                         const float* colours, const float* phase, const float* opac, const float* planes,
                         const float* view, const float* grad_field, const float* final_T, const int32_t* n_contrib,
                         const int32_t* point_list, const int32_t* ranges, float* g_cam, float* g_z, float* g_q,
                         float* g_s, float* g_col, float* g_ph, float* g_op, float* g_pl) {
  Scene s = {N, K, C, W, H, fx, fy, px, py, near_plane, far_plane, cam, z, quats, scales, colours, phase, opac, planes, view};
  const int gx = (W + TILE - 1) / TILE, gy = (H + TILE - 1) / TILE, T = gx * gy;
  float* m2 = (float*)malloc(sizeof(float) * 2 * (N + 1));
  float* cv = (float*)malloc(sizeof(float) * 4 * (N + 1));
  float* gm = (float*)calloc(2 * (size_t)N + 2, sizeof(float));
  float* gc = (float*)calloc(4 * (size_t)N + 4, sizeof(float));
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    float J[6], Sig[9], JW[6];
    means2d(&s, i, m2 + 2 * i);
    cov2d(&s, i, cv + 4 * i, J, Sig, JW);
  }
  memset(g_z, 0, sizeof(float) * N);
  memset(g_col, 0, sizeof(float) * N * C);
  memset(g_ph, 0, sizeof(float) * N * C);
  memset(g_op, 0, sizeof(float) * N);
  memset(g_pl, 0, sizeof(float) * N * K);
  const size_t HW = (size_t)H * W;
#pragma omp parallel for schedule(dynamic, 4)
  for (int t = 0; t < T; ++t) {
    const int a = ranges[2 * t], b = ranges[2 * t + 1];
    if (b <= a) continue;
    const int tx = t % gx, ty = t / gx;
    for (int py_ = ty * TILE; py_ < ty * TILE + TILE && py_ < H; ++py_)
      for (int px_ = tx * TILE; px_ < tx * TILE + TILE && px_ < W; ++px_) {
        const size_t pix = (size_t)py_ * W + px_;
        for (int p = 0; p < K; ++p) {
          float Tr = final_T[p * HW + pix];
          const int lastc = n_contrib[p * HW + pix];
          float acc_re[3] = {0, 0, 0}, acc_im[3] = {0, 0, 0}, lc_re[3] = {0, 0, 0}, lc_im[3] = {0, 0, 0};
          float last_alpha = 0.f;
          for (int j = b - 1; j >= a; --j) {
            if (j - a >= lastc) continue;
            const int g = point_list[j];
            const float pp = planes[g * K + p];
            if (pp < PLANE_CUTOFF) continue;
            const float dx = m2[2 * g] - (float)px_, dy = m2[2 * g + 1] - (float)py_;
            const float* c4 = cv + 4 * g;
            const float det = c4[0] * c4[3] - c4[1] * c4[2];
            if (det == 0.0f) continue;
            const float di = 1.0f / det;
            const float cx = c4[3] * di, cy = -c4[1] * di, cz = c4[0] * di;
            const float power = -0.5f * (cx * dx * dx + cz * dy * dy) - cy * dx * dy;
            if (power > 0.0f) continue;
            const float G = expf(power);
            const float alpha = fminf(0.99f, opac[g] * G * pp);
            if (alpha < 1.0f / 255.0f) continue;
            Tr = Tr / (1.0f - alpha);
            const float dcd = alpha * Tr;
            float dL_dalpha = 0.f;
            for (int c = 0; c < C; ++c) {
              const float col = colours[g * C + c], cs = cosf(phase[g * C + c]), sn = sinf(phase[g * C + c]);
              const float cr = col * cs, ci = col * sn;
              acc_re[c] = last_alpha * lc_re[c] + (1.0f - last_alpha) * acc_re[c];
              acc_im[c] = last_alpha * lc_im[c] + (1.0f - last_alpha) * acc_im[c];
              lc_re[c] = cr; lc_im[c] = ci;
              const float dre = grad_field[2 * ((p * C + c) * HW + pix)], dim = grad_field[2 * ((p * C + c) * HW + pix) + 1];
              dL_dalpha += (cr - acc_re[c]) * dre;
              dL_dalpha += (ci - acc_im[c]) * dim;
              #pragma omp atomic
              g_col[g * C + c] += dcd * (cs * dre + sn * dim);
              #pragma omp atomic
              g_ph[g * C + c] += dcd * col * (-sn * dre + cs * dim);
            }
            dL_dalpha *= Tr;
            last_alpha = alpha;
            const float dL_dG = opac[g] * pp * dL_dalpha;
            const float gdx = G * dx, gdy = G * dy;
            #pragma omp atomic
            gm[2 * g] += dL_dG * (-gdx * cx - gdy * cy) * (0.5f * W);
            #pragma omp atomic
            gm[2 * g + 1] += dL_dG * (-gdy * cz - gdx * cy) * (0.5f * H);
            const float dcx = -0.5f * gdx * dx * dL_dG, dcy = -0.5f * gdx * dy * dL_dG, dcz = -0.5f * gdy * dy * dL_dG;
            const float xx = dcx * (c4[3] * di * di) * c4[3] + dcz * (-c4[1] * di * di) * (-c4[1]);
            const float xy = dcx * (c4[3] * di * di) * (-c4[1]) + dcy * (-di) + dcz * (-c4[1] * di * di) * c4[0];
            const float yy = dcx * (-c4[1] * di * di) * (-c4[1]) + dcz * (c4[0] * di * di) * c4[0];
            #pragma omp atomic
            gc[4 * g] += xx;
            #pragma omp atomic
            gc[4 * g + 1] += xy;
            #pragma omp atomic
            gc[4 * g + 2] += xy;
            #pragma omp atomic
            gc[4 * g + 3] += yy;
            #pragma omp atomic
            g_op[g] += G * pp * dL_dalpha;
            #pragma omp atomic
            g_pl[g * K + p] += opac[g] * G * dL_dalpha;
          }
        }
      }
  }
  /* geometry backward (backward.cu:363-497, backward_splat.cu:364-417) */
#pragma omp parallel for schedule(static)
  for (int i = 0; i < N; ++i) {
    const float x = cam[3 * i], y = cam[3 * i + 1], zz = cam[3 * i + 2];
    float J[6], Sig[9], JW[6], c4[4];
    cov2d(&s, i, c4, J, Sig, JW);
    float dcam[3] = {0, 0, 0};
    const int clip = (zz <= near_plane || zz >= far_plane);
    if (!clip) {
      dcam[0] = -fx * gm[2 * i] / zz;
      dcam[1] = -fy * gm[2 * i + 1] / zz;
      dcam[2] = (fx * x * gm[2 * i] / (zz * zz)) + (fy * y * gm[2 * i + 1] / (zz * zz));
    }
    float G2[4] = {gc[4 * i], gc[4 * i + 1], gc[4 * i + 2], gc[4 * i + 3]};
    float dC[6], dB[6], GJW[6], JWt[6], dS[9], St[9], dA[6], dJ[6], Wt[9];
    matmul(G2, J, dC, 2, 2, 3);
    matmul(dC, view, dB, 2, 3, 3);
    matmul(G2, JW, GJW, 2, 2, 3);
    transpose(JW, JWt, 2, 3);
    matmul(JWt, GJW, dS, 3, 2, 3);
    transpose(Sig, St, 3, 3);
    matmul(dB, St, dA, 2, 3, 3);
    transpose(view, Wt, 3, 3);
    matmul(dA, Wt, dJ, 2, 3, 3);
    if (!clip) {
      const float tz2 = zz * zz, tz3 = tz2 * zz;
      const float lim_x = 1.3f * (0.5f * W / fx), lim_y = 1.3f * (0.5f * H / fy);
      const float xm = (x / zz < -lim_x || x / zz > lim_x) ? 0.f : 1.f;
      const float ym = (y / zz < -lim_y || y / zz > lim_y) ? 0.f : 1.f;
      dcam[0] += dJ[2] * (xm * (-fx / tz2));
      dcam[1] += dJ[5] * (ym * (-fy / tz2));
      dcam[2] += dJ[0] * (-fx / tz2) + dJ[2] * (xm * (2.0f * fx * x / tz3)) + dJ[4] * (-fy / tz2) +
                 dJ[5] * (ym * (2.0f * fy * y / tz3));
    }
    g_cam[3 * i] = dcam[0]; g_cam[3 * i + 1] = dcam[1]; g_cam[3 * i + 2] = dcam[2];
    /* cov3d backward */
    float Gm[3][3], R[3][3], rr[4], Rt[3][3], T1[3][3], T2[3][3];
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) Gm[a][b] = dS[a * 3 + b];
    quat_rot(quats + 4 * i, rr, R);
    const float r = rr[0], qx = rr[1], qy = rr[2], qz = rr[3];
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) Rt[a][b] = 2.0f * R[b][a];
    glm_mul(Rt, Gm, T1);
    glm_mul(T1, R, T2);
    const float* sc = scales + 3 * i;
    g_s[3 * i] = T2[0][0] * sc[0]; g_s[3 * i + 1] = T2[1][1] * sc[1]; g_s[3 * i + 2] = T2[2][2] * sc[2];
    float dR[4][3][3] = {
        {{0.f, -2.f * qz, 2.f * qy}, {2.f * qz, 0.f, -2.f * qx}, {-2.f * qy, 2.f * qx, 0.f}},
        {{0.f, 2.f * qy, 2.f * qz}, {2.f * qy, -4.f * qx, -2.f * r}, {2.f * qz, 2.f * r, -4.f * qx}},
        {{-4.f * qy, 2.f * qx, 2.f * r}, {2.f * qx, 0.f, 2.f * qz}, {-2.f * r, 2.f * qz, -4.f * qy}},
        {{-4.f * qz, -2.f * r, 2.f * qx}, {2.f * r, -4.f * qz, 2.f * qy}, {2.f * qx, 2.f * qy, 0.f}}};
    for (int q = 0; q < 4; ++q) {
      float acc = 0.f;
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b)
          acc += Gm[a][b] * ((sc[a] * dR[q][b][a]) * (sc[b] * R[a][b]) + (sc[a] * R[b][a]) * (sc[b] * dR[q][a][b]));
      g_q[4 * i + q] = acc;
    }
  }
  free(m2); free(cv); free(gm); free(gc);
}

int ora_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Fused sparse Adam restatement (conv.cu:1200-1228): rows `visible`, grad dense. */
void ora_sparse_adam(float* p, const float* g, float* m, float* v, int N, int D, const int64_t* visible, int V,
                     float lr, float b1, float b2, float eps) {
  (void)N;
  for (int i = 0; i < V; ++i)
    for (int d = 0; d < D; ++d) {
      const size_t k = (size_t)visible[i] * D + d;
      m[k] = b1 * m[k] + (1.0f - b1) * g[k];
      v[k] = b2 * v[k] + (1.0f - b2) * g[k] * g[k];
      p[k] += -lr * m[k] / (sqrtf(v[k]) + eps);
    }
}
