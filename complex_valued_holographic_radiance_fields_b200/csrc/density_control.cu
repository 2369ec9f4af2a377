// Adaptive density control (clone / split / prune) and opacity regularisation of the
// Gaussian set, on the device.  Replaces Gaussians.density_control (model.py:626-1047)
// and Gaussians.opacity_regularization (model.py:1049-1077).
//
// The reference builds boolean masks, gathers every parameter and gradient tensor once
// per category (keep / clone / split-1 / split-2; about 60 gathers and 14 concatenations)
// and synchronises on each mask count.  Here the whole pass is four launches:
//   1. classify: one thread per row writes three 0/1 flags into a 3N u32 array laid out
//      [keep(N) | clone(N) | split(N)];
//   2. one inclusive scan over the 3N flags.  Because the output order is
//      [kept rows | clones | split children 1 | split children 2], the scanned value at
//      a set flag is already the row's 1-based output position: keep at scan[i],
//      clone at scan[N+i] (= kept total + clone rank), first split child at scan[2N+i];
//      the second child sits n_split rows after the first;
//   3. a one-thread kernel turns the scan totals into the four counts;
//   4. apply: one thread per source row writes its 0-3 output rows with their gradients.
// Only the host's read of the counts (to size the output) synchronises.
#include <math.h>
#include "common.cuh"
#include "scan_sort.cuh"

namespace cvhrf {
namespace {

constexpr int kThreads = 256;

struct DensityArgs {
  cvhrf_gaussian_set in;
  cvhrf_density_params p;
};

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// grad_mag and avg_scale of model.py:656-659: |grad_means| and the mean of exp(scales).
__device__ __forceinline__ void row_stats(const cvhrf_gaussian_set& s, long long i, float& gx, float& gy, float& gz,
                                         float& gmag, float& avg) {
  gx = s.grad_means[3 * i];
  gy = s.grad_means[3 * i + 1];
  gz = s.grad_means[3 * i + 2];
  gmag = sqrtf(gx * gx + gy * gy + gz * gz);
  const float e0 = expf(s.pre_scales[3 * i]), e1 = expf(s.pre_scales[3 * i + 1]), e2 = expf(s.pre_scales[3 * i + 2]);
  avg = (e0 + e1 + e2) / 3.0f;
}

// model.py:665-672.
__global__ void __launch_bounds__(kThreads) density_classify_kernel(DensityArgs a, uint32_t* __restrict__ flags) {
  const long long N = a.in.N;
  const long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i >= N) return;
  float gx, gy, gz, gmag, avg;
  row_stats(a.in, i, gx, gy, gz, gmag, avg);
  const bool keep = !(sigmoid_f(a.in.pre_opac[i]) < a.p.opacity_threshold);
  const bool large_grad = gmag >= a.p.grad_threshold;
  flags[i] = keep;
  flags[N + i] = keep && large_grad && avg < a.p.small_scale_threshold;
  flags[2 * N + i] = keep && large_grad && avg > a.p.large_scale_threshold;
}

__global__ void density_counts_kernel(const uint32_t* __restrict__ scan, long long N, uint32_t* __restrict__ counts) {
  const uint32_t k = scan[N - 1], kc = scan[2 * N - 1], kcs = scan[3 * N - 1];
  counts[0] = k;
  counts[1] = kc - k;
  counts[2] = kcs - kc;
  counts[3] = (uint32_t)N - k;
}

__device__ __forceinline__ void copy_row(const float* __restrict__ src, float* __restrict__ dst, long long i,
                                         long long o, int D, float scale) {
#pragma unroll 4
  for (int d = 0; d < D; ++d) dst[o * D + d] = src[i * D + d] * scale;
}
// Gradient row: zeros when the source gradient is absent (model.py:715-718, :778-786).
__device__ __forceinline__ void copy_grad_row(const float* __restrict__ src, float* __restrict__ dst, long long i,
                                              long long o, int D, float scale) {
  if (src) copy_row(src, dst, i, o, D, scale);
  else
    for (int d = 0; d < D; ++d) dst[o * D + d] = 0.0f;
}

// Every parameter and gradient of row i copied to output row o (gradients times gscale).
__device__ __forceinline__ void copy_all(const cvhrf_gaussian_set& s, const cvhrf_gaussian_set& t, long long i,
                                         long long o, float gscale) {
  copy_row(s.means, t.means, i, o, 3, 1.0f);
  copy_row(s.pre_quats, t.pre_quats, i, o, 4, 1.0f);
  copy_row(s.pre_scales, t.pre_scales, i, o, 3, 1.0f);
  copy_row(s.colours, t.colours, i, o, s.C, 1.0f);
  copy_row(s.pre_phase, t.pre_phase, i, o, s.C, 1.0f);
  t.pre_opac[o] = s.pre_opac[i];
  copy_row(s.pre_planes, t.pre_planes, i, o, s.K, 1.0f);
  copy_row(s.grad_means, t.grad_means, i, o, 3, gscale);
  copy_row(s.grad_pre_quats, t.grad_pre_quats, i, o, 4, gscale);
  copy_row(s.grad_pre_scales, t.grad_pre_scales, i, o, 3, gscale);
  copy_row(s.grad_colours, t.grad_colours, i, o, s.C, gscale);
  copy_row(s.grad_pre_phase, t.grad_pre_phase, i, o, s.C, gscale);
  copy_grad_row(s.grad_pre_opac, t.grad_pre_opac, i, o, 1, gscale);
  copy_grad_row(s.grad_pre_planes, t.grad_pre_planes, i, o, s.K, gscale);
}

__global__ void __launch_bounds__(kThreads) density_apply_kernel(DensityArgs a, cvhrf_gaussian_set out,
                                                                 const uint32_t* __restrict__ scan,
                                                                 const float* __restrict__ noise, float log_split) {
  const cvhrf_gaussian_set& s = a.in;
  const long long N = s.N;
  const long long i = (long long)blockIdx.x * kThreads + threadIdx.x;
  if (i >= N) return;
  const uint32_t k_i = scan[i], c_i = scan[N + i], s_i = scan[2 * N + i];
  const uint32_t keep = k_i - (i > 0 ? scan[i - 1] : 0u);
  const uint32_t clone = c_i - scan[N + i - 1];
  const uint32_t split = s_i - scan[2 * N + i - 1];
  if (!keep) return;  // clone and split imply keep
  copy_all(s, out, i, (long long)k_i - 1, 1.0f);
  if (!clone && !split) return;

  float gx, gy, gz, gmag, avg;
  row_stats(s, i, gx, gy, gz, gmag, avg);
  if (clone) {
    // model.py:749-772: opacity correction 1 - sqrt(1 - o), offset along the gradient.
    const long long o = (long long)c_i - 1;
    copy_all(s, out, i, o, 1.0f);
    const float op = sigmoid_f(s.pre_opac[i]);
    const float c = 1.0f - sqrtf(1.0f - op);
    const float eps = 1e-6f;
    out.pre_opac[o] = logf(c / (1.0f - c + eps) + eps);
    const float nrm = fmaxf(gmag, 1e-8f);
    const float f = a.p.clone_offset_factor;
    out.means[3 * o] = s.means[3 * i] + f * gx / nrm;
    out.means[3 * o + 1] = s.means[3 * i + 1] + f * gy / nrm;
    out.means[3 * o + 2] = s.means[3 * i + 2] + f * gz / nrm;
  }
  if (split) {
    // model.py:868-910: children at means +/- R(q) (noise * stdev), scales / split_factor,
    // same orientation, colour, phase, opacity and plane logits; gradients halved.
    const long long n_split = (long long)scan[3 * N - 1] - scan[2 * N - 1];
    const long long r = (long long)s_i - 1 - scan[2 * N - 1];
    const long long o1 = (long long)s_i - 1, o2 = o1 + n_split;
    copy_all(s, out, i, o1, 0.5f);
    copy_all(s, out, i, o2, 0.5f);
    // F.normalize (q / max(|q|, 1e-12)) then the unit-quaternion rotation matrix with
    // real part first, two_s = 2 / |q|^2 (the standard quaternion-to-matrix formula).
    float qr = s.pre_quats[4 * i], qi = s.pre_quats[4 * i + 1], qj = s.pre_quats[4 * i + 2],
          qk = s.pre_quats[4 * i + 3];
    const float qn = fmaxf(sqrtf(qr * qr + qi * qi + qj * qj + qk * qk), 1e-12f);
    qr /= qn; qi /= qn; qj /= qn; qk /= qn;
    const float ts = 2.0f / (qr * qr + qi * qi + qj * qj + qk * qk);
    const float R00 = 1.0f - ts * (qj * qj + qk * qk), R01 = ts * (qi * qj - qk * qr), R02 = ts * (qi * qk + qj * qr);
    const float R10 = ts * (qi * qj + qk * qr), R11 = 1.0f - ts * (qi * qi + qk * qk), R12 = ts * (qj * qk - qi * qr);
    const float R20 = ts * (qi * qk - qj * qr), R21 = ts * (qj * qk + qi * qr), R22 = 1.0f - ts * (qi * qi + qj * qj);
    const float sd = avg * 0.5f;
    const float n0 = noise[3 * r] * sd, n1 = noise[3 * r + 1] * sd, n2 = noise[3 * r + 2] * sd;
    const float d0 = R00 * n0 + R01 * n1 + R02 * n2;
    const float d1 = R10 * n0 + R11 * n1 + R12 * n2;
    const float d2 = R20 * n0 + R21 * n1 + R22 * n2;
    const float m0 = s.means[3 * i], m1 = s.means[3 * i + 1], m2 = s.means[3 * i + 2];
    out.means[3 * o1] = m0 + d0;
    out.means[3 * o1 + 1] = m1 + d1;
    out.means[3 * o1 + 2] = m2 + d2;
    out.means[3 * o2] = m0 - d0;
    out.means[3 * o2 + 1] = m1 - d1;
    out.means[3 * o2 + 2] = m2 - d2;
    for (int d = 0; d < 3; ++d) {
      const float v = s.pre_scales[3 * i + d] - log_split;
      out.pre_scales[3 * o1 + d] = v;
      out.pre_scales[3 * o2 + d] = v;
    }
  }
}

// model.py:1063-1071.
__global__ void __launch_bounds__(kThreads) opacity_reg_kernel(float* __restrict__ pre_opac, int N, float amount,
                                                               uint32_t* __restrict__ affected) {
  const int i = blockIdx.x * kThreads + threadIdx.x;
  uint32_t hit = 0;
  if (i < N) {
    const float o = sigmoid_f(pre_opac[i]);
    const float den = fmaxf(o * (1.0f - o), 1e-6f);
    pre_opac[i] = pre_opac[i] - amount / den;
    hit = o > amount;
  }
  const uint32_t w = __popc(__ballot_sync(0xffffffffu, hit));
  if ((threadIdx.x & 31) == 0 && w) atomicAdd(affected, w);
}

bool set_ok(const cvhrf_gaussian_set* s, bool need_all_grads) {
  if (!s || s->N < 0 || s->K < 1 || s->C < 1) return false;
  if (s->N == 0) return true;
  if (!s->means || !s->pre_quats || !s->pre_scales || !s->colours || !s->pre_phase || !s->pre_opac ||
      !s->pre_planes || !s->grad_means || !s->grad_pre_quats || !s->grad_pre_scales || !s->grad_colours ||
      !s->grad_pre_phase)
    return false;
  if (need_all_grads && (!s->grad_pre_opac || !s->grad_pre_planes)) return false;
  return true;
}

struct DensityWs {
  uint32_t* flags;
  uint32_t* scratch;
};
DensityWs carve(void* ws, size_t bytes, long long N, bool& ok) {
  Carver c(ws, bytes);
  DensityWs w;
  w.flags = c.take<uint32_t>((size_t)(3 * N));
  w.scratch = c.take<uint32_t>(scan_scratch_words((int)(3 * N)));
  ok = !c.overflow;
  return w;
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" size_t cvhrf_density_workspace_bytes(int N) {
  if (N < 0 || 3LL * N >= (1LL << 30)) return 0;
  Carver c(nullptr, ~(size_t)0);
  c.take<uint32_t>((size_t)3 * N);
  c.take<uint32_t>(scan_scratch_words(3 * N));
  return c.used;
}

extern "C" int cvhrf_density_classify(const cvhrf_gaussian_set* in, const cvhrf_density_params* params,
                                      void* workspace, size_t workspace_bytes, uint32_t* counts, void* stream) {
  if (!set_ok(in, false) || !params || !counts || 3LL * in->N >= (1LL << 30)) return CVHRF_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  const long long N = in->N;
  if (N == 0) {
    CVHRF_CUDA_TRY(cudaMemsetAsync(counts, 0, 4 * sizeof(uint32_t), st));
    return CVHRF_OK;
  }
  if (!workspace) return CVHRF_EINVAL;
  bool ok;
  DensityWs w = carve(workspace, workspace_bytes, N, ok);
  if (!ok) return CVHRF_EWORKSPACE;
  DensityArgs a{*in, *params};
  density_classify_kernel<<<(unsigned)((N + kThreads - 1) / kThreads), kThreads, 0, st>>>(a, w.flags);
  CVHRF_LAUNCH_CHECK();
  int rc = inclusive_scan_u32(w.flags, w.flags, (int)(3 * N), w.scratch, st);
  if (rc != CVHRF_OK) return rc;
  density_counts_kernel<<<1, 1, 0, st>>>(w.flags, N, counts);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_density_apply(const cvhrf_gaussian_set* in, const cvhrf_density_params* params,
                                   const float* noise, const void* workspace, size_t workspace_bytes,
                                   const cvhrf_gaussian_set* out, void* stream) {
  if (!set_ok(in, false) || !params || !set_ok(out, true) || out->K != in->K || out->C != in->C ||
      3LL * in->N >= (1LL << 30) || !(params->split_factor > 0.0f))
    return CVHRF_EINVAL;
  const long long N = in->N;
  if (N == 0 || out->N == 0) return CVHRF_OK;
  if (!workspace || !noise) return CVHRF_EINVAL;
  bool ok;
  DensityWs w = carve(const_cast<void*>(workspace), workspace_bytes, N, ok);
  if (!ok) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  DensityArgs a{*in, *params};
  const float log_split = (float)log((double)params->split_factor);
  density_apply_kernel<<<(unsigned)((N + kThreads - 1) / kThreads), kThreads, 0, st>>>(a, *out, w.flags, noise,
                                                                                        log_split);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_opacity_regularization(float* pre_opac, int N, float amount, uint32_t* affected, void* stream) {
  if (N < 0 || !affected || (N > 0 && !pre_opac)) return CVHRF_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  CVHRF_CUDA_TRY(cudaMemsetAsync(affected, 0, sizeof(uint32_t), st));
  if (N == 0) return CVHRF_OK;
  opacity_reg_kernel<<<(N + kThreads - 1) / kThreads, kThreads, 0, st>>>(pre_opac, N, amount, affected);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
