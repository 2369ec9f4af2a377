// Band-limited angular-spectrum propagation fused into a hand-written FFT.
//
// Reference path (cuda_prop/python_function.py:109-218): zero_pad to 2S x 2S ->
// torch.fft.fft2 -> fftshift -> bandlimited_propagation_{forward,backward}_kernel
// (cuda/bandlimited_propagation_cuda.cu:29-147) -> ifftshift -> ifft2 -> crop.
// Here the same operator runs as three passes over HBM:
//
//   A (rows, forward):   each of the Hi non-zero input rows -> length-2S spectrum
//   B (columns):         each spectrum column: forward FFT, x transfer x aperture,
//                        inverse FFT, keep only the Ho cropped rows
//   C (rows, inverse):   each kept row: inverse FFT, keep the Wo cropped columns, / (2S)^2
//
// A length-2S transform of a zero-padded line is done as two length-S transforms
// (even and odd output bins): X[2m] = FFT_S(wrap(x))[m] and
// X[2m+1] = FFT_S(wrap(x * w_{2S}^n))[m], where wrap folds padded index n to n mod S
// (the non-zero window is never longer than S, so no two samples collide).  The
// inverse with a crop of at most S outputs folds back the same way:
// y[n] = e[n mod S] + w_{2S}^{-n} f[n mod S].  fftshift/ifftshift never move data:
// the transfer function is evaluated at each bin's shifted coordinates instead.
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <mutex>
#include <vector>
#include "common.cuh"
#include "fft_lines.cuh"
#include "asm_static.cuh"

namespace cvhrf {

// Per-launch list of column jobs (one job = one input spectrum item -> one output item).
constexpr int kMaxJobs = 32;
struct ColumnJobs {
  int n;
  int in_item[kMaxJobs];
  int out_item[kMaxJobs];
  TransferParams tp[kMaxJobs];
};

// ---- pass A: forward row transforms ------------------------------------------------
// in: items x Hi x Wi; A: items x Hi x P, each row in split digit-reversed bin order
// [even bins | odd bins].  One CTA handles `rows` consecutive rows (2 lines per row).
__global__ void __launch_bounds__(512) asm_rows_forward_kernel(
    const float2* __restrict__ in, int total_rows, int Wi, float2* __restrict__ A, FftDesc d, int rows) {
  extern __shared__ float2 sm[];
  const int S = d.S, P = 2 * S;
  const int ow = (P - Wi) / 2;
  const int row0 = blockIdx.x * rows;
  const int nrows = min(rows, total_rows - row0);
  if (nrows <= 0) return;
  // fill: position t of the even line takes padded index t or t+S, whichever is inside
  for (int e = threadIdx.x; e < nrows * S; e += blockDim.x) {
    const int r = e / S, t = e - r * S;
    const float2* src = in + (size_t)(row0 + r) * Wi;
    int pos = t;
    int j = pos - ow;
    if (j < 0 || j >= Wi) { pos = t + S; j = pos - ow; }
    float2 v = make_float2(0.f, 0.f), vo = v;
    if (j >= 0 && j < Wi) {
      v = src[j];
      vo = cmul(v, __ldg(&d.twP[pos]));
    }
    sm[(2 * r) * S + t] = v;
    sm[(2 * r + 1) * S + t] = vo;
  }
  __syncthreads();
  fft_forward_lines(sm, 2 * nrows, S, d);
  for (int e = threadIdx.x; e < nrows * P; e += blockDim.x) {
    const int r = e / P, q = e - r * P;
    A[(size_t)(row0 + r) * P + q] = sm[(2 * r) * S + q];  // lines 2r, 2r+1 are contiguous
  }
}

// ---- pass B: column transforms with the transfer function --------------------------
// A: in_items x Hi x P; B: out_items x Ho x P.  CTA = `cols` consecutive columns of one job.
__global__ void __launch_bounds__(512) asm_columns_kernel(
    const float2* __restrict__ A, int Hi, float2* __restrict__ B, int Ho, FftDesc d, int cols,
    ColumnJobs jobs, int accumulate) {
  extern __shared__ float2 sm[];
  const int S = d.S, P = 2 * S;
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * cols;
  const int ncols = min(cols, P - q0);
  const float2* Ain = A + (size_t)jobs.in_item[job] * Hi * P;
  float2* Bout = B + (size_t)jobs.out_item[job] * Ho * P;
  const TransferParams tp = jobs.tp[job];
  const int oh = (P - Hi) / 2;
  // lines: column c, half h -> line 2c + h
  for (int e = threadIdx.x; e < ncols * S; e += blockDim.x) {
    const int t = e / ncols, c = e - t * ncols;
    int pos = t;
    int r = pos - oh;
    if (r < 0 || r >= Hi) { pos = t + S; r = pos - oh; }
    float2 v = make_float2(0.f, 0.f), vo = v;
    if (r >= 0 && r < Hi) {
      v = Ain[(size_t)r * P + q0 + c];
      vo = cmul(v, __ldg(&d.twP[pos]));
    }
    sm[(2 * c) * S + t] = v;
    sm[(2 * c + 1) * S + t] = vo;
  }
  __syncthreads();
  fft_forward_lines(sm, 2 * ncols, S, d);
  for (int e = threadIdx.x; e < 2 * ncols * S; e += blockDim.x) {
    const int line = e / S, pos = e - line * S;
    const int c = line >> 1, h = line & 1;
    const int q = q0 + c;
    const int qh = q >= S ? 1 : 0;
    const int kv = 2 * __ldg(&d.digrev[q - qh * S]) + qh;
    const int ku = 2 * __ldg(&d.digrev[pos]) + h;
    sm[e] = cmul(sm[e], transfer_at(ku, kv, P, tp));
  }
  __syncthreads();
  fft_inverse_lines(sm, 2 * ncols, S, d);
  const int oc = (P - Ho) / 2;
  for (int e = threadIdx.x; e < Ho * ncols; e += blockDim.x) {
    const int rr = e / ncols, c = e - rr * ncols;
    const int n = oc + rr;
    const int t = n >= S ? n - S : n;
    const float2 ev = sm[(2 * c) * S + t];
    const float2 od = sm[(2 * c + 1) * S + t];
    float2 v = cadd(ev, cmul(cconj(__ldg(&d.twP[n])), od));
    float2* dst = Bout + (size_t)rr * P + q0 + c;
    if (accumulate) { float2 o = *dst; v = cadd(o, v); }
    *dst = v;
  }
}

// ---- pass C: inverse row transforms + crop + 1/P^2 ---------------------------------
__global__ void __launch_bounds__(512) asm_rows_inverse_kernel(
    const float2* __restrict__ B, int total_rows, float2* __restrict__ out, int Wo, FftDesc d, int rows,
    float scale, int accumulate) {
  extern __shared__ float2 sm[];
  const int S = d.S, P = 2 * S;
  const int row0 = blockIdx.x * rows;
  const int nrows = min(rows, total_rows - row0);
  if (nrows <= 0) return;
  for (int e = threadIdx.x; e < nrows * P; e += blockDim.x) {
    const int r = e / P, q = e - r * P;
    sm[(2 * r) * S + q] = B[(size_t)(row0 + r) * P + q];
  }
  __syncthreads();
  fft_inverse_lines(sm, 2 * nrows, S, d);
  const int oc = (P - Wo) / 2;
  for (int e = threadIdx.x; e < nrows * Wo; e += blockDim.x) {
    const int r = e / Wo, x = e - r * Wo;
    const int n = oc + x;
    const int t = n >= S ? n - S : n;
    const float2 ev = sm[(2 * r) * S + t];
    const float2 od = sm[(2 * r + 1) * S + t];
    float2 v = cadd(ev, cmul(cconj(__ldg(&d.twP[n])), od));
    v.x *= scale;
    v.y *= scale;
    float2* dst = out + (size_t)(row0 + r) * Wo + x;
    if (accumulate) { float2 o = *dst; v = cadd(o, v); }
    *dst = v;
  }
}

}  // namespace cvhrf

// ---------------------------------------------------------------------------------
using namespace cvhrf;

struct cvhrf_asm_plan {
  FftDesc desc;     // the plan the kernels of this size run (compile-time radices where they exist)
  FftDesc desc_rt;  // the runtime mixed-radix plan (its own digit-reversal table)
  void* dev_mem;
  int device;
};

static bool factorize(int S, FftDesc& d) {
  int n = S, a = 0;
  while (n % 2 == 0) { n /= 2; ++a; }
  int b = 0; while (n % 3 == 0) { n /= 3; ++b; }
  int c = 0; while (n % 5 == 0) { n /= 5; ++c; }
  if (n != 1) return false;
  std::vector<int> r;
  int n8 = a / 3, rem = a % 3;
  if (rem == 1 && n8 >= 1) { n8 -= 1; for (int i = 0; i < n8; ++i) r.push_back(8); r.push_back(4); r.push_back(4); }
  else { for (int i = 0; i < n8; ++i) r.push_back(8); if (rem == 1) r.push_back(2); if (rem == 2) r.push_back(4); }
  for (int i = 0; i < b; ++i) r.push_back(3);
  for (int i = 0; i < c; ++i) r.push_back(5);
  if ((int)r.size() > kMaxFftStages) return false;
  d.S = S;
  d.nst = (int)r.size();
  int L = S;
  for (int i = 0; i < d.nst; ++i) {
    d.radix[i] = r[i];
    L /= r[i];
    d.L[i] = L;
    d.span[i] = S / (r[i] * L);
  }
  return true;
}

extern "C" int cvhrf_asm_plan_create(int S, cvhrf_asm_plan** plan_out) {
  if (!plan_out || S < 8 || S > 4096) return CVHRF_EINVAL;
  FftDesc d{};
  if (!factorize(S, d)) return CVHRF_EUNSUPPORTED;
  const int P = 2 * S;
  std::vector<float2> tw(S), twP(P);
  for (int t = 0; t < S; ++t) {
    double a = -2.0 * M_PI * (double)t / (double)S;
    tw[t] = make_float2((float)cos(a), (float)sin(a));
  }
  for (int t = 0; t < P; ++t) {
    double a = -2.0 * M_PI * (double)t / (double)P;
    twP[t] = make_float2((float)cos(a), (float)sin(a));
  }
  // digit reversal: bin k = m1 + R1 (m2 + R2 (...)) sits at position sum_i L_i m_i.  One table for
  // the runtime radices of `d`, and, for a size with a compile-time plan, a second one for that
  // plan's radices (the kernels of the two plans order their spectra differently).
  auto digit_reversal = [S](const int* rad, const int* Ls, int nst) {
    std::vector<int> dr(S);
    for (int k = 0; k < S; ++k) {
      int rem = k, pos = 0;
      for (int i = 0; i < nst; ++i) {
        int m = rem % rad[i];
        rem /= rad[i];
        pos += Ls[i] * m;
      }
      dr[pos] = k;
    }
    return dr;
  };
  std::vector<int> digrev_rt = digit_reversal(d.radix, d.L, d.nst);
  std::vector<int> digrev_st = digrev_rt;
  const bool has_static = static_fft_size(S);
  if (has_static) {
    int rad[kMaxFftStages], Ls[kMaxFftStages], nst = 0;
    static_fft_radices(S, rad, &nst);
    int L = S;
    for (int i = 0; i < nst; ++i) { L /= rad[i]; Ls[i] = L; }
    digrev_st = digit_reversal(rad, Ls, nst);
  }
  const size_t dr_off = (size_t)(S + P) * sizeof(float2);
  size_t bytes = dr_off + 2 * (size_t)S * sizeof(int);
  cvhrf_asm_plan* plan = (cvhrf_asm_plan*)calloc(1, sizeof(cvhrf_asm_plan));
  if (!plan) return CVHRF_EINVAL;
  CVHRF_CUDA_TRY(cudaGetDevice(&plan->device));
  cudaError_t e = cudaMalloc(&plan->dev_mem, bytes);
  if (e != cudaSuccess) { free(plan); set_last_cuda_error((int)e); return CVHRF_ECUDA; }
  char* base = (char*)plan->dev_mem;
  e = cudaMemcpy(base, tw.data(), S * sizeof(float2), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(base + S * sizeof(float2), twP.data(), P * sizeof(float2), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(base + dr_off, digrev_st.data(), S * sizeof(int), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(base + dr_off + S * sizeof(int), digrev_rt.data(), S * sizeof(int), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) { cudaFree(plan->dev_mem); free(plan); set_last_cuda_error((int)e); return CVHRF_ECUDA; }
  d.tw = (const float2*)base;
  d.twP = (const float2*)(base + S * sizeof(float2));
  d.digrev = (const int*)(base + dr_off);
  plan->desc_rt = d;
  plan->desc_rt.digrev = (const int*)(base + dr_off + S * sizeof(int));
  plan->desc = d;
  *plan_out = plan;
  return CVHRF_OK;
}

extern "C" int cvhrf_asm_plan_destroy(cvhrf_asm_plan* plan) {
  if (!plan) return CVHRF_OK;
  cudaFree(plan->dev_mem);
  free(plan);
  return CVHRF_OK;
}

static const size_t kSmemBudget = 100 * 1024;

// Both intermediates, sized for the transposed layout of the compile-time passes (column
// stride col_stride(rows)); the runtime passes use the first rows x 2S values of each.
static size_t ws_bytes_impl(int S, int in_items, int Hi, int out_items, int Ho) {
  const size_t P = 2 * (size_t)S;
  return align_up((size_t)in_items * col_stride(Hi) * P * sizeof(float2), 256) +
         align_up((size_t)out_items * col_stride(Ho) * P * sizeof(float2), 256);
}

extern "C" size_t cvhrf_asm_workspace_bytes(int S, int items, int Hi, int Wi, int out_items, int Ho, int Wo) {
  (void)Wi; (void)Wo;
  return ws_bytes_impl(S, items, Hi, out_items, Ho);
}

namespace {

int rows_per_cta(int S) {
  int r = (int)(kSmemBudget / (2 * (size_t)S * sizeof(float2)));
  return r < 1 ? 1 : (r > 16 ? 16 : r);
}

int launch_rows_forward(const FftDesc& d, const float2* in, int total_rows, int Wi, float2* A, cudaStream_t st) {
  const int rows = rows_per_cta(d.S);
  const size_t smem = (size_t)rows * 2 * d.S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(asm_rows_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((total_rows + rows - 1) / rows);
  asm_rows_forward_kernel<<<grid, 512, smem, st>>>(in, total_rows, Wi, A, d, rows);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

int launch_columns(const FftDesc& d, const float2* A, int Hi, float2* B, int Ho, const ColumnJobs& jobs,
                   int accumulate, cudaStream_t st) {
  const int P = 2 * d.S;
  const int cols = rows_per_cta(d.S);
  const size_t smem = (size_t)cols * 2 * d.S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(asm_columns_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((P + cols - 1) / cols, jobs.n);
  asm_columns_kernel<<<grid, 512, smem, st>>>(A, Hi, B, Ho, d, cols, jobs, accumulate);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

int launch_rows_inverse(const FftDesc& d, const float2* B, int total_rows, float2* out, int Wo, int accumulate,
                        cudaStream_t st) {
  const int rows = rows_per_cta(d.S);
  const size_t smem = (size_t)rows * 2 * d.S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(asm_rows_inverse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const float P = 2.0f * d.S;
  const float scale = 1.0f / (P * P);
  dim3 grid((total_rows + rows - 1) / rows);
  asm_rows_inverse_kernel<<<grid, 512, smem, st>>>(B, total_rows, out, Wo, d, rows, scale, accumulate);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

bool dims_ok(int S, int H, int W) { return H >= 1 && W >= 1 && H <= S && W <= S; }

}  // namespace

extern "C" int cvhrf_asm_propagate(const cvhrf_asm_plan* plan, const void* in, int Hi, int Wi, void* out, int Ho,
                                   int Wo, float wavelength, float pixel_pitch, float distance, float aperture,
                                   int accumulate, void* workspace, size_t workspace_bytes, void* stream) {
  if (!plan || !in || !out) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (!dims_ok(d.S, Hi, Wi) || !dims_ok(d.S, Ho, Wo)) return CVHRF_EINVAL;
  if (!(wavelength > 0.0f) || !(pixel_pitch > 0.0f)) return CVHRF_EINVAL;
  Carver cv(workspace, workspace_bytes);
  const int P = 2 * d.S;
  float2* A = cv.take<float2>((size_t)col_stride(Hi) * P);
  float2* B = cv.take<float2>((size_t)col_stride(Ho) * P);
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if (static_fft_size(d.S)) {
    ColPlan cp;
    cp.njobs = 1;
    cp.item[0] = 0;
    cp.n[0] = 1;
    cp.items[0][0] = 0;
    cp.tpi[0][0] = 0;
    cp.tp[0] = make_transfer(wavelength, pixel_pitch, distance, aperture, P);
    if ((rc = static_rows_forward(d, (const float2*)in, 1, Hi, Wi, A, st))) return rc;
    if ((rc = static_columns(d, false, A, Hi, B, Ho, cp, nullptr, st))) return rc;
    return static_rows_inverse(d, B, 1, Ho, (float2*)out, Wo, accumulate, st);
  }
  if ((rc = launch_rows_forward(d, (const float2*)in, Hi, Wi, A, st))) return rc;
  ColumnJobs jobs{};
  jobs.n = 1;
  jobs.in_item[0] = 0;
  jobs.out_item[0] = 0;
  jobs.tp[0] = make_transfer(wavelength, pixel_pitch, distance, aperture, P);
  if ((rc = launch_columns(d, A, Hi, B, Ho, jobs, 0, st))) return rc;
  return launch_rows_inverse(d, B, Ho, (float2*)out, Wo, accumulate, st);
}

extern "C" int cvhrf_asm_propagate_planes(const cvhrf_asm_plan* plan, const void* fields, int K, int C, int H, int W,
                                          const float* wavelengths, const float* distances, float pixel_pitch,
                                          float aperture, void* holo, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (!plan || !fields || !holo || !wavelengths || !distances) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (K < 1 || C < 1 || K * C > kMaxJobs || !dims_ok(d.S, H, W)) return CVHRF_EINVAL;
  const int S = d.S, P = 2 * S;
  Carver cv(workspace, workspace_bytes);
  float2* A = cv.take<float2>((size_t)K * C * col_stride(H) * P);
  float2* B = cv.take<float2>((size_t)C * col_stride(S) * P);
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  for (int c = 0; c < C; ++c)
    if (!(wavelengths[c] > 0.0f)) return CVHRF_EINVAL;
  if (static_fft_size(d.S) && K * C <= kMaxTableItems) {
    ColPlan cp;
    cp.njobs = C;
    for (int c = 0; c < C; ++c) {
      cp.item[c] = c;
      cp.n[c] = K;
      for (int p = 0; p < K; ++p) {
        cp.items[c][p] = (short)(p * C + c);
        cp.tpi[c][p] = (short)(p * C + c);
        cp.tp[p * C + c] = make_transfer(wavelengths[c], pixel_pitch, distances[p], aperture, P);
      }
    }
    if ((rc = static_rows_forward(d, (const float2*)fields, K * C, H, W, A, st))) return rc;
    if ((rc = static_columns(d, false, A, H, B, S, cp, nullptr, st))) return rc;
    return static_rows_inverse(d, B, C, S, (float2*)holo, S, 0, st);
  }
  // runtime plan: more planes per channel than the compile-time column pass sums
  const FftDesc& dr = plan->desc_rt;
  if ((rc = launch_rows_forward(dr, (const float2*)fields, K * C * H, W, A, st))) return rc;
  for (int p = 0; p < K; ++p) {
    ColumnJobs jobs{};
    jobs.n = C;
    for (int c = 0; c < C; ++c) {
      if (!(wavelengths[c] > 0.0f)) return CVHRF_EINVAL;
      jobs.in_item[c] = p * C + c;
      jobs.out_item[c] = c;
      jobs.tp[c] = make_transfer(wavelengths[c], pixel_pitch, distances[p], aperture, P);
    }
    if ((rc = launch_columns(dr, A, H, B, S, jobs, p > 0 ? 1 : 0, st))) return rc;
  }
  return launch_rows_inverse(dr, B, C * S, (float2*)holo, S, 0, st);
}

extern "C" int cvhrf_asm_propagate_planes_adjoint(const cvhrf_asm_plan* plan, const void* grad_holo, int K, int C,
                                                  int H, int W, const float* wavelengths, const float* distances,
                                                  float pixel_pitch, float aperture, void* grad_fields,
                                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (!plan || !grad_holo || !grad_fields || !wavelengths || !distances) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (K < 1 || C < 1 || K * C > kMaxJobs || !dims_ok(d.S, H, W)) return CVHRF_EINVAL;
  const int S = d.S, P = 2 * S;
  Carver cv(workspace, workspace_bytes);
  float2* A = cv.take<float2>((size_t)C * col_stride(S) * P);
  float2* B = cv.take<float2>((size_t)K * C * col_stride(H) * P);
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  for (int c = 0; c < C; ++c)
    if (!(wavelengths[c] > 0.0f)) return CVHRF_EINVAL;
  if (static_fft_size(d.S) && K * C <= kMaxTableItems) {
    ColPlan cp;
    cp.njobs = C;
    for (int c = 0; c < C; ++c) {
      cp.item[c] = c;
      cp.n[c] = K;
      for (int p = 0; p < K; ++p) {
        cp.items[c][p] = (short)(p * C + c);
        cp.tpi[c][p] = (short)(p * C + c);
        // the adjoint of propagation by d is propagation by -d: the scatter pass multiplies
        // by conj(H_d) = H_-d, as it does with a table of H_d
        cp.tp[p * C + c] = make_transfer(wavelengths[c], pixel_pitch, distances[p], aperture, P);
      }
    }
    if ((rc = static_rows_forward(d, (const float2*)grad_holo, C, S, S, A, st))) return rc;
    if ((rc = static_columns(d, true, A, S, B, H, cp, nullptr, st))) return rc;
    return static_rows_inverse(d, B, K * C, H, (float2*)grad_fields, W, 0, st);
  }
  if ((rc = launch_rows_forward(d, (const float2*)grad_holo, C * S, S, A, st))) return rc;
  ColumnJobs jobs{};
  jobs.n = K * C;
  for (int p = 0; p < K; ++p)
    for (int c = 0; c < C; ++c) {
      if (!(wavelengths[c] > 0.0f)) return CVHRF_EINVAL;
      jobs.in_item[p * C + c] = c;
      jobs.out_item[p * C + c] = p * C + c;
      jobs.tp[p * C + c] = make_transfer(wavelengths[c], pixel_pitch, -distances[p], aperture, P);
    }
  if ((rc = launch_columns(d, A, S, B, H, jobs, 0, st))) return rc;
  return launch_rows_inverse(d, B, K * C * H, (float2*)grad_fields, W, 0, st);
}

// ---------------------------------------------------------------------------------
// Allocation-free variant of cvhrf_asm_propagate.
//
// Some callers cannot allocate device memory at the moment they propagate: code
// running while a memory pool is frozen or exhausted, plugin hosts that forbid
// allocation inside their execute callback, or real-time loops that must not touch
// the allocator.  For them this entry point keeps everything it needs — the two
// intermediate spectra and the FFT tables — in one fixed file-scope device array
// (kNoAllocBytes, held by every GPU that loads the library until the process exits),
// so it needs neither a workspace nor a plan.  The limit is S <= kNoAllocMaxS.
// Every call shares that one array and overwrites it completely (tables, then the
// row and column passes), so nothing from a previous call is read; two calls that
// overlap on the GPU (different streams, or different host threads without ordering)
// race on it.
namespace cvhrf {
namespace {

constexpr int kNoAllocMaxS = 512;
constexpr size_t kNoAllocSpectrum = (size_t)kNoAllocMaxS * (2 * kNoAllocMaxS) * sizeof(float2);  // Hi x P
constexpr size_t kNoAllocTables =
    align_up_c((size_t)(3 * kNoAllocMaxS) * sizeof(float2) + (size_t)kNoAllocMaxS * sizeof(int), 256);
constexpr size_t kNoAllocBytes = 2 * kNoAllocSpectrum + kNoAllocTables;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// One device address per device, looked up once with that device current.
constexpr int kMaxDevices = 64;
static void* g_noalloc_addr[kMaxDevices] = {nullptr};
static std::mutex g_noalloc_mutex;

int noalloc_scratch(void** out) {
  int dev = 0;
  CVHRF_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return CVHRF_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    CVHRF_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return CVHRF_OK;
}

// Twiddle and digit-reversal tables of a plan, computed on the device (the same
// values cvhrf_asm_plan_create uploads: w = exp(-2 pi i t / n) in double, rounded).
__global__ void noalloc_tables_kernel(FftDesc d, float2* tw, float2* twP, int* digrev) {
  const int S = d.S, P = 2 * S;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < P; t += gridDim.x * blockDim.x) {
    double s, c;
    sincospi(-2.0 * (double)t / (double)P, &s, &c);
    twP[t] = make_float2((float)c, (float)s);
    if (t < S) {
      sincospi(-2.0 * (double)t / (double)S, &s, &c);
      tw[t] = make_float2((float)c, (float)s);
      int rem = t, pos = 0;
      for (int i = 0; i < d.nst; ++i) {
        const int m = rem % d.radix[i];
        rem /= d.radix[i];
        pos += d.L[i] * m;
      }
      digrev[pos] = t;
    }
  }
}

}  // namespace
}  // namespace cvhrf

// ---- precomputed transfer tables (compile-time sizes) ---------------------------------

extern "C" size_t cvhrf_asm_transfer_table_bytes(int S, int K, int C) {
  if (S < 1 || K < 1 || C < 1 || K * C > kMaxTableItems || !static_fft_size(S)) return 0;
  return (size_t)K * C * 4 * S * S * sizeof(float2);
}

extern "C" int cvhrf_asm_transfer_table_build(const cvhrf_asm_plan* plan, int K, int C, const float* wavelengths,
                                              const float* distances, float pixel_pitch, float aperture, void* table,
                                              void* stream) {
  if (!plan || !table || !wavelengths || !distances) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (K < 1 || C < 1 || K * C > kMaxTableItems) return CVHRF_EINVAL;
  if (!static_fft_size(d.S)) return CVHRF_EUNSUPPORTED;
  TransferTable tt{};
  for (int p = 0; p < K; ++p)
    for (int c = 0; c < C; ++c) {
      if (!(wavelengths[c] > 0.0f)) return CVHRF_EINVAL;
      tt.tp[p * C + c] = make_transfer(wavelengths[c], pixel_pitch, distances[p], aperture, 2 * d.S);
    }
  return static_transfer_table(d, (float2*)table, tt, K * C, (cudaStream_t)stream);
}

extern "C" int cvhrf_asm_transfer_table_upload(const cvhrf_asm_plan* plan, int items, const void* centred,
                                               void* table, void* stream) {
  if (!plan || !table || !centred || items < 1 || items > kMaxTableItems) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (!static_fft_size(d.S)) return CVHRF_EUNSUPPORTED;
  return static_transfer_upload(d, (float2*)table, (const float2*)centred, items, (cudaStream_t)stream);
}

extern "C" int cvhrf_asm_propagate_planes_table(const cvhrf_asm_plan* plan, const void* fields, int K, int C, int H,
                                                int W, const void* table, void* holo, void* workspace,
                                                size_t workspace_bytes, void* stream) {
  if (!plan || !fields || !holo || !table) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (K < 1 || C < 1 || K * C > kMaxTableItems || !dims_ok(d.S, H, W)) return CVHRF_EINVAL;
  if (!static_fft_size(d.S)) return CVHRF_EUNSUPPORTED;
  const int S = d.S, P = 2 * S;
  Carver cv(workspace, workspace_bytes);
  float2* A = cv.take<float2>((size_t)K * C * col_stride(H) * P);
  float2* B = cv.take<float2>((size_t)C * col_stride(S) * P);
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  ColPlan cp;
  cp.njobs = C;
  for (int c = 0; c < C; ++c) {
    cp.item[c] = c;
    cp.n[c] = K;
    for (int p = 0; p < K; ++p) cp.items[c][p] = cp.tpi[c][p] = (short)(p * C + c);
  }
  int rc;
  if ((rc = static_rows_forward(d, (const float2*)fields, K * C, H, W, A, st))) return rc;
  if ((rc = static_columns(d, false, A, H, B, S, cp, (const float2*)table, st))) return rc;
  return static_rows_inverse(d, B, C, S, (float2*)holo, S, 0, st);
}

extern "C" int cvhrf_asm_propagate_planes_adjoint_table(const cvhrf_asm_plan* plan, const void* grad_holo, int K,
                                                        int C, int H, int W, const void* table, void* grad_fields,
                                                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!plan || !grad_holo || !grad_fields || !table) return CVHRF_EINVAL;
  const FftDesc& d = plan->desc;
  if (K < 1 || C < 1 || K * C > kMaxTableItems || !dims_ok(d.S, H, W)) return CVHRF_EINVAL;
  if (!static_fft_size(d.S)) return CVHRF_EUNSUPPORTED;
  const int S = d.S, P = 2 * S;
  Carver cv(workspace, workspace_bytes);
  float2* A = cv.take<float2>((size_t)C * col_stride(S) * P);
  float2* B = cv.take<float2>((size_t)K * C * col_stride(H) * P);
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  ColPlan cp;
  cp.njobs = C;
  for (int c = 0; c < C; ++c) {
    cp.item[c] = c;
    cp.n[c] = K;
    for (int p = 0; p < K; ++p) cp.items[c][p] = cp.tpi[c][p] = (short)(p * C + c);
  }
  int rc;
  if ((rc = static_rows_forward(d, (const float2*)grad_holo, C, S, S, A, st))) return rc;
  if ((rc = static_columns(d, true, A, S, B, H, cp, (const float2*)table, st))) return rc;
  return static_rows_inverse(d, B, K * C, H, (float2*)grad_fields, W, 0, st);
}

extern "C" int cvhrf_asm_propagate_noalloc(const void* in, int Hi, int Wi, void* out, int Ho, int Wo, int S,
                                           float wavelength, float pixel_pitch, float distance, float aperture,
                                           int accumulate, void* stream) {
  if (!in || !out) return CVHRF_EINVAL;
  if (S < 8 || S > kNoAllocMaxS) return CVHRF_EUNSUPPORTED;
  if (!dims_ok(S, Hi, Wi) || !dims_ok(S, Ho, Wo)) return CVHRF_EINVAL;
  if (!(wavelength > 0.0f) || !(pixel_pitch > 0.0f)) return CVHRF_EINVAL;
  FftDesc d{};
  if (!factorize(S, d)) return CVHRF_EUNSUPPORTED;
  void* base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  char* b = (char*)base;
  float2* A = (float2*)b;
  float2* B = (float2*)(b + kNoAllocSpectrum);
  float2* tw = (float2*)(b + 2 * kNoAllocSpectrum);
  float2* twP = tw + S;
  int* digrev = (int*)(twP + 2 * S);
  d.tw = tw;
  d.twP = twP;
  d.digrev = digrev;
  cudaStream_t st = (cudaStream_t)stream;
  const int P = 2 * S;
  noalloc_tables_kernel<<<(P + 255) / 256, 256, 0, st>>>(d, tw, twP, digrev);
  CVHRF_LAUNCH_CHECK();
  if ((rc = launch_rows_forward(d, (const float2*)in, Hi, Wi, A, st))) return rc;
  ColumnJobs jobs{};
  jobs.n = 1;
  jobs.tp[0] = make_transfer(wavelength, pixel_pitch, distance, aperture, P);
  if ((rc = launch_columns(d, A, Hi, B, Ho, jobs, 0, st))) return rc;
  return launch_rows_inverse(d, B, Ho, (float2*)out, Wo, accumulate, st);
}
