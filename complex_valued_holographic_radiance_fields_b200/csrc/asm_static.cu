// Propagation passes specialised for compile-time line lengths (see fft_static.cuh).
//
// Same three-pass algorithm and arithmetic as asm_propagation.cu (rows forward; columns
// with the transfer function; rows inverse with crop), with two differences:
//   * the FFTs use StaticPlan<S> (composite radices <= 32 in registers);
//   * the column pass sums several inputs (the K planes of one channel, each with its own
//     transfer function) into one output in shared memory, so a multi-plane propagation
//     writes the intermediate once instead of read-modify-writing it per plane.
#include "asm_static.cuh"
#include "fft_static.cuh"

namespace cvhrf {
namespace {

constexpr int kThreads = 256;

template <int S>
__global__ void __launch_bounds__(kThreads) rows_forward_s(const float2* __restrict__ in, int total_rows, int Wi,
                                                          float2* __restrict__ A, const float2* __restrict__ tw,
                                                          const float2* __restrict__ twP, int rows) {
  extern __shared__ float2 sm[];
  constexpr int P = 2 * S;
  const int ow = (P - Wi) / 2;
  const int row0 = blockIdx.x * rows;
  const int nrows = min(rows, total_rows - row0);
  if (nrows <= 0) return;
  // all of the block's row loads in flight at once (asynchronous copies), then the odd
  // half-lines are formed in place
  for (int e = threadIdx.x; e < nrows * S; e += blockDim.x) {
    const int r = e / S, t = e - r * S;
    int j = t - ow;
    if (j < 0 || j >= Wi) j = t + S - ow;
    float2* dst = sm + (2 * r) * S + t;
    if (j >= 0 && j < Wi) cp_async8(dst, in + (size_t)(row0 + r) * Wi + j);
    else *dst = make_float2(0.f, 0.f);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  for (int e = threadIdx.x; e < nrows * S; e += blockDim.x) {
    const int r = e / S, t = e - r * S;
    const int j = t - ow;
    const int pos = (j < 0 || j >= Wi) ? t + S : t;
    sm[(2 * r + 1) * S + t] = cmul(sm[(2 * r) * S + t], __ldg(&twP[pos]));
  }
  __syncthreads();
  static_fft_forward<S>(sm, 2 * nrows, S, tw);
  for (int e = threadIdx.x; e < nrows * P; e += blockDim.x) {
    const int r = e / P, q = e - r * P;
    A[(size_t)(row0 + r) * P + q] = sm[(2 * r) * S + q];
  }
}

template <int S>
__global__ void __launch_bounds__(kThreads) columns_s(const float2* __restrict__ A, int Hi, float2* __restrict__ B,
                                                     int Ho, const float2* __restrict__ tw,
                                                     const float2* __restrict__ twP, const int* __restrict__ digrev,
                                                     int cols, const SumJobs jobs) {
  extern __shared__ float2 sm[];
  constexpr int P = 2 * S;
  constexpr int LD = S + 1;  // padded line stride: consecutive lines start in different banks
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * cols;
  const int ncols = min(cols, P - q0);
  float2* acc = sm + 2 * cols * LD;  // Ho x ncols output accumulator
  const int oh = (P - Hi) / 2, oc = (P - Ho) / 2;
  const int nin = jobs.nin[job];
  for (int k = 0; k < nin; ++k) {
    const float2* Ain = A + (size_t)jobs.in_item[job][k] * Hi * P;
    const TransferParams tp = jobs.tp[job][k];
#pragma unroll 4
    for (int e = threadIdx.x; e < ncols * S; e += blockDim.x) {
      const int t = e / ncols, c = e - t * ncols;
      int pos = t;
      int r = pos - oh;
      if (r < 0 || r >= Hi) { pos = t + S; r = pos - oh; }
      float2 v = make_float2(0.f, 0.f), vo = v;
      if (r >= 0 && r < Hi) {
        v = Ain[(size_t)r * P + q0 + c];
        vo = cmul(v, __ldg(&twP[pos]));
      }
      sm[(2 * c) * LD + t] = v;
      sm[(2 * c + 1) * LD + t] = vo;
    }
    __syncthreads();
    static_fft_forward<S>(sm, 2 * ncols, LD, tw);
    for (int e = threadIdx.x; e < 2 * ncols * S; e += blockDim.x) {
      const int line = e / S, pos = e - line * S;
      const int c = line >> 1, h = line & 1;
      const int q = q0 + c;
      const int qh = q >= S ? 1 : 0;
      const int kv = 2 * __ldg(&digrev[q - qh * S]) + qh;
      const int ku = 2 * __ldg(&digrev[pos]) + h;
      sm[line * LD + pos] = cmul(sm[line * LD + pos], transfer_at(ku, kv, P, tp));
    }
    __syncthreads();
    static_fft_inverse<S>(sm, 2 * ncols, LD, tw);
    for (int e = threadIdx.x; e < Ho * ncols; e += blockDim.x) {
      const int rr = e / ncols, c = e - rr * ncols;
      const int n = oc + rr;
      const int t = n >= S ? n - S : n;
      const float2 v = cadd(sm[(2 * c) * LD + t], cmul(cconj(__ldg(&twP[n])), sm[(2 * c + 1) * LD + t]));
      acc[e] = k == 0 ? v : cadd(acc[e], v);
    }
    __syncthreads();
  }
  float2* Bout = B + (size_t)jobs.out_item[job] * Ho * P;
  for (int e = threadIdx.x; e < Ho * ncols; e += blockDim.x) {
    const int rr = e / ncols, c = e - rr * ncols;
    Bout[(size_t)rr * P + q0 + c] = acc[e];
  }
}

template <int S>
__global__ void __launch_bounds__(kThreads) rows_inverse_s(const float2* __restrict__ B, int total_rows,
                                                          float2* __restrict__ out, int Wo,
                                                          const float2* __restrict__ tw,
                                                          const float2* __restrict__ twP, int rows, float scale,
                                                          int accumulate) {
  extern __shared__ float2 sm[];
  constexpr int P = 2 * S;
  const int row0 = blockIdx.x * rows;
  const int nrows = min(rows, total_rows - row0);
  if (nrows <= 0) return;
  for (int e = threadIdx.x; e < nrows * P; e += blockDim.x) {
    const int r = e / P, q = e - r * P;
    cp_async8(sm + (2 * r) * S + q, B + (size_t)(row0 + r) * P + q);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  static_fft_inverse<S>(sm, 2 * nrows, S, tw);
  const int oc = (P - Wo) / 2;
  for (int e = threadIdx.x; e < nrows * Wo; e += blockDim.x) {
    const int r = e / Wo, x = e - r * Wo;
    const int n = oc + x;
    const int t = n >= S ? n - S : n;
    float2 v = cadd(sm[(2 * r) * S + t], cmul(cconj(__ldg(&twP[n])), sm[(2 * r + 1) * S + t]));
    v.x *= scale;
    v.y *= scale;
    float2* dst = out + (size_t)(row0 + r) * Wo + x;
    if (accumulate) v = cadd(*dst, v);
    *dst = v;
  }
}

// Transfer table of one input item: H[(q * 2 + h) * S + pos] = transfer x aperture at row
// bin ku = 2 digrev[pos] + h and column bin kv of column q (the column pass layout).
template <int S>
__global__ void __launch_bounds__(kThreads) transfer_table_s(float2* __restrict__ table, const int* __restrict__ digrev,
                                                            const TransferTable tt) {
  constexpr int P = 2 * S;
  const int item = blockIdx.y;
  const TransferParams tp = tt.tp[item];
  float2* H = table + (size_t)item * P * P;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < (size_t)P * P; e += (size_t)gridDim.x * blockDim.x) {
    const int q = (int)(e / P), r = (int)(e - (size_t)q * P);
    const int h = r / S, pos = r - h * S;
    const int qh = q >= S ? 1 : 0;
    const int kv = 2 * __ldg(&digrev[q - qh * S]) + qh;
    const int ku = 2 * __ldg(&digrev[pos]) + h;
    H[e] = transfer_at(ku, kv, P, tp);
  }
}

// Transfer table from a caller's transfer function given in centred (fftshifted) order,
// Hc[item][y][x] at row bin (y + S) mod P and column bin (x + S) mod P, reordered into the
// column pass layout of transfer_table_s.
template <int S>
__global__ void __launch_bounds__(kThreads) transfer_upload_s(float2* __restrict__ table, const int* __restrict__ digrev,
                                                             const float2* __restrict__ Hc) {
  constexpr int P = 2 * S;
  const int item = blockIdx.y;
  float2* H = table + (size_t)item * P * P;
  const float2* src = Hc + (size_t)item * P * P;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < (size_t)P * P; e += (size_t)gridDim.x * blockDim.x) {
    const int q = (int)(e / P), r = (int)(e - (size_t)q * P);
    const int h = r / S, pos = r - h * S;
    const int qh = q >= S ? 1 : 0;
    const int kv = 2 * __ldg(&digrev[q - qh * S]) + qh;
    const int ku = 2 * __ldg(&digrev[pos]) + h;
    const int ys = ku >= S ? ku - S : ku + S, xs = kv >= S ? kv - S : kv + S;
    H[e] = src[(size_t)ys * P + xs];
  }
}

// Column pass of a K-plane propagation with a precomputed transfer table: for channel c
// = blockIdx.y, sum over planes p of H[p, c] * FFT(column of A[p * C + c]) is accumulated
// in shared memory and inverse-transformed once (the inverse transform is linear), so a
// column costs K forward transforms and one inverse.  The columns of plane p + 1 are
// fetched with asynchronous copies into a staging line while plane p is transformed.
// Shared memory: 2 COLS work lines, 2 COLS spectrum lines, COLS staging lines (stride S+1).
template <int S, int COLS, int NT>
__global__ void __launch_bounds__(NT) columns_sum_table_s(const float2* __restrict__ A, int Hi,
                                                         float2* __restrict__ B, int Ho,
                                                         const float2* __restrict__ tw,
                                                         const float2* __restrict__ twP,
                                                         const float2* __restrict__ table, int K, int C) {
  extern __shared__ float2 sm[];
  constexpr int P = 2 * S;
  constexpr int LD = S + 1;
  float2* work = sm;
  float2* spec = sm + 2 * COLS * LD;
  float2* raw = sm + 4 * COLS * LD;
  const int c = blockIdx.y;
  const int q0 = blockIdx.x * COLS;
  const int ncols = min(COLS, P - q0);
  const int oh = (P - Hi) / 2, oc = (P - Ho) / 2;
  auto fetch = [&](int p) {
    const float2* Ain = A + (size_t)(p * C + c) * Hi * P + q0;
    for (int e = threadIdx.x; e < ncols * S; e += NT) {
      const int t = e / ncols, cc = e - t * ncols;
      int r = t - oh;
      if (r < 0 || r >= Hi) r = t + S - oh;
      float2* dst = raw + cc * LD + t;
      if (r >= 0 && r < Hi) cp_async8(dst, Ain + (size_t)r * P + cc);
      else *dst = make_float2(0.f, 0.f);
    }
    cp_async_commit();
  };
  fetch(0);
  for (int p = 0; p < K; ++p) {
    cp_async_wait_all();
    __syncthreads();
    for (int e = threadIdx.x; e < ncols * S; e += NT) {
      const int cc = e / S, t = e - cc * S;
      const int r = t - oh;
      const int pos = (r < 0 || r >= Hi) ? t + S : t;
      const float2 v = raw[cc * LD + t];
      work[(2 * cc) * LD + t] = v;
      work[(2 * cc + 1) * LD + t] = cmul(v, __ldg(&twP[pos]));
    }
    __syncthreads();
    if (p + 1 < K) fetch(p + 1);
    static_fft_forward_head<S>(work, 2 * ncols, LD, tw);
    static_last_forward_mul_acc<S>(work, spec, 2 * ncols, LD, table + (size_t)(p * C + c) * P * P, q0, p == 0);
  }
  __syncthreads();
  static_fft_inverse<S>(spec, 2 * ncols, LD, tw);
  float2* Bout = B + (size_t)c * Ho * P;
  for (int e = threadIdx.x; e < Ho * ncols; e += NT) {
    const int rr = e / ncols, cc = e - rr * ncols;
    const int n = oc + rr;
    const int t = n >= S ? n - S : n;
    Bout[(size_t)rr * P + q0 + cc] = cadd(spec[(2 * cc) * LD + t], cmul(cconj(__ldg(&twP[n])), spec[(2 * cc + 1) * LD + t]));
  }
}

// Adjoint column pass with the same table: the column of A[c] is transformed once, then
// for every plane p the spectrum times conj(H[p, c]) (the transfer function of distance
// -d_p) is inverse-transformed, cropped and written to B[p * C + c].
// Shared memory: 2 COLS spectrum lines and 2 COLS work lines (stride S+1).
template <int S, int COLS, int NT>
__global__ void __launch_bounds__(NT) columns_scatter_table_s(const float2* __restrict__ A, int Hi,
                                                             float2* __restrict__ B, int Ho,
                                                             const float2* __restrict__ tw,
                                                             const float2* __restrict__ twP,
                                                             const float2* __restrict__ table, int K, int C) {
  extern __shared__ float2 sm[];
  constexpr int P = 2 * S;
  constexpr int LD = S + 1;
  float2* work = sm;
  float2* spec = sm + 2 * COLS * LD;
  const int c = blockIdx.y;
  const int q0 = blockIdx.x * COLS;
  const int ncols = min(COLS, P - q0);
  const int oh = (P - Hi) / 2, oc = (P - Ho) / 2;
  const float2* Ain = A + (size_t)c * Hi * P + q0;
  for (int e = threadIdx.x; e < ncols * S; e += NT) {
    const int t = e / ncols, cc = e - t * ncols;
    int r = t - oh;
    if (r < 0 || r >= Hi) r = t + S - oh;
    float2* dst = spec + (2 * cc) * LD + t;
    if (r >= 0 && r < Hi) cp_async8(dst, Ain + (size_t)r * P + cc);
    else *dst = make_float2(0.f, 0.f);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  for (int e = threadIdx.x; e < ncols * S; e += NT) {
    const int cc = e / S, t = e - cc * S;
    const int r = t - oh;
    const int pos = (r < 0 || r >= Hi) ? t + S : t;
    spec[(2 * cc + 1) * LD + t] = cmul(spec[(2 * cc) * LD + t], __ldg(&twP[pos]));
  }
  __syncthreads();
  static_fft_forward<S>(spec, 2 * ncols, LD, tw);
  for (int p = 0; p < K; ++p) {
    static_first_inverse_mul<S>(spec, work, 2 * ncols, LD, table + (size_t)(p * C + c) * P * P, q0);
    __syncthreads();
    static_fft_inverse_rest<S>(work, 2 * ncols, LD, tw);
    float2* Bout = B + (size_t)(p * C + c) * Ho * P;
    for (int e = threadIdx.x; e < Ho * ncols; e += NT) {
      const int rr = e / ncols, cc = e - rr * ncols;
      const int n = oc + rr;
      const int t = n >= S ? n - S : n;
      Bout[(size_t)rr * P + q0 + cc] = cadd(work[(2 * cc) * LD + t], cmul(cconj(__ldg(&twP[n])), work[(2 * cc + 1) * LD + t]));
    }
    __syncthreads();
  }
}

constexpr size_t kStaticSmem = 64 * 1024;

template <int S>
int static_lines(size_t extra_per_line, size_t budget = kStaticSmem) {
  const size_t per = 2 * (size_t)S * sizeof(float2) + extra_per_line;
  int r = (int)(budget / per);
  int p2 = 1;
  while (p2 * 2 <= r && p2 < 8) p2 *= 2;
  return p2;
}

template <int S>
int run_rows_forward(const float2* in, int total_rows, int Wi, float2* A, const float2* tw, const float2* twP,
                     cudaStream_t st) {
  const int rows = static_lines<S>(0);
  const size_t smem = (size_t)rows * 2 * S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(rows_forward_s<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rows_forward_s<S><<<(total_rows + rows - 1) / rows, kThreads, smem, st>>>(in, total_rows, Wi, A, tw, twP, rows);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_columns(const float2* A, int Hi, float2* B, int Ho, const float2* tw, const float2* twP, const int* digrev,
                const SumJobs& jobs, int njobs, cudaStream_t st) {
  const int cols = static_lines<S>((size_t)S * sizeof(float2) + 16, 100 * 1024);  // + Ho x cols accumulator (Ho <= S)
  const size_t smem = (size_t)cols * 2 * (S + 1) * sizeof(float2) + (size_t)cols * S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(columns_s<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((2 * S + cols - 1) / cols, njobs);
  columns_s<S><<<grid, kThreads, smem, st>>>(A, Hi, B, Ho, tw, twP, digrev, cols, jobs);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_rows_inverse(const float2* B, int total_rows, float2* out, int Wo, const float2* tw, const float2* twP,
                     int accumulate, cudaStream_t st) {
  const int rows = static_lines<S>(0);
  const size_t smem = (size_t)rows * 2 * S * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(rows_inverse_s<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const float P = 2.0f * S;
  rows_inverse_s<S><<<(total_rows + rows - 1) / rows, kThreads, smem, st>>>(B, total_rows, out, Wo, tw, twP, rows,
                                                                            1.0f / (P * P), accumulate);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_transfer_table(float2* table, const int* digrev, const TransferTable& tt, int items, cudaStream_t st) {
  const size_t n = (size_t)4 * S * S;
  const size_t nb = (n + kThreads - 1) / kThreads;
  dim3 grid((unsigned)(nb < 1184 ? nb : 1184), items);
  transfer_table_s<S><<<grid, kThreads, 0, st>>>(table, digrev, tt);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_transfer_upload(float2* table, const int* digrev, const float2* Hc, int items, cudaStream_t st) {
  const size_t n = (size_t)4 * S * S;
  const size_t nb = (n + kThreads - 1) / kThreads;
  dim3 grid((unsigned)(nb < 1184 ? nb : 1184), items);
  transfer_upload_s<S><<<grid, kThreads, 0, st>>>(table, digrev, Hc);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

// Columns per CTA and threads of the table column passes at S = 1024 (build-time choice).
#ifndef CVHRF_TABLE_COLS_1024
#define CVHRF_TABLE_COLS_1024 1
#endif
#ifndef CVHRF_TABLE_NT_1024
#define CVHRF_TABLE_NT_1024 128
#endif

template <int S>
int run_columns_table(bool adjoint, const float2* A, int Hi, float2* B, int Ho, const float2* tw, const float2* twP,
                      const float2* table, int K, int C, cudaStream_t st) {
  // columns per CTA and threads, measured on B200: 3 columns (96 KB, two CTAs per SM) below
  // 1024; one column above, with 128 threads where the radix-32 stages have 64 or 128
  // butterflies per line pair (1024, 2048) and 256 for 1920 (its radix-2 stage is wide)
  constexpr int COLS = S == 1024 ? CVHRF_TABLE_COLS_1024 : (S > 1024 ? 1 : 3);
  constexpr int NT = S == 1024 ? CVHRF_TABLE_NT_1024 : (S == 2048 ? 128 : 256);
  dim3 grid((2 * S + COLS - 1) / COLS, C);
  if (!adjoint) {
    const size_t smem = (size_t)COLS * 5 * (S + 1) * sizeof(float2);
    CVHRF_CUDA_TRY(cudaFuncSetAttribute(columns_sum_table_s<S, COLS, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    columns_sum_table_s<S, COLS, NT><<<grid, NT, smem, st>>>(A, Hi, B, Ho, tw, twP, table, K, C);
  } else {
    const size_t smem = (size_t)COLS * 4 * (S + 1) * sizeof(float2);
    CVHRF_CUDA_TRY(cudaFuncSetAttribute(columns_scatter_table_s<S, COLS, NT>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    columns_scatter_table_s<S, COLS, NT><<<grid, NT, smem, st>>>(A, Hi, B, Ho, tw, twP, table, K, C);
  }
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

}  // namespace

bool static_fft_size(int S) {
  switch (S) {
    case 64: case 128: case 256: case 384: case 512: case 800: case 1024: case 1920: case 2048: return true;
    default: return false;
  }
}

void static_fft_radices(int S, int* radix, int* nst) {
#define CVHRF_PLAN(SS) \
  case SS: radix[0] = StaticPlan<SS>::r0; radix[1] = StaticPlan<SS>::r1; radix[2] = StaticPlan<SS>::r2; \
    *nst = StaticPlan<SS>::nst; break;
  switch (S) {
    CVHRF_PLAN(64) CVHRF_PLAN(128) CVHRF_PLAN(256) CVHRF_PLAN(384) CVHRF_PLAN(512) CVHRF_PLAN(800)
    CVHRF_PLAN(1024) CVHRF_PLAN(1920) CVHRF_PLAN(2048)
    default: *nst = 0;
  }
#undef CVHRF_PLAN
}

int static_rows_forward(const FftDesc& d, const float2* in, int total_rows, int Wi, float2* A, cudaStream_t st) {
#define CALL run_rows_forward
#define ARGS (in, total_rows, Wi, A, d.tw, d.twP, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

int static_columns(const FftDesc& d, const float2* A, int Hi, float2* B, int Ho, const SumJobs& jobs, int njobs,
                   cudaStream_t st) {
#define CALL run_columns
#define ARGS (A, Hi, B, Ho, d.tw, d.twP, d.digrev, jobs, njobs, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

int static_rows_inverse(const FftDesc& d, const float2* B, int total_rows, float2* out, int Wo, int accumulate,
                        cudaStream_t st) {
#define CALL run_rows_inverse
#define ARGS (B, total_rows, out, Wo, d.tw, d.twP, accumulate, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

int static_transfer_table(const FftDesc& d, float2* table, const TransferTable& tt, int items, cudaStream_t st) {
#define CALL run_transfer_table
#define ARGS (table, d.digrev, tt, items, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

int static_transfer_upload(const FftDesc& d, float2* table, const float2* centred, int items, cudaStream_t st) {
#define CALL run_transfer_upload
#define ARGS (table, d.digrev, centred, items, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

int static_columns_table(const FftDesc& d, bool adjoint, const float2* A, int Hi, float2* B, int Ho,
                         const float2* table, int K, int C, cudaStream_t st) {
#define CALL run_columns_table
#define ARGS (adjoint, A, Hi, B, Ho, d.tw, d.twP, table, K, C, st)
  switch (d.S) {
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return CALL<800> ARGS;
    case 1024: return CALL<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS;
    default: return CVHRF_EUNSUPPORTED;
  }
#undef CALL
#undef ARGS
}

}  // namespace cvhrf
