// Shared pieces of the propagation passes: transfer-function constants and evaluation,
// and the compile-time-size (static) pass entry points of asm_static.cu.
#pragma once
#include <math.h>
#include "fft_lines.cuh"

namespace cvhrf {

struct TransferParams {
  float k;          // (float)(2 pi / lambda), computed in double as the reference host code does
  float distance;
  float fx_max, fy_max;
  float inv_np;     // (float)(1 / (P * pitch)): torch.fft.fftfreq scale
  float aperture;   // radius in shifted index space; <= 0 disables
  float offset_x, offset_y;
};

// Host-side constants of bandlimited_propagation_cuda.cu:149-170 (float arithmetic,
// k via double), for a square padded grid of side P.
inline TransferParams make_transfer(float wavelength, float pitch, float distance, float aperture, int P) {
  TransferParams t;
  t.k = (float)(2.0f * M_PI / wavelength);
  const float x_size = pitch * P;
  const float y_size = pitch * P;
  const float ax = 2.0f * distance * (1.0f / x_size);
  const float ay = 2.0f * distance * (1.0f / y_size);
  t.fx_max = 1.0f / sqrtf(ax * ax + 1.0f) / wavelength;
  t.fy_max = 1.0f / sqrtf(ay * ay + 1.0f) / wavelength;
  t.distance = distance;
  t.inv_np = (float)(1.0 / ((double)P * (double)pitch));
  t.aperture = aperture;
  t.offset_x = P / 2.0f - 0.5f;
  t.offset_y = P / 2.0f - 0.5f;
  return t;
}

// Transfer function x aperture at unshifted bin (ku = row, kv = column) of a P x P
// grid.  Row bins carry FX (meshgrid 'ij', python_function.py:137-142), column bins FY.
// The expressions follow bandlimited_propagation_cuda.cu:50-85 term by term (kz^2 in
// double, stored to float, sqrtf, phase = d*kz, accurate sincosf); the aperture test is
// on shifted indices (i + P/2) mod P.
__device__ __forceinline__ float2 transfer_at(int ku, int kv, int P, const TransferParams& tp) {
  const int half = P >> 1;
  const float fx_val = __fmul_rn((float)(ku < half ? ku : ku - P), tp.inv_np);
  const float fy_val = __fmul_rn((float)(kv < half ? kv : kv - P), tp.inv_np);
  const bool within_bandlimit = (fabsf(fx_val) < tp.fx_max) && (fabsf(fy_val) < tp.fy_max);
  const float k = tp.k;
  const float kz_squared = k * k - (2 * M_PI * fx_val) * (2 * M_PI * fx_val) - (2 * M_PI * fy_val) * (2 * M_PI * fy_val);
  float2 tr = make_float2(0.0f, 0.0f);
  if (kz_squared > 0.0f && within_bandlimit) {
    const float kz = sqrtf(kz_squared);
    const float phase = tp.distance * kz;
    float s, c;
    sincosf(phase, &s, &c);
    tr = make_float2(c, s);
  }
  if (tp.aperture > 0.0f) {
    const int idx = (kv + half) % P;  // shifted column index
    const int idy = (ku + half) % P;  // shifted row index
    const float x = (float)idx - tp.offset_x;
    const float y = (float)idy - tp.offset_y;
    const float r = tp.aperture;
    const float m = (x * x + y * y < r * r) ? 1.0f : 0.0f;
    tr.x *= m;
    tr.y *= m;
  }
  return tr;
}

// transfer_at split by axis for a column pass, where the column bin kv is fixed per line:
// the column's terms are formed once (TransferCol) and each row bin adds its own.  Same
// operations and operand order as transfer_at, so the values are the same.
struct TransferCol {
  double fy2pi;   // 2 pi fy in double
  float fy_abs;
  int idx;        // shifted column index
};
__device__ __forceinline__ TransferCol transfer_col(int kv, int P, const TransferParams& tp) {
  const int half = P >> 1;
  const float fy_val = __fmul_rn((float)(kv < half ? kv : kv - P), tp.inv_np);
  TransferCol c;
  c.fy2pi = 2 * M_PI * fy_val;
  c.fy_abs = fabsf(fy_val);
  c.idx = (kv + half) % P;
  return c;
}
__device__ __forceinline__ float2 transfer_row(int ku, int P, const TransferCol& col, const TransferParams& tp) {
  const int half = P >> 1;
  const float fx_val = __fmul_rn((float)(ku < half ? ku : ku - P), tp.inv_np);
  const bool within_bandlimit = (fabsf(fx_val) < tp.fx_max) && (col.fy_abs < tp.fy_max);
  const float k = tp.k;
  const float kz_squared = k * k - (2 * M_PI * fx_val) * (2 * M_PI * fx_val) - col.fy2pi * col.fy2pi;
  float2 tr = make_float2(0.0f, 0.0f);
  if (kz_squared > 0.0f && within_bandlimit) {
    const float kz = sqrtf(kz_squared);
    const float phase = tp.distance * kz;
    float s, c;
    sincosf(phase, &s, &c);
    tr = make_float2(c, s);
  }
  if (tp.aperture > 0.0f) {
    const int idy = (ku + half) % P;  // shifted row index
    const float x = (float)col.idx - tp.offset_x;
    const float y = (float)idy - tp.offset_y;
    const float r = tp.aperture;
    const float m = (x * x + y * y < r * r) ? 1.0f : 0.0f;
    tr.x *= m;
    tr.y *= m;
  }
  return tr;
}

// Transfer parameters of up to kMaxTableItems table items (item = p * C + c).
constexpr int kMaxTableItems = 64;
struct TransferTable {
  TransferParams tp[kMaxTableItems];
};

// What a column pass computes.  Sum form: output item item[j] = sum over k < n[j] of the
// propagation of input item items[j][k] (spectrum times H).  Scatter form: input item
// item[j] goes to the n[j] output items items[j][k] (spectrum times conj(H): the adjoint).  Term (j, k) uses transfer function tpi[j][k]: an index
// into tp, or, with a precomputed table, the table item.
constexpr int kMaxColJobs = 32;
constexpr int kMaxColTerms = 64;
struct ColPlan {
  int njobs;
  int item[kMaxColJobs];
  int n[kMaxColJobs];
  short items[kMaxColJobs][kMaxColTerms];
  short tpi[kMaxColJobs][kMaxColTerms];
  TransferParams tp[kMaxTableItems];
};

// The compile-time-size passes keep their intermediate spectra transposed: item-major,
// then spectrum column q (2S of them), then row, with a column stride of
// col_stride(rows) elements (a multiple of 4, so every column starts 32-byte aligned).
__host__ __device__ inline int col_stride(int rows) { return (rows + 3) & ~3; }

// Sizes with a compile-time plan (the rest use the runtime plan of asm_propagation.cu).
bool static_fft_size(int S);
// Stage radices of the static plan (radix[0..2], *nst stages) for the digit-reversal table.
void static_fft_radices(int S, int* radix, int* nst);
// items x Hi rows of width Wi -> transposed spectra A (items x 2S columns x col_stride(Hi)).
int static_rows_forward(const FftDesc& d, const float2* in, int items, int Hi, int Wi, float2* A, cudaStream_t st);
// Column pass, sum or scatter form; `table` (nullable) replaces the evaluated transfer function.
int static_columns(const FftDesc& d, bool scatter, const float2* A, int Hi, float2* B, int Ho, const ColPlan& plan,
                   const float2* table, cudaStream_t st);
// Transposed spectra B (items x 2S columns x col_stride(Ho)) -> items x Ho rows of width Wo.
int static_rows_inverse(const FftDesc& d, const float2* B, int items, int Ho, float2* out, int Wo, int accumulate,
                        cudaStream_t st);
// Precomputed transfer tables (items x P x P complex64, column-pass layout).
int static_transfer_table(const FftDesc& d, float2* table, const TransferTable& tt, int items, cudaStream_t st);
// Table from a caller-supplied transfer function in centred (fftshifted) order, items x P x P.
int static_transfer_upload(const FftDesc& d, float2* table, const float2* centred, int items, cudaStream_t st);
// Device-side count of bulk-copy waits that gave up (each sets the result invalid).
int static_copy_wait_timeouts();

}  // namespace cvhrf
