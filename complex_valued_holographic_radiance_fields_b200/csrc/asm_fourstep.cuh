// Propagation passes for S = 800 and S = 1024 on the register-resident four-step FFT
// (fft_fourstep.cuh).  Included by asm_static.cu only.
//
// Same operator, layouts and entry points as the warp-line passes of asm_static.cu
// (transposed intermediates, one warp per transform line), with three differences:
//   * a line lives in registers (M = S / 32 values per lane) and is transformed with one
//     shared-memory transpose, so an 800-point line costs about half the instructions;
//   * spectra are in natural bin order (the plan's digit-reversal table is the identity
//     for these sizes), spectrum column q holds row bin 2 (q mod S) + (q >= S);
//   * the column passes accumulate the K-plane spectrum sum in registers and stage both
//     the columns and, with a precomputed table, the matching transfer-table slice with
//     double-buffered bulk copies (TMA): the copies for plane k + 2 are in flight while
//     plane k + 1's data is consumed.
#pragma once
#include "asm_static.cuh"
#include "fft_fourstep.cuh"

namespace cvhrf {
namespace {

constexpr int kFsRows = 4;   // rows per block in the row passes (one warp each)
constexpr int kFsCols = 2;   // columns per block in the column passes (two warps each)

// First row-pass input position: line position t holds input column t - ow, or
// t + S - ow for the wrapped part; pos is the 2S index (t or t + S).
template <int S>
__device__ __forceinline__ void fs_fold_index(int t, int ow, int W, int& j, int& pos) {
  j = t - ow;
  pos = t;
  if (j < 0 || j >= W) {
    j = t + S - ow;
    pos = t + S;
  }
}

// The four-step twiddles w_S^(k2 n1) (k2 < M, n1 < 32) staged in shared memory in the
// transpose's swizzled layout, entry (k2, n1) at fs_tslot(k2, n1): the forward reads a
// fixed k2 across lanes n1, the inverse a fixed n1 across lanes k2, both conflict-free.
// (Read from global memory they would be evicted from L1 by the streamed data.)
template <int S>
__device__ __forceinline__ void fs_stage_roots(float2* dst, const float2* __restrict__ tw) {
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    const int k2 = i >> 5, n1 = i & 31;
    dst[fs_tslot(k2, n1)] = __ldg(&tw[k2 * n1]);
  }
}

// Crop window [oc, oc + n) of the 2S-periodic inverse: the output index n of line
// position t (t or t + S), or -1 when neither lies in the window.
__device__ __forceinline__ int fs_crop(int t, int S, int oc, int n) {
  if (t >= oc && t < oc + n) return t;
  if (t + S >= oc && t + S < oc + n) return t + S;
  return -1;
}

// Row passes: a block takes kFsRows rows; warp w handles half-line h = w & 1 of row
// r = w >> 1.  The block's spectra live in one tile [2S][kFsRows + 1] (row r of spectrum
// column q at q (kFsRows + 1) + r); the warp's own strided slice of the tile (its row,
// its half) doubles as the four-step transpose buffer, so the tile is all the shared
// memory a block uses.
template <int S>
__global__ void __launch_bounds__(2 * kFsRows * 32) fs_rows_fwd(const float2* __restrict__ in, int items, int Hi,
                                                               int Wi, float2* __restrict__ A,
                                                               const float2* __restrict__ tw,
                                                               const float2* __restrict__ twP) {
  constexpr int M = S / 32, P = 2 * S, TL = kFsRows + 1;
  extern __shared__ __align__(16) float2 sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = warp >> 1, h = warp & 1;
  float2* region = sm + (h * S) * TL + r;              // this warp's S slots, stride TL
  float2* roots = sm + P * TL;
  const int total = items * Hi;
  const int row0 = blockIdx.x * kFsRows;
  const int g = row0 + r;
  const bool valid = g < total;
  const int ow = (P - Wi) / 2;
  const float2* src = in + (size_t)(valid ? g : 0) * Wi;
  float2 x[M], y[32];
#pragma unroll
  for (int j = 0; j < M; ++j) {
    int jj, pos;
    fs_fold_index<S>(lane + 32 * j, ow, Wi, jj, pos);
    float2 v = make_float2(0.f, 0.f);
    if (valid && jj >= 0 && jj < Wi) v = __ldcs(&src[jj]);
    x[j] = h ? pmul(v, __ldg(&twP[pos])) : v;
  }
  fs_stage_roots<S>(roots, tw);
  __syncthreads();
  fs_forward<S>(x, y, region, TL, lane, roots);
  if (lane < M) {
#pragma unroll
    for (int k1 = 0; k1 < 32; ++k1) region[(lane + M * k1) * TL] = y[k1];
  }
  __syncthreads();
  const int HiS = col_stride(Hi);
  for (int e = threadIdx.x; e < kFsRows * P; e += 2 * kFsRows * 32) {
    const int q = e / kFsRows, rr0 = e - q * kFsRows;
    const int gg = row0 + rr0;
    if (gg >= total) continue;
    const int item = gg / Hi, rr = gg - item * Hi;
    A[((size_t)item * P + q) * HiS + rr] = sm[q * TL + rr0];
  }
}

template <int S>
__global__ void __launch_bounds__(2 * kFsRows * 32) fs_rows_inv(const float2* __restrict__ B, int items, int Ho,
                                                               float2* __restrict__ out, int Wo,
                                                               const float2* __restrict__ tw,
                                                               const float2* __restrict__ twP, float scale,
                                                               int accumulate) {
  constexpr int M = S / 32, P = 2 * S, TL = kFsRows + 1;
  extern __shared__ __align__(16) float2 sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = warp >> 1, h = warp & 1;
  float2* region = sm + (h * S) * TL + r;
  float2* roots = sm + P * TL;
  fs_stage_roots<S>(roots, tw);
  const int total = items * Ho;
  const int row0 = blockIdx.x * kFsRows;
  const int HoS = col_stride(Ho);
  for (int e = threadIdx.x; e < kFsRows * P; e += 2 * kFsRows * 32) {
    const int q = e / kFsRows, rr0 = e - q * kFsRows;
    const int gg = row0 + rr0;
    float2* dst = sm + q * TL + rr0;
    if (gg < total) {
      const int item = gg / Ho, rr = gg - item * Ho;
      cp_async8(dst, B + ((size_t)item * P + q) * HoS + rr);
    } else {
      *dst = make_float2(0.f, 0.f);
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  const int g = row0 + r;
  float2 x[M], y[32];
  if (lane < M) {
#pragma unroll
    for (int k1 = 0; k1 < 32; ++k1) y[k1] = region[(lane + M * k1) * TL];
  }
  fs_inverse<S>(y, x, region, TL, lane, roots);
  if (h) {                                 // the odd half-line goes to the even warp
#pragma unroll
    for (int j = 0; j < M; ++j) region[(lane + 32 * j) * TL] = x[j];
  }
  __syncthreads();
  if (h || g >= total) return;
  const float2* odd = sm + S * TL + r;
  const int oc = (P - Wo) / 2;
  float2* dst = out + (size_t)g * Wo;
#pragma unroll
  for (int j = 0; j < M; ++j) {
    const int t = lane + 32 * j;
    const int n = fs_crop(t, S, oc, Wo);
    if (n < 0) continue;
    float2 v = padd(x[j], pmul(cconj(__ldg(&twP[n])), odd[t * TL]));
    v = pscale(scale, v);
    float2* d = dst + (n - oc);
    if (accumulate) v = padd(*d, v);
    *d = v;
  }
}

// Shared-memory plan of the column passes (float2 offsets; every buffer 16-byte aligned).
template <int S>
struct FsColSmem {
  static constexpr int M = S / 32;
  static constexpr int STAGE = kFsCols * (S + 4);      // one buffer of staged columns
  static constexpr int HSLICE = kFsCols * 2 * S;       // one transfer-table slice
  static constexpr int stage(int b) { return b * STAGE; }
  static constexpr int hbuf(int b) { return 2 * STAGE + b * HSLICE; }
  static constexpr int tbuf(bool table) { return 2 * STAGE + (table ? 2 * HSLICE : 0); }
  static constexpr int roots(bool table) { return tbuf(table) + 2 * kFsCols * M * 32; }
  static constexpr size_t bytes(bool table) {
    return (size_t)(roots(table) + S) * sizeof(float2);
  }
};

// Fold the staged column (rows r < Hi of spectrum column cc) into this warp's half-line:
// position t = lane + 32 j holds row t - oh (or the wrapped t + S - oh); the odd
// half-line is multiplied by w_2S^n.
template <int S>
__device__ __forceinline__ void fs_fold_column(float2 (&x)[S / 32], const float2* col, int Hi, int h, int lane,
                                               const float2* __restrict__ twP) {
  constexpr int M = S / 32, P = 2 * S;
  const int oh = (P - Hi) / 2;
#pragma unroll
  for (int j = 0; j < M; ++j) {
    int r, pos;
    fs_fold_index<S>(lane + 32 * j, oh, Hi, r, pos);
    float2 v = make_float2(0.f, 0.f);
    if (r >= 0 && r < Hi) v = col[r];
    x[j] = h ? pmul(v, __ldg(&twP[pos])) : v;
  }
}

template <int S, bool TABLE>
__global__ void __launch_bounds__(2 * kFsCols * 32) fs_cols_sum(const float2* __restrict__ A, int Hi,
                                                               float2* __restrict__ B, int Ho, const ColPlan plan,
                                                               const float2* __restrict__ table,
                                                               const float2* __restrict__ tw,
                                                               const float2* __restrict__ twP) {
  using L = FsColSmem<S>;
  constexpr int M = S / 32, P = 2 * S;
  extern __shared__ __align__(16) float2 sm[];
  __shared__ uint64_t bar[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cc = warp >> 1, h = warp & 1;
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * kFsCols;
  const int ncols = min(kFsCols, P - q0);
  const bool active = cc < ncols;
  const int q = q0 + (active ? cc : 0);
  const int HiS = col_stride(Hi), HoS = col_stride(Ho);
  float2* T = sm + L::tbuf(TABLE) + warp * M * 32;
  float2* roots = sm + L::roots(TABLE);
  fs_stage_roots<S>(roots, tw);
  const int K = plan.n[job];
  const unsigned abytes = (unsigned)(ncols * HiS * sizeof(float2));
  const unsigned hbytes = TABLE ? (unsigned)(ncols * 2 * S * sizeof(float2)) : 0u;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int k) {
    const int b = k & 1;
    mbar_arrive_expect_tx(&bar[b], abytes + hbytes);
    bulk_copy_g2s(sm + L::stage(b), A + ((size_t)plan.items[job][k] * P + q0) * HiS, abytes, &bar[b]);
    if constexpr (TABLE)
      bulk_copy_g2s(sm + L::hbuf(b), table + (size_t)plan.tpi[job][k] * P * P + (size_t)q0 * 2 * S, hbytes, &bar[b]);
  };
  if (threadIdx.x == 0) {
    issue(0);
    if (K > 1) issue(1);
  }
  // the column bin of this warp's column (natural order: column q is bin 2 (q mod S) + (q >= S))
  const int kv = 2 * (q >= S ? q - S : q) + (q >= S ? 1 : 0);
  float2 x[M], y[32], acc[32];
#pragma unroll
  for (int k1 = 0; k1 < 32; ++k1) acc[k1] = make_float2(0.f, 0.f);
  for (int k = 0; k < K; ++k) {
    const int b = k & 1;
    wait_copies(&bar[b], (k >> 1) & 1);
    if (active) {
      fs_fold_column<S>(x, sm + L::stage(b) + cc * HiS, Hi, h, lane, twP);
      fs_forward<S>(x, y, T, 1, lane, roots);
      if (lane < M) {
        if constexpr (TABLE) {
          const float2* Hl = sm + L::hbuf(b) + (cc * 2 + h) * S + lane;
#pragma unroll
          for (int k1 = 0; k1 < 32; ++k1) acc[k1] = padd(acc[k1], pmul(y[k1], Hl[M * k1]));
        } else {
          const TransferParams tp = plan.tp[plan.tpi[job][k]];
          const TransferCol col = transfer_col(kv, P, tp);
#pragma unroll
          for (int k1 = 0; k1 < 32; ++k1)
            acc[k1] = padd(acc[k1], pmul(y[k1], transfer_row(2 * (lane + M * k1) + h, P, col, tp)));
        }
      }
    }
    __syncthreads();                       // buffer b is consumed by every warp
    if (threadIdx.x == 0 && k + 2 < K) {
      fence_proxy_async_smem();
      issue(k + 2);
    }
  }
  float2* comb = sm + L::stage(0);         // free now: the odd half-lines of the block
  if (active) {
    fs_inverse<S>(acc, x, T, 1, lane, roots);
    if (h) {
#pragma unroll
      for (int j = 0; j < M; ++j) comb[cc * S + lane + 32 * j] = x[j];
    }
  }
  __syncthreads();
  if (!active || h) return;
  const int oc = (P - Ho) / 2;
  float2* Bout = B + ((size_t)plan.item[job] * P + q) * HoS;
#pragma unroll
  for (int j = 0; j < M; ++j) {
    const int t = lane + 32 * j;
    const int n = fs_crop(t, S, oc, Ho);
    if (n < 0) continue;
    Bout[n - oc] = padd(x[j], pmul(cconj(__ldg(&twP[n])), comb[cc * S + t]));
  }
}

template <int S, bool TABLE>
__global__ void __launch_bounds__(2 * kFsCols * 32) fs_cols_scatter(const float2* __restrict__ A, int Hi,
                                                                   float2* __restrict__ B, int Ho,
                                                                   const ColPlan plan,
                                                                   const float2* __restrict__ table,
                                                                   const float2* __restrict__ tw,
                                                                   const float2* __restrict__ twP) {
  using L = FsColSmem<S>;
  constexpr int M = S / 32, P = 2 * S;
  extern __shared__ __align__(16) float2 sm[];
  __shared__ uint64_t bar[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cc = warp >> 1, h = warp & 1;
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * kFsCols;
  const int ncols = min(kFsCols, P - q0);
  const bool active = cc < ncols;
  const int q = q0 + (active ? cc : 0);
  const int HiS = col_stride(Hi), HoS = col_stride(Ho);
  float2* T = sm + L::tbuf(TABLE) + warp * M * 32;
  float2* roots = sm + L::roots(TABLE);
  fs_stage_roots<S>(roots, tw);
  const int K = plan.n[job];
  const unsigned abytes = (unsigned)(ncols * HiS * sizeof(float2));
  const unsigned hbytes = TABLE ? (unsigned)(ncols * 2 * S * sizeof(float2)) : 0u;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  // bar[0]: the input columns (+ table slice 0); bar[b]: table slice k for k & 1 == b
  auto issue_h = [&](int k) {
    const int b = k & 1;
    mbar_arrive_expect_tx(&bar[b], hbytes + (k == 0 ? abytes : 0u));
    if (k == 0) bulk_copy_g2s(sm + L::stage(0), A + ((size_t)plan.item[job] * P + q0) * HiS, abytes, &bar[0]);
    if constexpr (TABLE)
      bulk_copy_g2s(sm + L::hbuf(b), table + (size_t)plan.tpi[job][k] * P * P + (size_t)q0 * 2 * S, hbytes, &bar[b]);
  };
  if (threadIdx.x == 0) {
    issue_h(0);
    if (TABLE && K > 1) issue_h(1);
  }
  const int kv = 2 * (q >= S ? q - S : q) + (q >= S ? 1 : 0);
  float2 x[M], y[32], z[32];
  wait_copies(&bar[0], 0);
  if (active) {
    fs_fold_column<S>(x, sm + L::stage(0) + cc * HiS, Hi, h, lane, twP);
    fs_forward<S>(x, y, T, 1, lane, roots);
  }
  __syncthreads();                         // the staged input is consumed: it becomes comb
  float2* comb = sm + L::stage(0);
  const int oc = (P - Ho) / 2;
  for (int k = 0; k < K; ++k) {
    const int b = k & 1;
    if (TABLE && k > 0) wait_copies(&bar[b], (k >> 1) & 1);
    if (active) {
      if (lane < M) {
        if constexpr (TABLE) {
          const float2* Hl = sm + L::hbuf(b) + (cc * 2 + h) * S + lane;
#pragma unroll
          for (int k1 = 0; k1 < 32; ++k1) z[k1] = pmul(y[k1], cconj(Hl[M * k1]));
        } else {
          const TransferParams tp = plan.tp[plan.tpi[job][k]];
          const TransferCol col = transfer_col(kv, P, tp);
#pragma unroll
          for (int k1 = 0; k1 < 32; ++k1)
            z[k1] = pmul(y[k1], cconj(transfer_row(2 * (lane + M * k1) + h, P, col, tp)));
        }
      }
      fs_inverse<S>(z, x, T, 1, lane, roots);
      if (h) {
#pragma unroll
        for (int j = 0; j < M; ++j) comb[cc * S + lane + 32 * j] = x[j];
      }
    }
    __syncthreads();
    if (active && !h) {
      float2* Bout = B + ((size_t)plan.items[job][k] * P + q) * HoS;
#pragma unroll
      for (int j = 0; j < M; ++j) {
        const int t = lane + 32 * j;
        const int n = fs_crop(t, S, oc, Ho);
        if (n < 0) continue;
        Bout[n - oc] = padd(x[j], pmul(cconj(__ldg(&twP[n])), comb[cc * S + t]));
      }
    }
    __syncthreads();                       // comb and table slice b are consumed
    if (TABLE && threadIdx.x == 0 && k + 2 < K) {
      fence_proxy_async_smem();
      issue_h(k + 2);
    }
  }
}

template <int S>
int fs_run_rows_forward(const float2* in, int items, int Hi, int Wi, float2* A, const float2* tw, const float2* twP,
                        cudaStream_t st) {
  const int total = items * Hi;
  const size_t smem = (size_t)(2 * S * (kFsRows + 1) + S) * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(fs_rows_fwd<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  fs_rows_fwd<S><<<(total + kFsRows - 1) / kFsRows, 2 * kFsRows * 32, smem, st>>>(in, items, Hi, Wi, A, tw, twP);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int fs_run_rows_inverse(const float2* B, int items, int Ho, float2* out, int Wo, const float2* tw, const float2* twP,
                        int accumulate, cudaStream_t st) {
  const int total = items * Ho;
  const size_t smem = (size_t)(2 * S * (kFsRows + 1) + S) * sizeof(float2);
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(fs_rows_inv<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const float P = 2.0f * S;
  fs_rows_inv<S><<<(total + kFsRows - 1) / kFsRows, 2 * kFsRows * 32, smem, st>>>(B, items, Ho, out, Wo, tw, twP,
                                                                                1.0f / (P * P), accumulate);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int fs_run_columns(bool scatter, const float2* A, int Hi, float2* B, int Ho, const ColPlan& plan, const float2* table,
                   const float2* tw, const float2* twP, cudaStream_t st) {
  const bool tab = table != nullptr;
  const size_t smem = FsColSmem<S>::bytes(tab);
  dim3 grid((2 * S + kFsCols - 1) / kFsCols, plan.njobs);
  auto launch = [&](auto kern) -> int {
    CVHRF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, 2 * kFsCols * 32, smem, st>>>(A, Hi, B, Ho, plan, table, tw, twP);
    CVHRF_LAUNCH_CHECK();
    return CVHRF_OK;
  };
  if (scatter) return tab ? launch(fs_cols_scatter<S, true>) : launch(fs_cols_scatter<S, false>);
  return tab ? launch(fs_cols_sum<S, true>) : launch(fs_cols_sum<S, false>);
}

}  // namespace
}  // namespace cvhrf
