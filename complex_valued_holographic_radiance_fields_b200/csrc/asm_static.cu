// Propagation passes specialised for compile-time line lengths (S = 64 ... 2048).
//
// The operator and its arithmetic are those of asm_propagation.cu: rows forward; columns
// with the band-limited transfer function; rows inverse with the crop.  The layout and
// the work split are built for the B200 memory system:
//
//   * The intermediate spectra are stored TRANSPOSED (item, column q, row): the row pass
//     writes each column's rows as 32- or 64-byte runs, the column pass reads and writes
//     whole contiguous columns, and the inverse row pass reads the runs back.  Every DRAM
//     sector moved carries only useful bytes.
//   * The column pass stages its columns with bulk asynchronous copies (TMA
//     cp.async.bulk, completion on an mbarrier): one thread issues a block's whole
//     column group for the next plane while the warps transform the current one.
//   * Every transform line belongs to one warp from its first FFT stage to its last
//     (fft_warp.cuh), so FFT stages are separated by __syncwarp(), not block barriers;
//     a block synchronises only where its warps hand data to one another (staging
//     buffer, transposed stores).
//   * The K planes of a channel are summed in the spectrum (the inverse transform is
//     linear): a column costs K forward transforms and one inverse; the adjoint costs one
//     forward and K inverse transforms.  The transfer function is evaluated in the pass
//     (per-column terms hoisted) or read from a precomputed table.
#include "asm_static.cuh"
#include "fft_warp.cuh"

namespace cvhrf {

__device__ int g_copy_wait_timeouts;

namespace {

constexpr long kMaxPolls = 1L << 24;

// Bounded wait on a bulk-copy mbarrier phase; on give-up it counts a timeout (the result
// of that launch is then invalid) and returns false.
__device__ __forceinline__ bool wait_copies(uint64_t* bar, unsigned parity) {
  for (long i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicAdd(&g_copy_wait_timeouts, 1);
  return false;
}

}  // namespace
}  // namespace cvhrf

#include "asm_fourstep.cuh"

namespace cvhrf {
namespace {

// Work split per line length (the warp-line passes: sizes other than 800 and 1024).
template <int S>
struct Split {
  // For the longest lines (BLK) a whole block transforms its lines together (one warp per
  // 1920- or 2048-point line would leave too few warps per SM to hide the shared-memory
  // latency of its stages); otherwise each warp owns its lines.
  static constexpr bool BLK = S >= 1920;
  // row passes: RPW rows per warp, NWR warps, ROWS rows per block, NTR threads per row group
  static constexpr int RPW = S >= 800 ? 1 : (S >= 256 ? 2 : 4);
  static constexpr int NWR = BLK ? 8 : (S >= 1024 ? 4 : 8);
  static constexpr int ROWS = BLK ? 2 : RPW * NWR;
  static constexpr int NTR = BLK ? NWR * 32 : 32;
  // column passes: COLS columns per block, LPW lines per group, NWC warps, NTH threads per group
  static constexpr int COLS = S == 800 ? 3 : (S == 1024 ? 2 : (S > 1024 ? 1 : 4));
  static constexpr int LPW = BLK ? 2 * COLS : (S >= 800 ? 1 : (S >= 256 ? 2 : 4));
  static constexpr int NWC = BLK ? 8 : 2 * COLS / LPW;
  static constexpr int NTH = BLK ? NWC * 32 : 32;
  static constexpr int LD = line_ld(S);
};

// ---- pass A: rows forward, transposed store ------------------------------------------
template <int S>
__global__ void __launch_bounds__(Split<S>::NWR * 32) rows_fwd_t(const float2* __restrict__ in, int items, int Hi,
                                                                int Wi, float2* __restrict__ A,
                                                                const float2* __restrict__ tw,
                                                                const float2* __restrict__ twP) {
  using SP = Split<S>;
  constexpr int P = 2 * S, LD = SP::LD, ROWS = SP::ROWS, NT = SP::NWR * 32;
  extern __shared__ __align__(16) float2 sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int total = items * Hi;
  const int row0 = blockIdx.x * ROWS;
  const int ow = (P - Wi) / 2;
  // each row group (a warp, or the whole block) loads and folds its rows: line 2r holds
  // x[n] at n mod S, line 2r + 1 holds x[n] w_2S^n (the odd output bins).  The loads are
  // asynchronous copies, all in flight at once; the odd lines are formed once they land.
  constexpr int GN = SP::NTR;
  const int gt = SP::BLK ? (int)threadIdx.x : lane;
  const int gr0 = SP::BLK ? 0 : warp * SP::RPW, grn = SP::BLK ? ROWS : SP::RPW;
  for (int e = gt; e < grn * S; e += GN) {
    const int r = gr0 + e / S, t = e % S;
    const int g = row0 + r;
    float2* le = sm + (2 * r) * LD;
    const float2* src = in + (size_t)(g < total ? g : 0) * Wi;
    int j = t - ow;
    if (j < 0 || j >= Wi) j = t + S - ow;
    if (g < total && j >= 0 && j < Wi) cp_async8(le + pidx(t), src + j);
    else le[pidx(t)] = make_float2(0.f, 0.f);
  }
  cp_async_commit();
  cp_async_wait_all();
  group_sync<GN>();
  for (int e = gt; e < grn * S; e += GN) {
    const int r = gr0 + e / S, t = e % S;
    const float2* le = sm + (2 * r) * LD;
    float2* lo = sm + (2 * r + 1) * LD;
    const int j = t - ow;
    const int pos = (j < 0 || j >= Wi) ? t + S : t;
    lo[pidx(t)] = pmul(le[pidx(t)], __ldg(&twP[pos]));
  }
  group_sync<GN>();
  warp_fft_forward<S, GN>(sm + (2 * gr0) * LD, 2 * grn, gt, tw);
  __syncthreads();
  // transposed store: for every spectrum column q, the block's ROWS rows are one run
  const int HiS = col_stride(Hi);
  for (int e = threadIdx.x; e < ROWS * P; e += NT) {
    const int q = e / ROWS, r = e - q * ROWS;
    const int g = row0 + r;
    if (g >= total) continue;
    const int item = g / Hi, rr = g - item * Hi;
    const int h = q >= S ? 1 : 0;
    A[((size_t)item * P + q) * HiS + rr] = sm[(2 * r + h) * LD + pidx(q - h * S)];
  }
}

// ---- pass C: rows inverse from the transposed spectra, crop, scale -------------------
template <int S>
__global__ void __launch_bounds__(Split<S>::NWR * 32) rows_inv_t(const float2* __restrict__ B, int items, int Ho,
                                                                float2* __restrict__ out, int Wo,
                                                                const float2* __restrict__ tw,
                                                                const float2* __restrict__ twP, float scale,
                                                                int accumulate) {
  using SP = Split<S>;
  constexpr int P = 2 * S, LD = SP::LD, ROWS = SP::ROWS, NT = SP::NWR * 32;
  extern __shared__ __align__(16) float2 sm[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int total = items * Ho;
  const int row0 = blockIdx.x * ROWS;
  const int HoS = col_stride(Ho);
  for (int e = threadIdx.x; e < ROWS * P; e += NT) {
    const int q = e / ROWS, r = e - q * ROWS;
    const int g = row0 + r;
    const int h = q >= S ? 1 : 0;
    float2* dst = sm + (2 * r + h) * LD + pidx(q - h * S);
    if (g < total) {
      const int item = g / Ho, rr = g - item * Ho;
      cp_async8(dst, B + ((size_t)item * P + q) * HoS + rr);
    } else {
      *dst = make_float2(0.f, 0.f);
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  constexpr int GN = SP::NTR;
  const int gt = SP::BLK ? (int)threadIdx.x : lane;
  const int gr0 = SP::BLK ? 0 : warp * SP::RPW, grn = SP::BLK ? ROWS : SP::RPW;
  warp_fft_inverse<S, GN>(sm + (2 * gr0) * LD, 2 * grn, gt, tw);
  const int oc = (P - Wo) / 2;
  for (int e = gt; e < grn * Wo; e += GN) {
    const int r = gr0 + e / Wo, x = e % Wo;
    const int g = row0 + r;
    if (g >= total) continue;
    const float2* le = sm + (2 * r) * LD;
    const float2* lo = le + LD;
    const int n = oc + x;
    const int t = n >= S ? n - S : n;
    float2 v = padd(le[pidx(t)], pmul(cconj(__ldg(&twP[n])), lo[pidx(t)]));
    v = pscale(scale, v);
    float2* dst = out + (size_t)g * Wo + x;
    if (accumulate) v = padd(*dst, v);
    *dst = v;
  }
}

// Fill this warp's lines (line gl = 2 cc + h of the block) from the staged columns:
// the even half-line takes the column, the odd one the column times w_2S^n.
template <int S, int NTH = 32>
__device__ __forceinline__ void fold_columns(float2* lines, int gl0, int nl, const float2* stage, int HiS, int Hi,
                                             int lane, const float2* __restrict__ twP) {
  constexpr int P = 2 * S, LD = line_ld(S);
  const int oh = (P - Hi) / 2;
  for (int l = 0; l < nl; ++l) {
    const int gl = gl0 + l, cc = gl >> 1, h = gl & 1;
    const float2* col = stage + cc * HiS;
    float2* line = lines + l * LD;
#pragma unroll 4
    for (int t = lane; t < S; t += NTH) {
      int r = t - oh, pos = t;
      if (r < 0 || r >= Hi) { r = t + S - oh; pos = t + S; }
      float2 v = make_float2(0.f, 0.f);
      if (r >= 0 && r < Hi) v = col[r];
      line[pidx(t)] = h ? pmul(v, __ldg(&twP[pos])) : v;
    }
  }
  group_sync<NTH>();
}

// ---- pass B, sum form: out[job] = sum_k P_k(in[k]) per column ------------------------
// Shared memory: staging (COLS x col_stride(Hi) values, bulk-copy target), then 2 COLS
// work lines and 2 COLS spectrum lines.
template <int S, bool TABLE>
__global__ void __launch_bounds__(Split<S>::NWC * 32, 2) cols_sum_t(const float2* __restrict__ A, int Hi,
                                                                float2* __restrict__ B, int Ho, const ColPlan plan,
                                                                const float2* __restrict__ table,
                                                                const float2* __restrict__ tw,
                                                                const float2* __restrict__ twP,
                                                                const int* __restrict__ digrev) {
  using SP = Split<S>;
  constexpr int P = 2 * S, LD = SP::LD, COLS = SP::COLS, LPW = SP::LPW, NT = SP::NWC * 32;
  extern __shared__ __align__(16) float2 sm[];
  __shared__ uint64_t bar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * COLS;
  const int ncols = min(COLS, P - q0);
  const int HiS = col_stride(Hi), HoS = col_stride(Ho);
  float2* stage = sm;
  float2* work = sm + ((COLS * HiS + 1) & ~1);
  float2* spec = work + 2 * COLS * LD;
  constexpr int NTH = SP::NTH;
  const int gt = SP::BLK ? (int)threadIdx.x : lane;    // thread index within the line group
  const int gl0 = SP::BLK ? 0 : warp * LPW;
  const int nl = max(0, min(LPW, 2 * ncols - gl0));
  float2* wl = work + gl0 * LD;
  float2* sl = spec + gl0 * LD;
  const int nin = plan.n[job];
  const unsigned bytes = (unsigned)(ncols * HiS * sizeof(float2));
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  auto issue = [&](int k) {
    const float2* src = A + ((size_t)plan.items[job][k] * P + q0) * HiS;
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_copy_g2s(stage, src, bytes, &bar);
  };
  if (threadIdx.x == 0) issue(0);
  // per-line column terms of the transfer function (the column bin is fixed per line)
  int kv[LPW];
#pragma unroll
  for (int l = 0; l < LPW; ++l) {
    int q = q0 + ((gl0 + l) >> 1);
    q = q < P ? q : 0;
    const int qh = q >= S ? 1 : 0;
    kv[l] = 2 * __ldg(&digrev[q - qh * S]) + qh;
  }
  for (int k = 0; k < nin; ++k) {
    wait_copies(&bar, k & 1);
    fold_columns<S, NTH>(wl, gl0, nl, stage, HiS, Hi, gt, twP);
    __syncthreads();                       // every warp is done with the staging buffer
    if (threadIdx.x == 0 && k + 1 < nin) {
      fence_proxy_async_smem();
      issue(k + 1);
    }
    warp_fft_forward_head<S, NTH>(wl, nl, gt, tw);
    const int ti = plan.tpi[job][k];
    if constexpr (TABLE) {
      const float2* Hb = table + (size_t)ti * P * P;
      warp_last_forward_mul_acc<S, NTH>(wl, sl, nl, gt, k == 0, [&](int l, int pos) {
        const int gl = gl0 + l;
        return __ldg(&Hb[((size_t)(q0 + (gl >> 1)) * 2 + (gl & 1)) * S + pos]);
      });
    } else {
      const TransferParams tp = plan.tp[ti];
      TransferCol col[LPW];
#pragma unroll
      for (int l = 0; l < LPW; ++l) col[l] = transfer_col(kv[l], P, tp);
      warp_last_forward_mul_acc<S, NTH>(wl, sl, nl, gt, k == 0, [&](int l, int pos) {
        const int ku = 2 * __ldg(&digrev[pos]) + ((gl0 + l) & 1);
        TransferCol c = col[0];
#pragma unroll
        for (int i = 1; i < LPW; ++i)
          if (l == i) c = col[i];
        return transfer_row(ku, P, c, tp);
      });
    }
  }
  warp_fft_inverse<S, NTH>(sl, nl, gt, tw);
  __syncthreads();
  // crop and fold back: y[n] = e[n mod S] + w_2S^-n o[n mod S]; each column is one run
  const int oc = (P - Ho) / 2;
  float2* Bout = B + ((size_t)plan.item[job] * P + q0) * HoS;
  for (int e = threadIdx.x; e < ncols * Ho; e += NT) {
    const int cc = e / Ho, rr = e - cc * Ho;
    const int n = oc + rr;
    const int t = n >= S ? n - S : n;
    const float2* se = spec + (2 * cc) * LD;
    Bout[(size_t)cc * HoS + rr] = padd(se[pidx(t)], pmul(cconj(__ldg(&twP[n])), se[LD + pidx(t)]));
  }
}

// ---- pass B, scatter form: out[items[k]] = P_k(in) per column ------------------------
template <int S, bool TABLE>
__global__ void __launch_bounds__(Split<S>::NWC * 32, 2) cols_scatter_t(const float2* __restrict__ A, int Hi,
                                                                    float2* __restrict__ B, int Ho,
                                                                    const ColPlan plan,
                                                                    const float2* __restrict__ table,
                                                                    const float2* __restrict__ tw,
                                                                    const float2* __restrict__ twP,
                                                                    const int* __restrict__ digrev) {
  using SP = Split<S>;
  constexpr int P = 2 * S, LD = SP::LD, COLS = SP::COLS, LPW = SP::LPW, NT = SP::NWC * 32;
  extern __shared__ __align__(16) float2 sm[];
  __shared__ uint64_t bar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int job = blockIdx.y;
  const int q0 = blockIdx.x * COLS;
  const int ncols = min(COLS, P - q0);
  const int HiS = col_stride(Hi), HoS = col_stride(Ho);
  float2* stage = sm;
  float2* work = sm + ((COLS * HiS + 1) & ~1);
  float2* spec = work + 2 * COLS * LD;
  constexpr int NTH = SP::NTH;
  const int gt = SP::BLK ? (int)threadIdx.x : lane;    // thread index within the line group
  const int gl0 = SP::BLK ? 0 : warp * LPW;
  const int nl = max(0, min(LPW, 2 * ncols - gl0));
  float2* wl = work + gl0 * LD;
  float2* sl = spec + gl0 * LD;
  const unsigned bytes = (unsigned)(ncols * HiS * sizeof(float2));
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_copy_g2s(stage, A + ((size_t)plan.item[job] * P + q0) * HiS, bytes, &bar);
  }
  int kv[LPW];
#pragma unroll
  for (int l = 0; l < LPW; ++l) {
    int q = q0 + ((gl0 + l) >> 1);
    q = q < P ? q : 0;
    const int qh = q >= S ? 1 : 0;
    kv[l] = 2 * __ldg(&digrev[q - qh * S]) + qh;
  }
  wait_copies(&bar, 0);
  fold_columns<S, NTH>(sl, gl0, nl, stage, HiS, Hi, gt, twP);
  warp_fft_forward<S, NTH>(sl, nl, gt, tw);
  const int oc = (P - Ho) / 2;
  const int nout = plan.n[job];
  for (int k = 0; k < nout; ++k) {
    const int ti = plan.tpi[job][k];
    if constexpr (TABLE) {
      const float2* Hb = table + (size_t)ti * P * P;
      warp_first_inverse_mul<S, NTH>(sl, wl, nl, gt, [&](int l, int pos) {
        const int gl = gl0 + l;
        return __ldg(&Hb[((size_t)(q0 + (gl >> 1)) * 2 + (gl & 1)) * S + pos]);
      });
    } else {
      const TransferParams tp = plan.tp[ti];
      TransferCol col[LPW];
#pragma unroll
      for (int l = 0; l < LPW; ++l) col[l] = transfer_col(kv[l], P, tp);
      warp_first_inverse_mul<S, NTH>(sl, wl, nl, gt, [&](int l, int pos) {
        const int ku = 2 * __ldg(&digrev[pos]) + ((gl0 + l) & 1);
        TransferCol c = col[0];
#pragma unroll
        for (int i = 1; i < LPW; ++i)
          if (l == i) c = col[i];
        return transfer_row(ku, P, c, tp);
      });
    }
    warp_fft_inverse_rest<S, NTH>(wl, nl, gt, tw);
    __syncthreads();
    float2* Bout = B + ((size_t)plan.items[job][k] * P + q0) * HoS;
    for (int e = threadIdx.x; e < ncols * Ho; e += NT) {
      const int cc = e / Ho, rr = e - cc * Ho;
      const int n = oc + rr;
      const int t = n >= S ? n - S : n;
      const float2* we = work + (2 * cc) * LD;
      Bout[(size_t)cc * HoS + rr] = padd(we[pidx(t)], pmul(cconj(__ldg(&twP[n])), we[LD + pidx(t)]));
    }
    __syncthreads();                       // the work lines are rewritten by the next output
  }
}

// Transfer table of one input item: H[(q * 2 + h) * S + pos] = transfer x aperture at row
// bin ku = 2 digrev[pos] + h and column bin kv of column q (the column pass layout).
template <int S>
__global__ void __launch_bounds__(256) transfer_table_s(float2* __restrict__ table, const int* __restrict__ digrev,
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
__global__ void __launch_bounds__(256) transfer_upload_s(float2* __restrict__ table, const int* __restrict__ digrev,
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

template <int S>
size_t row_smem() {
  return (size_t)Split<S>::ROWS * 2 * Split<S>::LD * sizeof(float2);
}
template <int S>
size_t col_smem(int Hi) {
  using SP = Split<S>;
  return (size_t)((SP::COLS * col_stride(Hi) + 1) & ~1) * sizeof(float2) + (size_t)4 * SP::COLS * SP::LD * sizeof(float2);
}

template <int S>
int run_rows_forward(const float2* in, int items, int Hi, int Wi, float2* A, const float2* tw, const float2* twP,
                     cudaStream_t st) {
  using SP = Split<S>;
  const int total = items * Hi;
  const size_t smem = row_smem<S>();
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(rows_fwd_t<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  rows_fwd_t<S><<<(total + SP::ROWS - 1) / SP::ROWS, SP::NWR * 32, smem, st>>>(in, items, Hi, Wi, A, tw, twP);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_rows_inverse(const float2* B, int items, int Ho, float2* out, int Wo, const float2* tw, const float2* twP,
                     int accumulate, cudaStream_t st) {
  using SP = Split<S>;
  const int total = items * Ho;
  const size_t smem = row_smem<S>();
  CVHRF_CUDA_TRY(cudaFuncSetAttribute(rows_inv_t<S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const float P = 2.0f * S;
  rows_inv_t<S><<<(total + SP::ROWS - 1) / SP::ROWS, SP::NWR * 32, smem, st>>>(B, items, Ho, out, Wo, tw, twP,
                                                                              1.0f / (P * P), accumulate);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_columns(bool scatter, const float2* A, int Hi, float2* B, int Ho, const ColPlan& plan, const float2* table,
                const float2* tw, const float2* twP, const int* digrev, cudaStream_t st) {
  using SP = Split<S>;
  const size_t smem = col_smem<S>(Hi);
  if (smem > 227 * 1024) return CVHRF_EUNSUPPORTED;
  dim3 grid((2 * S + SP::COLS - 1) / SP::COLS, plan.njobs);
  auto launch = [&](auto kern) -> int {
    CVHRF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, SP::NWC * 32, smem, st>>>(A, Hi, B, Ho, plan, table, tw, twP, digrev);
    CVHRF_LAUNCH_CHECK();
    return CVHRF_OK;
  };
  if (scatter) return table ? launch(cols_scatter_t<S, true>) : launch(cols_scatter_t<S, false>);
  return table ? launch(cols_sum_t<S, true>) : launch(cols_sum_t<S, false>);
}

template <int S>
int run_transfer_table(float2* table, const int* digrev, const TransferTable& tt, int items, cudaStream_t st) {
  const size_t n = (size_t)4 * S * S;
  const size_t nb = (n + 255) / 256;
  dim3 grid((unsigned)(nb < 1184 ? nb : 1184), items);
  transfer_table_s<S><<<grid, 256, 0, st>>>(table, digrev, tt);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

template <int S>
int run_transfer_upload(float2* table, const int* digrev, const float2* Hc, int items, cudaStream_t st) {
  const size_t n = (size_t)4 * S * S;
  const size_t nb = (n + 255) / 256;
  dim3 grid((unsigned)(nb < 1184 ? nb : 1184), items);
  transfer_upload_s<S><<<grid, 256, 0, st>>>(table, digrev, Hc);
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
    CVHRF_PLAN(64) CVHRF_PLAN(128) CVHRF_PLAN(256) CVHRF_PLAN(384) CVHRF_PLAN(512)
    CVHRF_PLAN(1920) CVHRF_PLAN(2048)
    // the four-step passes keep natural bin order: one "stage" of radix S (identity table)
    case 800: case 1024: radix[0] = S; *nst = 1; break;
    default: *nst = 0;
  }
#undef CVHRF_PLAN
}

// FS: the four-step pass for 800 and 1024 (same arguments), CALL: the warp-line pass.
#define CVHRF_STATIC_DISPATCH2(CALL, FS, ARGS)                                                             \
  switch (d.S) {                                                                                           \
    case 64: return CALL<64> ARGS; case 128: return CALL<128> ARGS; case 256: return CALL<256> ARGS;      \
    case 384: return CALL<384> ARGS; case 512: return CALL<512> ARGS; case 800: return FS<800> ARGS;      \
    case 1024: return FS<1024> ARGS; case 1920: return CALL<1920> ARGS; case 2048: return CALL<2048> ARGS; \
    default: return CVHRF_EUNSUPPORTED;                                                                    \
  }
#define CVHRF_STATIC_DISPATCH(CALL, ARGS) CVHRF_STATIC_DISPATCH2(CALL, CALL, ARGS)

int static_rows_forward(const FftDesc& d, const float2* in, int items, int Hi, int Wi, float2* A, cudaStream_t st) {
  CVHRF_STATIC_DISPATCH2(run_rows_forward, fs_run_rows_forward, (in, items, Hi, Wi, A, d.tw, d.twP, st))
}

int static_columns(const FftDesc& d, bool scatter, const float2* A, int Hi, float2* B, int Ho, const ColPlan& plan,
                   const float2* table, cudaStream_t st) {
  if (plan.njobs < 1 || plan.njobs > kMaxColJobs) return CVHRF_EINVAL;
  switch (d.S) {
    case 800: return fs_run_columns<800>(scatter, A, Hi, B, Ho, plan, table, d.tw, d.twP, st);
    case 1024: return fs_run_columns<1024>(scatter, A, Hi, B, Ho, plan, table, d.tw, d.twP, st);
    default: break;
  }
  CVHRF_STATIC_DISPATCH(run_columns, (scatter, A, Hi, B, Ho, plan, table, d.tw, d.twP, d.digrev, st))
}

int static_rows_inverse(const FftDesc& d, const float2* B, int items, int Ho, float2* out, int Wo, int accumulate,
                        cudaStream_t st) {
  CVHRF_STATIC_DISPATCH2(run_rows_inverse, fs_run_rows_inverse, (B, items, Ho, out, Wo, d.tw, d.twP, accumulate, st))
}

int static_transfer_table(const FftDesc& d, float2* table, const TransferTable& tt, int items, cudaStream_t st) {
  CVHRF_STATIC_DISPATCH(run_transfer_table, (table, d.digrev, tt, items, st))
}

int static_transfer_upload(const FftDesc& d, float2* table, const float2* centred, int items, cudaStream_t st) {
  CVHRF_STATIC_DISPATCH(run_transfer_upload, (table, d.digrev, centred, items, st))
}

#undef CVHRF_STATIC_DISPATCH
#undef CVHRF_STATIC_DISPATCH2

int static_copy_wait_timeouts() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_copy_wait_timeouts, sizeof(int));
  return v;
}

}  // namespace cvhrf

extern "C" int cvhrf_copy_wait_timeouts(void) { return cvhrf::static_copy_wait_timeouts(); }
