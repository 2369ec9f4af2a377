// Warp-owned compile-time FFT lines in shared memory.
//
// The stages, radices, twiddles and the digit-reversed bin order are those of
// fft_static.cuh (StaticPlan<S>), so the digit-reversal table of a plan serves both.  The
// difference is ownership: a warp transforms its own lines from the first stage to the
// last, so stages are separated by __syncwarp() instead of block-wide barriers, and a
// block's warps never wait on one another inside a transform.
//
// Lines are stored padded: element i of a line sits at pidx(i) = i + i / 32, and lines
// are line_ld(S) float2 apart (line_ld = 1 mod 8).  With that layout the strided
// butterfly loads and stores of every stage, and the 8-line-wide transposed accesses
// of the row passes, fall in distinct banks (64-bit accesses are served per half-warp).
#pragma once
#include "fft_static.cuh"

namespace cvhrf {

__device__ __forceinline__ int pidx(int i) { return i + (i >> 5); }

// A group of NTH threads owns a set of lines: one warp (NTH = 32, synchronised with
// __syncwarp) or a whole block (NTH = blockDim.x, synchronised with __syncthreads; used for
// the longest lines, where one warp per line leaves too few warps per SM).
template <int NTH>
__device__ __forceinline__ void group_sync() {
  if constexpr (NTH == 32) __syncwarp();
  else __syncthreads();
}

constexpr int line_ld(int S) {
  int ld = S + S / 32;
  while (ld % 8 != 1) ++ld;
  return ld;
}

// One stage over the warp's `nl` lines (line l at lines + l * LD).  Forward: DIF
// butterfly then twiddle; inverse: conjugated twiddle then butterfly (conjugate DIT).
template <int S, int ST, bool INV, int NTH = 32>
__device__ __forceinline__ void warp_stage(float2* lines, int nl, int lane, const float2* __restrict__ tw) {
  using P = StaticPlan<S>;
  constexpr int R = P::R(ST), L = P::L(ST), span = P::span(ST);
  constexpr int bpl = S / R;
  constexpr int LD = line_ld(S);
  for (int b = lane; b < nl * bpl; b += NTH) {
    const int l = b / bpl;
    const int bb = b - l * bpl;
    const int blk = bb / L;
    const int j = bb - blk * L;
    float2* p = lines + l * LD;
    const int base = blk * R * L + j;
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = p[pidx(base + m * L)];
    if constexpr (!INV) {
      regdft<R>(x);
      if constexpr (L > 1) {
#pragma unroll
        for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&tw[j * m * span]));
      }
#pragma unroll
      for (int m = 0; m < R; ++m) p[pidx(base + m * L)] = x[m];
    } else {
#pragma unroll
      for (int m = 0; m < R; ++m) x[m] = cconj(x[m]);
      if constexpr (L > 1) {
#pragma unroll
        for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&tw[j * m * span]));
      }
      regdft<R>(x);
#pragma unroll
      for (int m = 0; m < R; ++m) p[pidx(base + m * L)] = cconj(x[m]);
    }
  }
  group_sync<NTH>();
}

template <int S, int NTH = 32>
__device__ __forceinline__ void warp_fft_forward(float2* lines, int nl, int lane, const float2* tw) {
  using P = StaticPlan<S>;
  warp_stage<S, 0, false, NTH>(lines, nl, lane, tw);
  if constexpr (P::nst > 1) warp_stage<S, 1, false, NTH>(lines, nl, lane, tw);
  if constexpr (P::nst > 2) warp_stage<S, 2, false, NTH>(lines, nl, lane, tw);
}

template <int S, int NTH = 32>
__device__ __forceinline__ void warp_fft_inverse(float2* lines, int nl, int lane, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 2) warp_stage<S, 2, true, NTH>(lines, nl, lane, tw);
  if constexpr (P::nst > 1) warp_stage<S, 1, true, NTH>(lines, nl, lane, tw);
  warp_stage<S, 0, true, NTH>(lines, nl, lane, tw);
}

// Forward transform without its last stage (the last stage is fused with a product).
template <int S, int NTH = 32>
__device__ __forceinline__ void warp_fft_forward_head(float2* lines, int nl, int lane, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 1) warp_stage<S, 0, false, NTH>(lines, nl, lane, tw);
  if constexpr (P::nst > 2) warp_stage<S, 1, false, NTH>(lines, nl, lane, tw);
}

// Inverse transform without its first stage (the first stage is fused with a product).
template <int S, int NTH = 32>
__device__ __forceinline__ void warp_fft_inverse_rest(float2* lines, int nl, int lane, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 2) warp_stage<S, 1, true, NTH>(lines, nl, lane, tw);
  if constexpr (P::nst > 1) warp_stage<S, 0, true, NTH>(lines, nl, lane, tw);
}

// Last forward stage (unit stride) fused with a pointwise product: spec[l][pos] = (or +=)
// X[l][pos] * h(l, pos), where X is the stage's output.  h(l, pos) gives the transfer
// value of line l at spectrum position pos.
template <int S, int NTH = 32, typename HFn>
__device__ __forceinline__ void warp_last_forward_mul_acc(float2* lines, float2* spec, int nl, int lane, bool first,
                                                          HFn h) {
  using P = StaticPlan<S>;
  constexpr int ST = P::nst - 1;
  constexpr int R = P::R(ST), L = P::L(ST);
  static_assert(L == 1, "last stage has unit stride");
  constexpr int bpl = S / R;
  constexpr int LD = line_ld(S);
  for (int b = lane; b < nl * bpl; b += NTH) {
    const int l = b / bpl;
    const int blk = b - l * bpl;
    const float2* p = lines + l * LD;
    float2* o = spec + l * LD;
    // the transfer values first: their loads are in flight during the butterfly
    float2 hv[R];
#pragma unroll
    for (int m = 0; m < R; ++m) hv[m] = h(l, blk * R + m);
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = p[pidx(blk * R + m)];
    regdft<R>(x);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const int i = pidx(blk * R + m);
      const float2 y = pmul(x[m], hv[m]);
      o[i] = first ? y : padd(o[i], y);
    }
  }
  group_sync<NTH>();
}

// First inverse stage fused with a pointwise product by conj(h): reads `spec`, writes the
// stage's outputs to `lines`; warp_fft_inverse_rest completes the transform.
template <int S, int NTH = 32, typename HFn>
__device__ __forceinline__ void warp_first_inverse_mul(const float2* spec, float2* lines, int nl, int lane, HFn h) {
  using P = StaticPlan<S>;
  constexpr int ST = P::nst - 1;
  constexpr int R = P::R(ST), L = P::L(ST);
  static_assert(L == 1, "last stage has unit stride");
  constexpr int bpl = S / R;
  constexpr int LD = line_ld(S);
  for (int b = lane; b < nl * bpl; b += NTH) {
    const int l = b / bpl;
    const int blk = b - l * bpl;
    const float2* p = spec + l * LD;
    float2* o = lines + l * LD;
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = h(l, blk * R + m);
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = cconj(pmul(p[pidx(blk * R + m)], cconj(x[m])));
    regdft<R>(x);
#pragma unroll
    for (int m = 0; m < R; ++m) o[pidx(blk * R + m)] = cconj(x[m]);
  }
  group_sync<NTH>();
}

}  // namespace cvhrf
