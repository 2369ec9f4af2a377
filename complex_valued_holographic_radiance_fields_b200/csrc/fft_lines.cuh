// In-place mixed-radix (2,3,4,5,8) complex FFT over lines held in shared memory.
//
// Forward transforms are decimation-in-frequency: natural-order input, output in
// mixed-radix digit-reversed order.  Inverse transforms are the exact transpose
// (decimation-in-time, conjugated), taking digit-reversed input to natural order.
// The propagation never needs natural-order spectra: the transfer function is
// evaluated per bin through the `digrev` table, so no permutation pass exists.
//
// Stage i of the forward transform has radix R_i and stride L_i = S / (R_1...R_i);
// the butterfly at (block, j) reads x[block*R_i*L_i + j + m*L_i], m < R_i, applies
// an R_i-point DFT and multiplies output m by w_{R_i L_i}^{j m}.  The output of
// bin k = m_1 + R_1 (m_2 + R_2 (m_3 + ...)) ends at position sum_i L_i m_i.
#pragma once
#include "common.cuh"

namespace cvhrf {

constexpr int kMaxFftStages = 12;

struct FftDesc {
  int S;                       // line length
  int nst;                     // number of stages
  int radix[kMaxFftStages];
  int L[kMaxFftStages];        // stride of stage i
  int span[kMaxFftStages];     // S / (R_i * L_i): twiddle index multiplier
  const float2* tw;            // S entries: exp(-2 pi i t / S)
  const float2* twP;           // 2S entries: exp(-2 pi i t / (2S))
  const int* digrev;           // S entries: position -> natural bin index
};

// Forward R-point DFTs (sign -1), in registers, on the packed f32x2 datapath.
__device__ __forceinline__ void dft2(float2* x) {
  float2 a = x[0], b = x[1];
  x[0] = padd(a, b);
  x[1] = psub(a, b);
}
// multiply by -i
__device__ __forceinline__ float2 mul_mi(float2 a) { return make_float2(a.y, -a.x); }

__device__ __forceinline__ void dft3(float2* x) {
  const float c = -0.5f, s = 0.86602540378443864676f;
  float2 t = padd(x[1], x[2]);
  float2 d = psub(x[1], x[2]);
  float2 y0 = padd(x[0], t);
  float2 m = pfma(c, t, x[0]);
  float2 r = pscale(s, d);                         // s (x1 - x2)
  x[0] = y0;
  x[1] = padd(m, mul_mi(r));                       // m - i s (x1 - x2)
  x[2] = psub(m, mul_mi(r));
}

__device__ __forceinline__ void dft4(float2* x) {
  float2 a = padd(x[0], x[2]), b = psub(x[0], x[2]);
  float2 c = padd(x[1], x[3]), d = mul_mi(psub(x[1], x[3]));
  x[0] = padd(a, c);
  x[2] = psub(a, c);
  x[1] = padd(b, d);
  x[3] = psub(b, d);
}

__device__ __forceinline__ void dft5(float2* x) {
  const float c1 = 0.30901699437494742410f, c2 = -0.80901699437494742410f;
  const float s1 = 0.95105651629515357212f, s2 = 0.58778525229247312917f;
  float2 a1 = padd(x[1], x[4]), b1 = psub(x[1], x[4]);
  float2 a2 = padd(x[2], x[3]), b2 = psub(x[2], x[3]);
  float2 x0 = x[0];
  float2 r1 = pfma(c2, a2, pfma(c1, a1, x0));
  float2 r2 = pfma(c1, a2, pfma(c2, a1, x0));
  float2 i1 = pfma(s2, b2, pscale(s1, b1));
  float2 i2 = pfma(-s1, b2, pscale(s2, b1));
  x[0] = padd(padd(x0, a1), a2);
  x[1] = padd(r1, mul_mi(i1));
  x[4] = psub(r1, mul_mi(i1));
  x[2] = padd(r2, mul_mi(i2));
  x[3] = psub(r2, mul_mi(i2));
}

__device__ __forceinline__ void dft8(float2* x) {
  const float h = 0.70710678118654752440f;
  float2 e[4] = {x[0], x[2], x[4], x[6]};
  float2 o[4] = {x[1], x[3], x[5], x[7]};
  dft4(e);
  dft4(o);
  // o_k *= w8^k
  o[1] = pscale(h, make_float2(o[1].x + o[1].y, o[1].y - o[1].x));
  o[2] = mul_mi(o[2]);
  o[3] = pscale(-h, make_float2(o[3].x - o[3].y, o[3].x + o[3].y));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    x[k] = padd(e[k], o[k]);
    x[k + 4] = psub(e[k], o[k]);
  }
}

template <int R>
__device__ __forceinline__ void dftR(float2* x) {
  if constexpr (R == 2) dft2(x);
  else if constexpr (R == 3) dft3(x);
  else if constexpr (R == 4) dft4(x);
  else if constexpr (R == 5) dft5(x);
  else dft8(x);
}

// One stage over `nlines` lines (line l at sm + l*ld), all threads of the block.
template <int R, bool INV>
__device__ __forceinline__ void fft_stage(float2* sm, int nlines, int ld, const FftDesc& d, int st) {
  const int L = d.L[st];
  const int span = d.span[st];
  const int bpl = d.S / R;
  const int total = nlines * bpl;
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int line = b / bpl;
    const int bb = b - line * bpl;
    const int blk = bb / L;
    const int j = bb - blk * L;
    float2* p = sm + line * ld + blk * R * L + j;
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = p[m * L];
    if constexpr (!INV) {
      dftR<R>(x);
#pragma unroll
      for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&d.tw[j * m * span]));
#pragma unroll
      for (int m = 0; m < R; ++m) p[m * L] = x[m];
    } else {
#pragma unroll
      for (int m = 0; m < R; ++m) x[m] = cconj(x[m]);
#pragma unroll
      for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&d.tw[j * m * span]));
      dftR<R>(x);
#pragma unroll
      for (int m = 0; m < R; ++m) p[m * L] = cconj(x[m]);
    }
  }
}

template <bool INV>
__device__ __forceinline__ void fft_stage_dispatch(float2* sm, int nlines, int ld, const FftDesc& d, int st) {
  switch (d.radix[st]) {
    case 2: fft_stage<2, INV>(sm, nlines, ld, d, st); break;
    case 3: fft_stage<3, INV>(sm, nlines, ld, d, st); break;
    case 4: fft_stage<4, INV>(sm, nlines, ld, d, st); break;
    case 5: fft_stage<5, INV>(sm, nlines, ld, d, st); break;
    default: fft_stage<8, INV>(sm, nlines, ld, d, st); break;
  }
}

// Forward DIF transform of all lines (natural -> digit-reversed).  The caller
// must __syncthreads() after filling the lines; returns after a barrier.
__device__ __forceinline__ void fft_forward_lines(float2* sm, int nlines, int ld, const FftDesc& d) {
  for (int st = 0; st < d.nst; ++st) {
    fft_stage_dispatch<false>(sm, nlines, ld, d, st);
    __syncthreads();
  }
}

// Unnormalised inverse DIT transform (digit-reversed -> natural).
__device__ __forceinline__ void fft_inverse_lines(float2* sm, int nlines, int ld, const FftDesc& d) {
  for (int st = d.nst - 1; st >= 0; --st) {
    fft_stage_dispatch<true>(sm, nlines, ld, d, st);
    __syncthreads();
  }
}

}  // namespace cvhrf
