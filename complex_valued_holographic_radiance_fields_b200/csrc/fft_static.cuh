// Compile-time-sized mixed-radix FFT over shared-memory lines.
//
// Same in-place DIF / conjugate-DIT structure and the same digit-reversed bin layout
// as fft_lines.cuh (so the same digit-reversal table serves both), but the line length
// S is a template parameter and each stage uses a composite radix of up to 32 whose
// butterfly is a full DFT in registers (nested radix 2/3/4/5/8, compile-time twiddles).
// 800 = 32 x 25, 1024 = 32 x 32 and 1920 = 32 x 30 x 2 therefore need two or three
// shared-memory round trips per transform instead of four or five, and every index
// division is by a constant.
#pragma once
#include "fft_lines.cuh"

namespace cvhrf {

// ---- compile-time trigonometry (double, Taylor series after reduction to [-pi/4, pi/4]) ----
constexpr double kPi = 3.14159265358979323846264338327950288;
constexpr double ct_sin_series(double x) {
  double t = x, s = x;
  for (int k = 1; k < 14; ++k) {
    t *= -x * x / ((2 * k) * (2 * k + 1));
    s += t;
  }
  return s;
}
constexpr double ct_cos_series(double x) {
  double t = 1.0, s = 1.0;
  for (int k = 1; k < 14; ++k) {
    t *= -x * x / ((2 * k - 1) * (2 * k));
    s += t;
  }
  return s;
}
// exp(-2 pi i num / den) as (cos, sin), exact-rational argument reduction by octant
constexpr double ct_cos_frac(long num, long den) {
  num %= den;
  if (num < 0) num += den;
  const long q8 = (num * 8) / den;          // octant
  const double r = 2.0 * kPi * (double)(num * 8 - q8 * den) / (double)(8 * den);  // [0, pi/4)
  switch (q8) {
    case 0: return ct_cos_series(r);
    case 1: return ct_sin_series(kPi / 4 - r);
    case 2: return -ct_sin_series(r);
    case 3: return -ct_cos_series(kPi / 4 - r);
    case 4: return -ct_cos_series(r);
    case 5: return -ct_sin_series(kPi / 4 - r);
    case 6: return ct_sin_series(r);
    default: return ct_cos_series(kPi / 4 - r);
  }
}
constexpr double ct_sin_frac(long num, long den) {  // sin(2 pi num / den)
  num %= den;
  if (num < 0) num += den;
  const long q8 = (num * 8) / den;
  const double r = 2.0 * kPi * (double)(num * 8 - q8 * den) / (double)(8 * den);
  switch (q8) {
    case 0: return ct_sin_series(r);
    case 1: return ct_cos_series(kPi / 4 - r);
    case 2: return ct_cos_series(r);
    case 3: return ct_sin_series(kPi / 4 - r);
    case 4: return -ct_sin_series(r);
    case 5: return -ct_cos_series(kPi / 4 - r);
    case 6: return -ct_cos_series(r);
    default: return -ct_sin_series(kPi / 4 - r);
  }
}

// ---- register DFT of composite size R (natural order in and out, sign -1) ----
template <int R>
struct RegSplit {
  static constexpr int a = (R % 8 == 0 && R > 8) ? 8
                           : (R % 4 == 0 && R > 4) ? 4
                           : (R % 5 == 0 && R > 5) ? 5
                           : (R % 3 == 0 && R > 3) ? 3
                           : (R % 2 == 0 && R > 2) ? 2 : R;
  static constexpr int b = R / a;
};

template <int R>
__device__ __forceinline__ void regdft(float2* x);

template <int R, int I2, int K1>
__device__ __forceinline__ float2 twiddle_mul(float2 v) {
  constexpr float c = (float)ct_cos_frac((long)I2 * K1, R);
  constexpr float s = (float)(-ct_sin_frac((long)I2 * K1, R));
  if constexpr (I2 * K1 == 0) return v;
  else return pfma(s, make_float2(-v.y, v.x), pscale(c, v));
}

template <int R, int A, int B, int I2, int K1>
__device__ __forceinline__ void twiddle_row(float2* x) {
  if constexpr (K1 < A) {
    x[I2 + B * K1] = twiddle_mul<R, I2, K1>(x[I2 + B * K1]);
    twiddle_row<R, A, B, I2, K1 + 1>(x);
  }
}
template <int R, int A, int B, int I2>
__device__ __forceinline__ void twiddle_all(float2* x) {
  if constexpr (I2 < B) {
    twiddle_row<R, A, B, I2, 1>(x);
    twiddle_all<R, A, B, I2 + 1>(x);
  }
}

template <int R>
__device__ __forceinline__ void regdft(float2* x) {
  if constexpr (R == 1) {
    return;
  } else if constexpr (R == 2 || R == 3 || R == 4 || R == 5 || R == 8) {
    dftR<R>(x);
  } else {
    constexpr int A = RegSplit<R>::a, B = RegSplit<R>::b;
    // A-point DFTs over stride B
#pragma unroll
    for (int i2 = 0; i2 < B; ++i2) {
      float2 t[A];
#pragma unroll
      for (int i1 = 0; i1 < A; ++i1) t[i1] = x[i2 + B * i1];
      dftR<A>(t);
#pragma unroll
      for (int k1 = 0; k1 < A; ++k1) x[i2 + B * k1] = t[k1];
    }
    twiddle_all<R, A, B, 1>(x);
    // B-point DFTs over contiguous blocks
#pragma unroll
    for (int k1 = 0; k1 < A; ++k1) regdft<B>(x + B * k1);
    // X[k1 + A k2] sits at B k1 + k2: permute to natural order
    float2 y[R];
#pragma unroll
    for (int k1 = 0; k1 < A; ++k1)
#pragma unroll
      for (int k2 = 0; k2 < B; ++k2) y[k1 + A * k2] = x[B * k1 + k2];
#pragma unroll
    for (int i = 0; i < R; ++i) x[i] = y[i];
  }
}

// ---- compile-time plan: stage radices (each <= 32, built from 2/3/4/5/8) ----
constexpr bool ct_smooth(int n) {
  while (n % 2 == 0) n /= 2;
  while (n % 3 == 0) n /= 3;
  while (n % 5 == 0) n /= 5;
  return n == 1;
}
constexpr int ct_big_radix(int n) {  // largest divisor of n that is <= 32
  for (int r = 32; r >= 2; --r)
    if (n % r == 0) return r;
  return n;
}
template <int S>
struct StaticPlan {
  static_assert(ct_smooth(S), "S must factor into 2, 3 and 5");
  static constexpr int r0 = ct_big_radix(S);
  static constexpr int r1 = S / r0 == 1 ? 1 : ct_big_radix(S / r0);
  static constexpr int r2 = S / r0 / r1 == 1 ? 1 : ct_big_radix(S / r0 / r1);
  static_assert(S / r0 / r1 / r2 == 1, "plan needs more than three stages");
  static constexpr int nst = r1 == 1 ? 1 : (r2 == 1 ? 2 : 3);
  static constexpr int R(int i) { return i == 0 ? r0 : (i == 1 ? r1 : r2); }
  static constexpr int L(int i) { return i == 0 ? S / r0 : (i == 1 ? S / r0 / r1 : 1); }
  static constexpr int span(int i) { return i == 0 ? 1 : (i == 1 ? r0 : r0 * r1); }
};

template <int S, int ST, bool INV>
__device__ __forceinline__ void static_stage(float2* sm, int nlines, int ld, const float2* __restrict__ tw) {
  using P = StaticPlan<S>;
  constexpr int R = P::R(ST), L = P::L(ST), span = P::span(ST);
  constexpr int bpl = S / R;
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
      regdft<R>(x);
      if constexpr (L > 1) {
#pragma unroll
        for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&tw[j * m * span]));
      }
#pragma unroll
      for (int m = 0; m < R; ++m) p[m * L] = x[m];
    } else {
#pragma unroll
      for (int m = 0; m < R; ++m) x[m] = cconj(x[m]);
      if constexpr (L > 1) {
#pragma unroll
        for (int m = 1; m < R; ++m) x[m] = pmul(x[m], __ldg(&tw[j * m * span]));
      }
      regdft<R>(x);
#pragma unroll
      for (int m = 0; m < R; ++m) p[m * L] = cconj(x[m]);
    }
  }
}

template <int S>
__device__ __forceinline__ void static_fft_forward(float2* sm, int nlines, int ld, const float2* tw) {
  using P = StaticPlan<S>;
  static_stage<S, 0, false>(sm, nlines, ld, tw);
  __syncthreads();
  if constexpr (P::nst > 1) {
    static_stage<S, 1, false>(sm, nlines, ld, tw);
    __syncthreads();
  }
  if constexpr (P::nst > 2) {
    static_stage<S, 2, false>(sm, nlines, ld, tw);
    __syncthreads();
  }
}

template <int S>
__device__ __forceinline__ void static_fft_inverse(float2* sm, int nlines, int ld, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 2) {
    static_stage<S, 2, true>(sm, nlines, ld, tw);
    __syncthreads();
  }
  if constexpr (P::nst > 1) {
    static_stage<S, 1, true>(sm, nlines, ld, tw);
    __syncthreads();
  }
  static_stage<S, 0, true>(sm, nlines, ld, tw);
  __syncthreads();
}

// The last forward stage (its L is 1) fused with a pointwise spectrum product: instead of
// writing the stage's outputs back, x * H is stored (first) or added into `spec` at the
// same positions.  H holds, per line pair (column q = q0 + line / 2, half h = line % 2),
// S values in position order: H[((q0 + line / 2) * 2 + h) * S + pos].
template <int S>
__device__ __forceinline__ void static_last_forward_mul_acc(float2* sm, float2* spec, int nlines, int ld,
                                                            const float2* __restrict__ H, int q0, bool first) {
  using P = StaticPlan<S>;
  constexpr int ST = P::nst - 1;
  constexpr int R = P::R(ST), L = P::L(ST);
  static_assert(L == 1, "last stage has unit stride");
  constexpr int bpl = S / R;
  const int total = nlines * bpl;
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int line = b / bpl;
    const int blk = b - line * bpl;
    const int off = line * ld + blk * R;
    const float2* hp = H + ((size_t)(q0 + (line >> 1)) * 2 + (line & 1)) * S + blk * R;
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = sm[off + m];
    regdft<R>(x);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const float2 y = pmul(x[m], __ldg(&hp[m]));
      spec[off + m] = first ? y : padd(spec[off + m], y);
    }
  }
}

// The first inverse stage fused with a pointwise product by conj(H) (same H layout as
// above): reads `spec`, writes the stage's outputs to `sm`; the remaining inverse stages
// then run on `sm` (static_fft_inverse_rest).
template <int S>
__device__ __forceinline__ void static_first_inverse_mul(const float2* spec, float2* sm, int nlines, int ld,
                                                         const float2* __restrict__ H, int q0) {
  using P = StaticPlan<S>;
  constexpr int ST = P::nst - 1;
  constexpr int R = P::R(ST), L = P::L(ST);
  static_assert(L == 1, "last stage has unit stride");
  constexpr int bpl = S / R;
  const int total = nlines * bpl;
  for (int b = threadIdx.x; b < total; b += blockDim.x) {
    const int line = b / bpl;
    const int blk = b - line * bpl;
    const int off = line * ld + blk * R;
    const float2* hp = H + ((size_t)(q0 + (line >> 1)) * 2 + (line & 1)) * S + blk * R;
    float2 x[R];
#pragma unroll
    for (int m = 0; m < R; ++m) x[m] = cconj(pmul(spec[off + m], cconj(__ldg(&hp[m]))));
    regdft<R>(x);
#pragma unroll
    for (int m = 0; m < R; ++m) sm[off + m] = cconj(x[m]);
  }
}

// Forward transform without its last stage (used with static_last_forward_mul_acc).
template <int S>
__device__ __forceinline__ void static_fft_forward_head(float2* sm, int nlines, int ld, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 1) {
    static_stage<S, 0, false>(sm, nlines, ld, tw);
    __syncthreads();
  }
  if constexpr (P::nst > 2) {
    static_stage<S, 1, false>(sm, nlines, ld, tw);
    __syncthreads();
  }
}

// Inverse transform without its first stage (used after static_first_inverse_mul).
template <int S>
__device__ __forceinline__ void static_fft_inverse_rest(float2* sm, int nlines, int ld, const float2* tw) {
  using P = StaticPlan<S>;
  if constexpr (P::nst > 2) {
    static_stage<S, 1, true>(sm, nlines, ld, tw);
    __syncthreads();
  }
  if constexpr (P::nst > 1) {
    static_stage<S, 0, true>(sm, nlines, ld, tw);
    __syncthreads();
  }
}

}  // namespace cvhrf
