// Register-resident four-step FFT of one line per warp, for S = 32 M (M <= 32).
//
// A length-S line x[n], n = n1 + 32 n2 (n1 = lane, n2 < M), is held as M values per lane.
//   forward:  X[k2 + M k1] = sum_n1 w32^(n1 k1) w_S^(n1 k2) sum_n2 x[n1 + 32 n2] w_M^(n2 k2)
//     1. an M-point DFT over n2 in each lane's registers,
//     2. the twiddle w_S^(n1 k2),
//     3. one transpose through shared memory (M x 32 values, swizzled),
//     4. a 32-point DFT over n1 in registers: lane k2 (< M) ends with X[k2 + M k1], k1 < 32.
//   inverse:  the same steps in reverse order with conjugated roots (unnormalised), from
//     lane k2 holding X[k2 + M k1] to lane n1 holding x[n1 + 32 n2].
// Bins come out in natural order, so no digit-reversal table is needed.  A stage never
// leaves the warp: the only synchronisation is __syncwarp() around the transpose, whose
// swizzled layout keeps both of its access patterns free of bank conflicts.
#pragma once
#include "fft_static.cuh"

namespace cvhrf {

// The transpose buffer holds M x 32 values; value (k2, n1) sits at
// base[(32 k2 + (n1 ^ k2)) * stride].  The XOR swizzle keeps both access patterns
// (fixed k2 across lanes n1, fixed n1 across lanes k2) free of bank conflicts for any odd
// stride, so the buffer can be a strided region of a larger tile.
__device__ __forceinline__ int fs_tslot(int k2, int n1) { return 32 * k2 + (n1 ^ k2); }

// x[j] = x[lane + 32 j] in, y[k1] = X[lane + M k1] out (meaningful for lane < M).
template <int S>
__device__ __forceinline__ void fs_forward(float2 (&x)[S / 32], float2 (&y)[32], float2* T, int ts, int lane,
                                           const float2* __restrict__ tw) {  // tw: fs_stage_roots table
  constexpr int M = S / 32;
  regdft<M>(x);
#pragma unroll
  for (int k2 = 1; k2 < M; ++k2) x[k2] = pmul(x[k2], tw[fs_tslot(k2, lane)]);
  __syncwarp();
#pragma unroll
  for (int k2 = 0; k2 < M; ++k2) T[fs_tslot(k2, lane) * ts] = x[k2];
  __syncwarp();
  if (lane < M) {
#pragma unroll
    for (int n1 = 0; n1 < 32; ++n1) y[n1] = T[fs_tslot(lane, n1) * ts];
    regdft<32>(y);
  }
  __syncwarp();
}

// y[k1] = X[lane + M k1] in (lane < M), x[j] = sum over bins (unnormalised inverse) at
// lane + 32 j out.
template <int S>
__device__ __forceinline__ void fs_inverse(float2 (&y)[32], float2 (&x)[S / 32], float2* T, int ts, int lane,
                                           const float2* __restrict__ tw) {  // tw: fs_stage_roots table
  constexpr int M = S / 32;
  __syncwarp();
  if (lane < M) {
#pragma unroll
    for (int k1 = 0; k1 < 32; ++k1) y[k1] = cconj(y[k1]);
    regdft<32>(y);
#pragma unroll
    for (int n1 = 0; n1 < 32; ++n1) {
      float2 v = cconj(y[n1]);
      if (n1 > 0) v = pmul(v, cconj(tw[fs_tslot(lane, n1)]));
      T[fs_tslot(lane, n1) * ts] = v;
    }
  }
  __syncwarp();
#pragma unroll
  for (int k2 = 0; k2 < M; ++k2) x[k2] = cconj(T[fs_tslot(k2, lane) * ts]);
  __syncwarp();
  regdft<M>(x);
#pragma unroll
  for (int k2 = 0; k2 < M; ++k2) x[k2] = cconj(x[k2]);
}

}  // namespace cvhrf
