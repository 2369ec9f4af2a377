// Fused sparse Adam over visible Gaussians (replaces conv.cu:1200-1246, sparse_adam_kernel /
// adamUpdate, and the per-group loop of utils/optimizer.py:180-265).
//
// The reference launches one kernel per parameter group with a (V, B) grid of
// D-thread blocks (3-4 threads per block) after gathering the visible gradient rows
// into a fresh (B, V, D) tensor.  Here all groups are one launch, one thread per
// updated element, reading the dense gradient rows in place.  Update per element
// (no bias correction, as in the reference):
//   m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g g;  p += -lr m / (sqrt(v) + eps)
// Dense groups (1-D parameters, optimizer.py:207-217) update every row.
#include "common.cuh"

namespace cvhrf {
namespace {

constexpr int kMaxGroups = 16;
// One element of the update, in the reference's operation order (moments first, then
// p += -lr m / (sqrt(v) + eps)).
__device__ __forceinline__ void adam_element(const cvhrf_adam_group& G, size_t idx, float b1, float b2) {
  const float g = G.grad[idx];
  const float m = b1 * G.exp_avg[idx] + (1.0f - b1) * g;
  const float v = b2 * G.exp_avg_sq[idx] + (1.0f - b2) * g * g;
  G.param[idx] += -G.lr * m / (sqrtf(v) + G.eps);
  G.exp_avg[idx] = m;
  G.exp_avg_sq[idx] = v;
}

struct AdamLaunch {
  int n;
  cvhrf_adam_group g[kMaxGroups];
  long long start[kMaxGroups + 1];  // element prefix over groups
};

__global__ void __launch_bounds__(256) sparse_adam_kernel(AdamLaunch L, const int64_t* __restrict__ visible,
                                                          float b1, float b2) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= L.start[L.n]) return;
  int gi = 0;
#pragma unroll 1
  while (gi + 1 < L.n && e >= L.start[gi + 1]) ++gi;
  const cvhrf_adam_group& G = L.g[gi];
  const long long local = e - L.start[gi];
  const long long r = local / G.D;
  const int d = (int)(local - r * G.D);
  const long long row = G.dense ? r : visible[r];
  const size_t idx = (size_t)row * G.D + d;
  adam_element(G, idx, b1, b2);
}

}  // namespace
}  // namespace cvhrf

using namespace cvhrf;

extern "C" int cvhrf_sparse_adam(const cvhrf_adam_group* groups, int ngroups, const int64_t* visible, int V, float b1,
                                 float b2, void* stream) {
  if (!groups || ngroups < 0 || ngroups > kMaxGroups || V < 0 || (V > 0 && !visible)) return CVHRF_EINVAL;
  AdamLaunch L{};
  L.n = 0;
  long long tot = 0;
  for (int i = 0; i < ngroups; ++i) {
    const cvhrf_adam_group& g = groups[i];
    if (g.D < 1 || g.N < 0 || !g.param || !g.grad || !g.exp_avg || !g.exp_avg_sq) return CVHRF_EINVAL;
    const long long rows = g.dense ? g.N : V;
    if (rows == 0) continue;
    L.g[L.n] = g;
    L.start[L.n] = tot;
    tot += rows * g.D;
    ++L.n;
  }
  L.start[L.n] = tot;
  if (tot == 0) return CVHRF_OK;
  const long long blocks = (tot + 255) / 256;
  sparse_adam_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(L, visible, b1, b2);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

// ---- row-mask form: every row streamed in order, updated where mask[row] != 0 ----
// Same update as cvhrf_sparse_adam; rows are visited in memory order (coalesced) instead
// of through the visible-index gather, which is faster when most rows are visible and
// lets a visibility union (e.g. an all-reduce MAX over ranks) be used without compaction.
namespace cvhrf {
namespace {

// grid (x: grid-stride over the group's elements, y: group); 32-bit element indices
__global__ void __launch_bounds__(256) sparse_adam_masked_kernel(AdamLaunch L, const uint8_t* __restrict__ mask,
                                                                 int mask_len, float b1, float b2) {
  const cvhrf_adam_group& G = L.g[blockIdx.y];
  const int n = (int)(L.start[blockIdx.y + 1] - L.start[blockIdx.y]);
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
    if (!G.dense) {
      const int row = e / G.D;
      if (row >= mask_len || mask[row] == 0) continue;
    }
    adam_element(G, (size_t)e, b1, b2);
  }
}

__global__ void rows_to_mask_kernel(const int64_t* __restrict__ rows, int V, int mask_len, uint8_t* mask) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < V && rows[i] >= 0 && rows[i] < mask_len) mask[rows[i]] = 1;
}

}  // namespace
}  // namespace cvhrf

extern "C" int cvhrf_rows_to_mask(const int64_t* rows, int V, uint8_t* mask, int mask_len, void* stream) {
  if (V < 0 || mask_len < 0 || (V > 0 && !rows) || (mask_len > 0 && !mask)) return CVHRF_EINVAL;
  cudaStream_t st = (cudaStream_t)stream;
  if (mask_len > 0) CVHRF_CUDA_TRY(cudaMemsetAsync(mask, 0, (size_t)mask_len, st));
  if (V == 0) return CVHRF_OK;
  rows_to_mask_kernel<<<(V + 255) / 256, 256, 0, st>>>(rows, V, mask_len, mask);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

extern "C" int cvhrf_sparse_adam_masked(const cvhrf_adam_group* groups, int ngroups, const uint8_t* mask,
                                        int mask_len, float b1, float b2, void* stream) {
  if (!groups || ngroups < 0 || ngroups > kMaxGroups || mask_len < 0 || (mask_len > 0 && !mask)) return CVHRF_EINVAL;
  AdamLaunch L{};
  long long tot = 0;
  for (int i = 0; i < ngroups; ++i) {
    const cvhrf_adam_group& g = groups[i];
    if (g.D < 1 || g.N < 0 || !g.param || !g.grad || !g.exp_avg || !g.exp_avg_sq) return CVHRF_EINVAL;
    if (g.N == 0) continue;
    L.g[L.n] = g;
    L.start[L.n] = tot;
    tot += (long long)g.N * g.D;
    ++L.n;
  }
  L.start[L.n] = tot;
  if (tot == 0) return CVHRF_OK;
  long long most = 0;
  for (int i = 0; i < L.n; ++i) most = L.start[i + 1] - L.start[i] > most ? L.start[i + 1] - L.start[i] : most;
  if (most >= (1ll << 31)) return CVHRF_EUNSUPPORTED;
  const long long bx = (most + 255) / 256;
  dim3 grid((unsigned)(bx < 148 * 4 ? bx : 148 * 4), L.n);
  sparse_adam_masked_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(L, mask, mask_len, b1, b2);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}
