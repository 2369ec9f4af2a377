// Device-wide scan and stable LSD radix sort (see scan_sort.cuh).
#include "scan_sort.cuh"

namespace cvhrf {

namespace {

__device__ __forceinline__ uint32_t warp_incl_scan(uint32_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Exclusive block scan of one value per thread (blockDim.x <= 1024); returns the total.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t& total, uint32_t* sh /* 32 */) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  uint32_t inc = warp_incl_scan(v);
  if (lane == 31) sh[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < nw ? sh[lane] : 0u;
    uint32_t wi = warp_incl_scan(w);
    sh[lane] = wi - w;
    if (lane == 31) sh[32] = wi;
  }
  __syncthreads();
  uint32_t r = sh[warp] + inc - v;
  total = sh[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kScanThreads) scan_reduce_kernel(const uint32_t* __restrict__ in, int n,
                                                                    uint32_t* __restrict__ sums) {
  __shared__ uint32_t sh[33];
  const int base = blockIdx.x * kScanTile;
  uint32_t s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int i = base + k * kScanThreads + threadIdx.x;
    if (i < n) s += in[i];
  }
  uint32_t total;
  block_excl_scan(s, total, sh);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Exclusive scan of nb block sums in place (one block of 1024 threads).
__global__ void __launch_bounds__(1024) scan_sums_kernel(uint32_t* sums, int nb) {
  __shared__ uint32_t sh[33];
  uint32_t carry = 0;
  for (int base = 0; base < nb; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const uint32_t v = i < nb ? sums[i] : 0u;
    uint32_t total;
    const uint32_t ex = block_excl_scan(v, total, sh);
    if (i < nb) sums[i] = carry + ex;
    carry += total;
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(const uint32_t* __restrict__ in,
                                                                   uint32_t* __restrict__ out, int n,
                                                                   const uint32_t* __restrict__ offs) {
  __shared__ uint32_t tile[kScanTile + kScanTile / 32];
  __shared__ uint32_t sh[33];
  const int base = blockIdx.x * kScanTile;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = k * kScanThreads + threadIdx.x;
    const int i = base + li;
    tile[li + (li >> 5)] = i < n ? in[i] : 0u;
  }
  __syncthreads();
  uint32_t v[kScanItems];
  uint32_t s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = threadIdx.x * kScanItems + k;
    s += tile[li + (li >> 5)];
    v[k] = s;
  }
  uint32_t total;
  const uint32_t ex = block_excl_scan(s, total, sh) + offs[blockIdx.x];
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = threadIdx.x * kScanItems + k;
    tile[li + (li >> 5)] = v[k] + ex;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = k * kScanThreads + threadIdx.x;
    const int i = base + li;
    if (i < n) out[i] = tile[li + (li >> 5)];
  }
}

// ---- radix sort -----------------------------------------------------------------
__global__ void __launch_bounds__(kSortThreads) radix_hist_kernel(const uint32_t* __restrict__ keys, int n, int shift,
                                                                  int radix, uint32_t* __restrict__ hist, int nb,
                                                                  const int* __restrict__ skip,
                                                                  const int* __restrict__ n_dev) {
  if (skip && *skip) return;
  if (n_dev) n = min(n, *n_dev);
  __shared__ uint32_t h[256];
  for (int d = threadIdx.x; d < 256; d += blockDim.x) h[d] = 0;
  __syncthreads();
  const int base = blockIdx.x * kSortTile;
  const uint32_t mask = (uint32_t)radix - 1;
#pragma unroll
  for (int k = 0; k < kSortItems; ++k) {
    const int i = base + k * kSortThreads + threadIdx.x;
    if (i < n) atomicAdd(&h[(keys[i] >> shift) & mask], 1u);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < radix; d += blockDim.x) hist[d * nb + blockIdx.x] = h[d];
}

// Stable scatter: items are ranked in their original order (round, warp, lane).
__global__ void __launch_bounds__(kSortThreads) radix_scatter_kernel(
    const uint32_t* __restrict__ kin, const uint32_t* __restrict__ vin, uint32_t* __restrict__ kout,
    uint32_t* __restrict__ vout, int n, int shift, int radix, const uint32_t* __restrict__ incl, int nb,
    const int* __restrict__ skip, const int* __restrict__ n_dev) {
  if (skip && *skip) return;
  if (n_dev) n = min(n, *n_dev);
  constexpr int NW = kSortThreads / 32;
  __shared__ uint32_t offs[256];
  __shared__ uint32_t wc[NW][256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = threadIdx.x; d < 256; d += blockDim.x) {
    if (d < radix) {
      const int idx = d * nb + blockIdx.x;
      offs[d] = idx == 0 ? 0u : incl[idx - 1];
    }
#pragma unroll
    for (int w = 0; w < NW; ++w) wc[w][d] = 0;
  }
  __syncthreads();
  const int base = blockIdx.x * kSortTile;
  const uint32_t mask = (uint32_t)radix - 1;
  const unsigned lt = (1u << lane) - 1u;
  for (int k = 0; k < kSortItems; ++k) {
    const int i = base + k * kSortThreads + threadIdx.x;
    const bool valid = i < n;
    uint32_t key = 0, val = 0, d = 256;
    if (valid) {
      key = kin[i];
      val = vin[i];
      d = (key >> shift) & mask;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const uint32_t rank = __popc(peers & lt);
    if (valid && rank == 0) wc[warp][d] = __popc(peers);
    __syncthreads();
    if (valid) {
      uint32_t pre = 0;
      for (int w = 0; w < warp; ++w) pre += wc[w][d];
      const uint32_t pos = offs[d] + pre + rank;
      kout[pos] = key;
      vout[pos] = val;
    }
    __syncthreads();
    for (int dd = threadIdx.x; dd < radix; dd += blockDim.x) {
      uint32_t t = 0;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        t += wc[w][dd];
        wc[w][dd] = 0;
      }
      offs[dd] += t;
    }
    __syncthreads();
  }
}

}  // namespace

__global__ void flag_set_kernel(int* flag) { *flag = 1; }

__global__ void sorted_check_kernel(const uint32_t* __restrict__ keys, int n, int* flag) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i + 1 < n && keys[i] > keys[i + 1]) *flag = 0;
}

int keys_sorted_flag(const uint32_t* keys, int n, int* flag, cudaStream_t st) {
  flag_set_kernel<<<1, 1, 0, st>>>(flag);
  sorted_check_kernel<<<(n + 255) / 256, 256, 0, st>>>(keys, n, flag);
  count_launch(1);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

size_t scan_scratch_words(int n) { return (size_t)scan_blocks(n) + 64; }

int inclusive_scan_u32(const uint32_t* in, uint32_t* out, int n, uint32_t* scratch, cudaStream_t st) {
  if (n <= 0) return CVHRF_OK;
  const int nb = scan_blocks(n);
  scan_reduce_kernel<<<nb, kScanThreads, 0, st>>>(in, n, scratch);
  scan_sums_kernel<<<1, 1024, 0, st>>>(scratch, nb);
  scan_apply_kernel<<<nb, kScanThreads, 0, st>>>(in, out, n, scratch);
  count_launch(2);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

size_t sort_scratch_words(int n) {
  const size_t h = (size_t)256 * sort_blocks(n);
  return align_up(h, 64) + scan_scratch_words((int)h) + 64;
}

int radix_sort_pairs(uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1, int n, int begin_bit, int end_bit,
                     uint32_t* scratch, cudaStream_t st, int* result_in_alt, const int* skip, const int* n_dev) {
  *result_in_alt = 0;
  if (n <= 1 || end_bit <= begin_bit) return CVHRF_OK;
  const int nb = sort_blocks(n);
  uint32_t* hist = scratch;
  uint32_t* sscr = scratch + align_up((size_t)256 * nb, 64);
  uint32_t *ki = k0, *vi = v0, *ko = k1, *vo = v1;
  int alt = 0;
  for (int b = begin_bit; b < end_bit; b += kSortBits) {
    const int bits = min(kSortBits, end_bit - b);
    const int radix = 1 << bits;
    radix_hist_kernel<<<nb, kSortThreads, 0, st>>>(ki, n, b, radix, hist, nb, skip, n_dev);
    count_launch(1);
    int rc = inclusive_scan_u32(hist, hist, radix * nb, sscr, st);
    if (rc) return rc;
    radix_scatter_kernel<<<nb, kSortThreads, 0, st>>>(ki, vi, ko, vo, n, b, radix, hist, nb, skip, n_dev);
    CVHRF_LAUNCH_CHECK();
    uint32_t* t;
    t = ki; ki = ko; ko = t;
    t = vi; vi = vo; vo = t;
    alt ^= 1;
  }
  *result_in_alt = alt;
  return CVHRF_OK;
}

}  // namespace cvhrf
