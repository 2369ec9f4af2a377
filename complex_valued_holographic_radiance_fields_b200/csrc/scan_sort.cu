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

// ---- single-pass inclusive scan (decoupled look-back) ---------------------------
// Tiles are numbered in the order their blocks start (atomic ticket), so every tile a
// block waits for is already running and publishes its aggregate without waiting
// itself.  Status word per tile: (flag << 32) | value, flag 1 = aggregate, 2 = inclusive.
constexpr unsigned long long kStAgg = 1ull << 32, kStInc = 2ull << 32;
constexpr int kSpinLimit = 1 << 22;

__device__ int g_lookback_timeouts;

__device__ __forceinline__ unsigned long long ld_status64(const unsigned long long* p) {
  return *(const volatile unsigned long long*)p;
}
__device__ __forceinline__ void st_status64(unsigned long long* p, unsigned long long v) {
  *(volatile unsigned long long*)p = v;
}

__global__ void __launch_bounds__(kScanThreads) scan_lookback_kernel(const uint32_t* __restrict__ in,
                                                                      uint32_t* __restrict__ out, int n,
                                                                      unsigned long long* __restrict__ status,
                                                                      unsigned* __restrict__ ticket) {
  __shared__ uint32_t tile_buf[kScanTile + kScanTile / 32];
  __shared__ uint32_t sh[33];
  __shared__ int s_tile;
  __shared__ uint32_t s_excl;
  if (threadIdx.x == 0) s_tile = (int)atomicAdd(ticket, 1u);
  __syncthreads();
  const int tile = s_tile;
  const int base = tile * kScanTile;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = k * kScanThreads + threadIdx.x;
    const int i = base + li;
    tile_buf[li + (li >> 5)] = i < n ? in[i] : 0u;
  }
  __syncthreads();
  uint32_t v[kScanItems];
  uint32_t run = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = threadIdx.x * kScanItems + k;
    run += tile_buf[li + (li >> 5)];
    v[k] = run;
  }
  uint32_t total;
  const uint32_t ex = block_excl_scan(run, total, sh);
  if (threadIdx.x < 32) {
    // warp 0: publish the aggregate, then look back 32 tiles at a time
    uint32_t excl = 0;
    if (tile == 0) {
      if (threadIdx.x == 0) st_status64(&status[0], kStInc | total);
    } else {
      if (threadIdx.x == 0) st_status64(&status[tile], kStAgg | total);
      int j = tile - 1 - (int)threadIdx.x;
      bool done = false;
      int spins = 0;
      while (!done) {
        unsigned long long st = j >= 0 ? ld_status64(&status[j]) : kStInc;
        while ((st >> 32) == 0 && ++spins < kSpinLimit) st = ld_status64(&status[j]);
        if ((st >> 32) == 0) {  // bounded wait ran out: record it and stop (result invalid)
          if (threadIdx.x == 0) atomicAdd(&g_lookback_timeouts, 1);
          st = kStInc;
        }
        const bool inc = (st >> 32) == 2;
        const unsigned incmask = __ballot_sync(0xffffffffu, inc);
        // lanes up to and including the nearest inclusive tile contribute
        const int first_inc = incmask ? __ffs(incmask) - 1 : 32;
        uint32_t val = (j >= 0 && (int)threadIdx.x <= first_inc) ? (uint32_t)(st & 0xffffffffu) : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) val += __shfl_xor_sync(0xffffffffu, val, o);
        excl += val;
        done = incmask != 0;
        j -= 32;
      }
      if (threadIdx.x == 0) st_status64(&status[tile], kStInc | (excl + total));
    }
    if (threadIdx.x == 0) s_excl = excl;
  }
  __syncthreads();
  const uint32_t off = ex + s_excl;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = threadIdx.x * kScanItems + k;
    tile_buf[li + (li >> 5)] = v[k] + off;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    const int li = k * kScanThreads + threadIdx.x;
    const int i = base + li;
    if (i < n) out[i] = tile_buf[li + (li >> 5)];
  }
}

// ---- onesweep LSD radix sort -------------------------------------------------------
// Per sort: one histogram kernel (all passes' digit counts in one read of the keys), then
// one kernel per pass.  A pass block takes the next tile by ticket, ranks its keys stably
// (warp w owns a contiguous 256-key run; within a run, 8 rounds of 32 keys ranked with
// __match_any_sync), publishes its per-digit counts and looks back over earlier tiles
// (one thread per digit) for the digit's running offset, then scatters.
constexpr int kOsThreads = 256, kOsWarps = 8, kOsItems = 8, kOsTile = kOsThreads * kOsItems;
constexpr uint32_t kOsAgg = 1u << 30, kOsInc = 2u << 30, kOsVal = (1u << 30) - 1;
constexpr int kOsMaxPasses = 4;

inline int os_blocks(int n) { return (n + kOsTile - 1) / kOsTile; }

__global__ void __launch_bounds__(256) onesweep_hist_kernel(const uint32_t* __restrict__ keys, int n,
                                                            const int* __restrict__ n_dev,
                                                            const int* __restrict__ skip, int begin_bit,
                                                            int end_bit, int npass, uint32_t* __restrict__ ghist) {
  if (skip && *skip) return;
  if (n_dev) n = min(n, *n_dev);
  __shared__ uint32_t h[kOsMaxPasses][256];
  for (int i = threadIdx.x; i < kOsMaxPasses * 256; i += blockDim.x) (&h[0][0])[i] = 0;
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t k = keys[i];
    for (int p = 0; p < npass; ++p) {
      const int b = begin_bit + 8 * p;
      const uint32_t m = end_bit - b >= 8 ? 0xffu : (1u << (end_bit - b)) - 1u;  // the pass's digit width
      atomicAdd(&h[p][(k >> b) & m], 1u);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < npass * 256; i += blockDim.x) {
    const uint32_t c = (&h[0][0])[i];
    if (c) atomicAdd(&ghist[i], c);
  }
}

__device__ __forceinline__ uint32_t ld_status32(const uint32_t* p) { return *(const volatile uint32_t*)p; }
__device__ __forceinline__ void st_status32(uint32_t* p, uint32_t v) { *(volatile uint32_t*)p = v; }

__global__ void __launch_bounds__(kOsThreads) onesweep_pass_kernel(
    const uint32_t* __restrict__ kin, const uint32_t* __restrict__ vin /* null: values = indices */,
    uint32_t* __restrict__ kout,
    uint32_t* __restrict__ vout, int n, const int* __restrict__ n_dev, const int* __restrict__ skip, int shift,
    int bits, const uint32_t* __restrict__ ghist, uint32_t* __restrict__ status, unsigned* __restrict__ ticket) {
  if (skip && *skip) return;
  if (n_dev) n = min(n, *n_dev);
  if (n > 0 && ghist[(kin[0] >> shift) & ((1u << bits) - 1u)] == (uint32_t)n) {
    // every key has the same digit in this pass: the stable order is the identity, so the
    // pass is a copy (no ranking, no look-back)
    for (int i = blockIdx.x * kOsThreads + threadIdx.x; i < n; i += gridDim.x * kOsThreads) {
      kout[i] = kin[i];
      vout[i] = vin ? vin[i] : (uint32_t)i;
    }
    return;
  }
  __shared__ uint32_t s_wcnt[kOsWarps][256];
  __shared__ uint32_t s_goff[256];
  __shared__ uint32_t s_bstart[256];
  __shared__ uint32_t s_key[kOsTile], s_val[kOsTile];
  __shared__ uint32_t sh[33];
  __shared__ int s_tile;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_tile = (int)atomicAdd(ticket, 1u);
  for (int i = tid; i < kOsWarps * 256; i += kOsThreads) (&s_wcnt[0][0])[i] = 0;
  // global offset of each digit: exclusive scan of this pass's histogram
  {
    uint32_t total;
    const uint32_t c = ghist[tid];
    s_goff[tid] = block_excl_scan(c, total, sh);
  }
  __syncthreads();
  const int tile = s_tile;
  const uint32_t mask = (1u << bits) - 1u;
  const int base = tile * kOsTile + warp * (32 * kOsItems);
  const unsigned lt = (1u << lane) - 1u;
  uint32_t key[kOsItems], val[kOsItems], rank[kOsItems];
#pragma unroll
  for (int r = 0; r < kOsItems; ++r) {
    const int i = base + r * 32 + lane;
    const bool valid = i < n;
    key[r] = valid ? kin[i] : 0u;
    val[r] = valid ? (vin ? vin[i] : (uint32_t)i) : 0u;
    const uint32_t d = valid ? (key[r] >> shift) & mask : 256u;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    uint32_t before = 0;
    if (valid) before = s_wcnt[warp][d];
    rank[r] = before + __popc(peers & lt);
    __syncwarp();
    if (valid && (peers & lt) == 0) s_wcnt[warp][d] = before + __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // per digit: exclusive offsets over warps, then the look-back over earlier tiles
  {
    const int d = tid;
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kOsWarps; ++w) {
      const uint32_t c = s_wcnt[w][d];
      s_wcnt[w][d] = run;
      run += c;
    }
    uint32_t btotal;
    s_bstart[d] = block_excl_scan(run, btotal, sh);  // start of digit d inside this tile
    uint32_t excl = 0;
    uint32_t* my = status + (size_t)tile * 256 + d;
    if (tile == 0) {
      st_status32(my, kOsInc | run);
    } else {
      st_status32(my, kOsAgg | run);
      for (int j = tile - 1; j >= 0; --j) {
        uint32_t st = ld_status32(status + (size_t)j * 256 + d);
        int spins = 0;
        while ((st >> 30) == 0 && ++spins < kSpinLimit) st = ld_status32(status + (size_t)j * 256 + d);
        if ((st >> 30) == 0) {  // bounded wait ran out: record it and stop (result invalid)
          atomicAdd(&g_lookback_timeouts, 1);
          break;
        }
        excl += st & kOsVal;
        if ((st >> 30) == 2) break;
      }
      st_status32(my, kOsInc | (excl + run));
    }
    s_goff[d] += excl;
  }
  __syncthreads();
  // order the tile by digit in shared memory, then write each digit's run contiguously
#pragma unroll
  for (int r = 0; r < kOsItems; ++r) {
    const int i = base + r * 32 + lane;
    if (i < n) {
      const uint32_t d = (key[r] >> shift) & mask;
      const uint32_t local = s_bstart[d] + s_wcnt[warp][d] + rank[r];
      s_key[local] = key[r];
      s_val[local] = val[r];
    }
  }
  __syncthreads();
  const int cnt = min(kOsTile, n - tile * kOsTile);
  for (int i = tid; i < cnt; i += kOsThreads) {
    const uint32_t k = s_key[i];
    const uint32_t d = (k >> shift) & mask;
    const uint32_t pos = s_goff[d] + (uint32_t)i - s_bstart[d];
    kout[pos] = k;
    vout[pos] = s_val[i];
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

// scan scratch: ticket (u64 slot) + one 64-bit status word per tile
size_t scan_scratch_words(int n) { return 2 * ((size_t)scan_blocks(n) + 2) + 64; }

int inclusive_scan_u32(const uint32_t* in, uint32_t* out, int n, uint32_t* scratch, cudaStream_t st) {
  if (n <= 0) return CVHRF_OK;
  const int nb = scan_blocks(n);
  unsigned long long* status = reinterpret_cast<unsigned long long*>(align_up((uintptr_t)scratch, 8));
  unsigned* ticket = reinterpret_cast<unsigned*>(status + nb);
  CVHRF_CUDA_TRY(cudaMemsetAsync(status, 0, ((size_t)nb + 1) * sizeof(unsigned long long), st));
  scan_lookback_kernel<<<nb, kScanThreads, 0, st>>>(in, out, n, status, ticket);
  CVHRF_LAUNCH_CHECK();
  return CVHRF_OK;
}

// sort scratch: per-pass histograms (256 each), tickets, per-pass tile status (256 per tile)
size_t sort_scratch_words(int n) {
  return (size_t)kOsMaxPasses * 256 + 64 + (size_t)kOsMaxPasses * 256 * os_blocks(n > 0 ? n : 1) + 64;
}

int radix_sort_pairs(uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1, int n, int begin_bit, int end_bit,
                     uint32_t* scratch, cudaStream_t st, int* result_in_alt, const int* skip, const int* n_dev,
                     bool index_values) {
  *result_in_alt = 0;
  if (index_values && skip) return CVHRF_EINVAL;
  if (n <= 1 || end_bit <= begin_bit) return CVHRF_OK;
  if (n > (int)kOsVal) return CVHRF_EUNSUPPORTED;
  const int npass = (end_bit - begin_bit + 7) / 8;
  if (npass > kOsMaxPasses) return CVHRF_EUNSUPPORTED;
  const int nb = os_blocks(n);
  uint32_t* ghist = scratch;                                   // npass x 256
  unsigned* tickets = scratch + kOsMaxPasses * 256;             // npass
  uint32_t* status = scratch + kOsMaxPasses * 256 + 64;         // npass x nb x 256
  CVHRF_CUDA_TRY(cudaMemsetAsync(scratch, 0, ((size_t)kOsMaxPasses * 256 + 64 + (size_t)npass * nb * 256) * 4, st));
  const int hb = nb < 148 * 8 ? nb : 148 * 8;
  onesweep_hist_kernel<<<hb, 256, 0, st>>>(k0, n, n_dev, skip, begin_bit, end_bit, npass, ghist);
  CVHRF_LAUNCH_CHECK();
  uint32_t *ki = k0, *vi = v0, *ko = k1, *vo = v1;
  int alt = 0;
  for (int p = 0; p < npass; ++p) {
    const int b = begin_bit + 8 * p;
    const int bits = min(8, end_bit - b);
    onesweep_pass_kernel<<<nb, kOsThreads, 0, st>>>(ki, (index_values && p == 0) ? nullptr : vi, ko, vo, n, n_dev,
                                                    skip, b, bits, ghist + 256 * p, status + (size_t)p * nb * 256,
                                                    tickets + p);
    CVHRF_LAUNCH_CHECK();
    uint32_t* t;
    t = ki; ki = ko; ko = t;
    t = vi; vi = vo; vo = t;
    alt ^= 1;
  }
  *result_in_alt = alt;
  return CVHRF_OK;
}

int lookback_timeouts() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_lookback_timeouts, sizeof(int));
  return v;
}

}  // namespace cvhrf

// ---- C ABI: the binning's scan and sort as standalone entry points ----------------

using namespace cvhrf;

extern "C" size_t cvhrf_sort_pairs_workspace_bytes(int n) {
  if (n < 0) return 0;
  const size_t m = n > 0 ? n : 1;
  return 2 * align_up(m * sizeof(uint32_t), 256) + align_up(sort_scratch_words((int)m) * sizeof(uint32_t), 256);
}

extern "C" int cvhrf_sort_pairs_u32(uint32_t* keys, uint32_t* values, int n, int begin_bit, int end_bit,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0 || (n > 0 && (!keys || !values)) || begin_bit < 0 || end_bit > 32 || begin_bit > end_bit)
    return CVHRF_EINVAL;
  if (n <= 1 || begin_bit == end_bit) return CVHRF_OK;
  Carver cv(workspace, workspace_bytes);
  uint32_t* k1 = cv.take<uint32_t>(n);
  uint32_t* v1 = cv.take<uint32_t>(n);
  uint32_t* scr = cv.take<uint32_t>(sort_scratch_words(n));
  if (cv.overflow || !workspace) return CVHRF_EWORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  int alt = 0, rc;
  if ((rc = radix_sort_pairs(keys, values, k1, v1, n, begin_bit, end_bit, scr, st, &alt))) return rc;
  if (alt) {
    CVHRF_CUDA_TRY(cudaMemcpyAsync(keys, k1, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
    CVHRF_CUDA_TRY(cudaMemcpyAsync(values, v1, (size_t)n * 4, cudaMemcpyDeviceToDevice, st));
  }
  return CVHRF_OK;
}

extern "C" size_t cvhrf_inclusive_scan_workspace_bytes(int n) {
  if (n < 0) return 0;
  return align_up(scan_scratch_words(n > 0 ? n : 1) * sizeof(uint32_t), 256);
}

extern "C" int cvhrf_inclusive_scan_u32(const uint32_t* in, uint32_t* out, int n, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (n < 0 || (n > 0 && (!in || !out))) return CVHRF_EINVAL;
  if (n == 0) return CVHRF_OK;
  if (!workspace || workspace_bytes < cvhrf_inclusive_scan_workspace_bytes(n)) return CVHRF_EWORKSPACE;
  return inclusive_scan_u32(in, out, n, (uint32_t*)workspace, (cudaStream_t)stream);
}

extern "C" int cvhrf_lookback_timeouts(void) { return lookback_timeouts(); }
