// Device-wide inclusive scan and stable LSD radix sort (u32 keys, u32 values), both
// single-pass with decoupled look-back (one launch per scan, one per sort pass).
//
// These replace the CUB calls of the reference binning (cub::DeviceScan::InclusiveSum,
// rasterizer_splat.cu:427, and cub::DeviceRadixSort::SortPairs, :475-480).  The sort
// is stable, so sorting (tile, slot) pairs emitted in (depth, index) order yields
// exactly the reference's (tile, depth, index) order.
#pragma once
#include "common.cuh"

namespace cvhrf {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 16;
constexpr int kScanTile = kScanThreads * kScanItems;   // items per block

constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;   // items per block
constexpr int kSortBits = 8;                           // max bits per pass

inline int scan_blocks(int n) { return (n + kScanTile - 1) / kScanTile; }
inline int sort_blocks(int n) { return (n + kSortTile - 1) / kSortTile; }

// Scratch (u32 count) for an inclusive scan of n items.
size_t scan_scratch_words(int n);
// Inclusive scan in -> out (in == out allowed).  scratch: scan_scratch_words(n) u32.
int inclusive_scan_u32(const uint32_t* in, uint32_t* out, int n, uint32_t* scratch, cudaStream_t st);

// Scratch (u32 count) for sorting n pairs.
size_t sort_scratch_words(int n);
// Stable sort by key bits [begin_bit, end_bit).  Ping-pongs between (k0,v0) and (k1,v1);
// sets *result_in_alt to 1 if the sorted result ended in (k1, v1).  If `skip` (device int)
// is non-null and non-zero when the passes run, every pass is a no-op: with an even
// number of passes the (already sorted) input stays in (k0, v0), which is what a stable
// sort of sorted keys with values 0..n-1 produces.
int radix_sort_pairs(uint32_t* k0, uint32_t* v0, uint32_t* k1, uint32_t* v1, int n, int begin_bit, int end_bit,
                     uint32_t* scratch, cudaStream_t st, int* result_in_alt, const int* skip = nullptr,
                     const int* n_dev = nullptr, bool index_values = false);
// (n_dev, when non-null, is a device count: only the first min(n, *n_dev) items are sorted;
//  n is then the capacity the launch grids are sized for.  index_values: the values are the
//  items' indices 0..n-1 and v0's contents are not read; not combined with skip.)
// *flag = 1 if keys[0..n) is non-decreasing, else 0 (device int, stream-ordered).
int keys_sorted_flag(const uint32_t* keys, int n, int* flag, cudaStream_t st);
// Number of look-back waits that ran out of their iteration limit since the library was
// loaded (each makes that scan/sort result invalid; expected 0).  Synchronises.
int lookback_timeouts();

}  // namespace cvhrf
