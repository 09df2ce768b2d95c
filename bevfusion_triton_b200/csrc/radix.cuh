// Stable LSD radix sort of 32-bit keys with 32-bit values.
//
// Each pass is upsweep (per-tile digit histogram) -> exclusive scan of the
// digit-major histogram matrix -> downsweep (stable scatter).  The downsweep
// gives every warp a private row of digit offsets: a warp walks its
// contiguous 1024-element sub-range in order and ranks equal digits inside a
// 32-element step with __match_any_sync, so the scatter keeps input order
// (stable) with no inter-CTA waiting.
#pragma once

#include "common.cuh"

namespace bfb {

constexpr int kRadixWarps = 8;
constexpr int kRadixThreads = kRadixWarps * 32;        // 256
constexpr int kRadixWarpItems = 1024;                  // per warp
constexpr int kRadixTile = kRadixWarps * kRadixWarpItems;  // 8192
constexpr int kRadixMaxBits = 10;                      // digit width

// Shared-memory slot of digit d in a per-warp / per-block counter array: one
// padding word per 32 digits, so digits that differ by a multiple of 32 (keys
// that step along a grid row of a multiple-of-32 width) land in different
// banks.
__host__ __device__ __forceinline__ int skew(int d) { return d + (d >> 5); }
__host__ __device__ __forceinline__ int skewed_size(int nd) { return nd + (nd >> 5); }

struct RadixPlan {
  int passes = 0;
  int digit_bits[4] = {0, 0, 0, 0};
  int shift[4] = {0, 0, 0, 0};
  int max_digit_bits = 0;
};

// Number of passes and digit split to sort keys in [0, max_key].
RadixPlan make_radix_plan(uint32_t max_key);

inline int64_t radix_tiles(int64_t n) { return ceil_div(n, kRadixTile); }

// Histogram matrix elements (digit-major) for n keys with the given plan.
inline size_t radix_hist_elems(int64_t n, const RadixPlan& p) {
  return (size_t)(1u << p.max_digit_bits) * (size_t)radix_tiles(n) + 1;
}

// Stable sort of the keys in keys0 carrying their indices: on return
// vals_out[i] is the input position of the i-th smallest key (ties in input
// order) and *keys_sorted points at the sorted keys (keys0 or keys1, by pass
// count).  keys1 and vals_tmp are scratch.  `hist0_ready`: the first pass's
// histogram was produced by the caller (fused into the key-producing kernel),
// so its upsweep is skipped.
int radix_sort_index(uint32_t* keys0, uint32_t* keys1, uint32_t* vals_tmp, uint32_t* vals_out,
                     int64_t n, const RadixPlan& plan, uint32_t* hist, uint32_t* scan_scratch,
                     bool hist0_ready, cudaStream_t stream, uint32_t** keys_sorted);

// The same sort carrying given values: vals_out[i] = vals_in[j] of the
// element j that lands at position i.  vals_in must not alias vals_tmp or
// vals_out.  Two stable sorts chained this way (low word first, then the
// high word carrying the first permutation) order 64-bit keys.
int radix_sort_pairs(uint32_t* keys0, uint32_t* keys1, const uint32_t* vals_in, uint32_t* vals_tmp,
                     uint32_t* vals_out, int64_t n, const RadixPlan& plan, uint32_t* hist,
                     uint32_t* scan_scratch, bool hist0_ready, cudaStream_t stream, uint32_t** keys_sorted);

}  // namespace bfb
