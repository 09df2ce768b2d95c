// Device-wide exclusive prefix sums over uint32 arrays.
//
// Reduce-then-scan in three launches for large arrays, one single-CTA launch
// for small ones.  No inter-CTA waiting, so nothing can spin.
#pragma once

#include "common.cuh"

namespace bfb {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;  // per thread
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096
constexpr int64_t kScanSmallMax = 8192;               // single-CTA path up to here
constexpr int64_t kScanMaxBlocks = 1 << 17;          // block sums scanned by one CTA

// Scratch elements (uint32) the scan of n elements needs.
inline size_t scan_scratch_elems(int64_t n) { return (size_t)ceil_div(n, kScanTile) + 2; }

// out[i] = sum(in[0..i)), i < n.  `out` may alias `in`.  If total_dev is not
// null, *total_dev = sum(in[0..n)).  n may be 0.
int exclusive_scan_u32(const uint32_t* in, uint32_t* out, int64_t n, uint32_t* scratch,
                       uint32_t* total_dev, cudaStream_t stream);

// Block-wide exclusive scan of one value per thread; returns the block total
// through *total.  `warp_sums` must hold blockDim.x / 32 entries.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums,
                                                         uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t s = lane < nwarps ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nwarps) warp_sums[lane] = s;  // inclusive
  }
  __syncthreads();
  uint32_t warp_prefix = warp ? warp_sums[warp - 1] : 0;
  *total = warp_sums[nwarps - 1];
  __syncthreads();  // warp_sums reusable after return
  return warp_prefix + x - v;
}

}  // namespace bfb
