#include "scan.cuh"

namespace bfb {
namespace {

__global__ __launch_bounds__(kScanThreads) void scan_reduce_kernel(const uint32_t* __restrict__ in,
                                                                   int64_t n,
                                                                   uint32_t* __restrict__ sums) {
  __shared__ uint32_t ws[kScanThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * kScanTile;
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    int64_t p = base + (int64_t)i * kScanThreads + threadIdx.x;
    if (p < n) s += in[p];
  }
  uint32_t total;
  block_exclusive_scan(s, ws, &total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

// Single CTA: exclusive scan of an array in chunks with a running carry.
__global__ __launch_bounds__(kScanThreads) void scan_single_kernel(const uint32_t* in,
                                                                   uint32_t* out, int64_t n,
                                                                   uint32_t* total_dev) {
  __shared__ uint32_t ws[kScanThreads / 32];
  uint32_t carry = 0;
  for (int64_t base = 0; base < n; base += kScanTile) {
    // each thread owns kScanItems consecutive elements
    uint32_t v[kScanItems];
    uint32_t s = 0;
    const int64_t p0 = base + (int64_t)threadIdx.x * kScanItems;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
      v[i] = (p0 + i < n) ? in[p0 + i] : 0u;
      s += v[i];
    }
    uint32_t total;
    uint32_t pre = block_exclusive_scan(s, ws, &total) + carry;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
      if (p0 + i < n) out[p0 + i] = pre;
      pre += v[i];
    }
    carry += total;
  }
  if (threadIdx.x == 0 && total_dev) *total_dev = carry;
}

__global__ __launch_bounds__(kScanThreads) void scan_downsweep_kernel(const uint32_t* in,
                                                                      uint32_t* out, int64_t n,
                                                                      const uint32_t* __restrict__ offs) {
  __shared__ uint32_t ws[kScanThreads / 32];
  const int64_t p0 = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  uint32_t v[kScanItems];
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    v[i] = (p0 + i < n) ? in[p0 + i] : 0u;
    s += v[i];
  }
  uint32_t total;
  uint32_t pre = block_exclusive_scan(s, ws, &total) + offs[blockIdx.x];
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    if (p0 + i < n) out[p0 + i] = pre;
    pre += v[i];
  }
}

}  // namespace

int exclusive_scan_u32(const uint32_t* in, uint32_t* out, int64_t n, uint32_t* scratch,
                       uint32_t* total_dev, cudaStream_t stream) {
  if (n <= kScanSmallMax) {
    scan_single_kernel<<<1, kScanThreads, 0, stream>>>(in, out, n, total_dev);
    BFB_CHECK_LAUNCH();
    return BFB_OK;
  }
  const int64_t nb = ceil_div(n, kScanTile);
  if (nb > kScanMaxBlocks) return BFB_ERR_TOO_LARGE;
  scan_reduce_kernel<<<(unsigned)nb, kScanThreads, 0, stream>>>(in, n, scratch);
  BFB_CHECK_LAUNCH();
  scan_single_kernel<<<1, kScanThreads, 0, stream>>>(scratch, scratch, nb, total_dev);
  BFB_CHECK_LAUNCH();
  scan_downsweep_kernel<<<(unsigned)nb, kScanThreads, 0, stream>>>(in, out, n, scratch);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

}  // namespace bfb
