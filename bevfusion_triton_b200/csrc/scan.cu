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

// Each thread owns kScanItems (8) consecutive elements, moved as two 16-byte
// vectors when the whole tile is in range and both arrays are 16-byte aligned.
__global__ __launch_bounds__(kScanThreads) void scan_downsweep_kernel(const uint32_t* in,
                                                                      uint32_t* out, int64_t n,
                                                                      const uint32_t* __restrict__ offs,
                                                                      bool vec) {
  static_assert(kScanItems == 8, "two 16-byte vectors per thread");
  __shared__ uint32_t ws[kScanThreads / 32];
  const int64_t p0 = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
  const bool full = vec && (int64_t)(blockIdx.x + 1) * kScanTile <= n;  // same for the whole CTA
  uint32_t v[kScanItems];
  if (full) {
    const uint4 a = *reinterpret_cast<const uint4*>(in + p0);
    const uint4 b = *reinterpret_cast<const uint4*>(in + p0 + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) v[i] = (p0 + i < n) ? in[p0 + i] : 0u;
  }
  uint32_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) s += v[i];
  uint32_t total;
  uint32_t pre = block_exclusive_scan(s, ws, &total) + offs[blockIdx.x];
  uint32_t o[kScanItems];
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    o[i] = pre;
    pre += v[i];
  }
  if (full) {
    *reinterpret_cast<uint4*>(out + p0) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(out + p0 + 4) = make_uint4(o[4], o[5], o[6], o[7]);
  } else {
#pragma unroll
    for (int i = 0; i < kScanItems; ++i)
      if (p0 + i < n) out[p0 + i] = o[i];
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
  const bool vec = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  scan_downsweep_kernel<<<(unsigned)nb, kScanThreads, 0, stream>>>(in, out, n, scratch, vec);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

}  // namespace bfb
