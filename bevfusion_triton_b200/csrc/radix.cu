#include "radix.cuh"
#include "scan.cuh"

namespace bfb {

RadixPlan make_radix_plan(uint32_t max_key) {
  int bits = 0;
  while (bits < 32 && (max_key >> bits) != 0) ++bits;
  if (bits == 0) bits = 1;
  RadixPlan p;
  p.passes = (bits + kRadixMaxBits - 1) / kRadixMaxBits;
  int per = (bits + p.passes - 1) / p.passes;
  int shift = 0;
  for (int i = 0; i < p.passes; ++i) {
    int b = bits - shift < per ? bits - shift : per;
    p.digit_bits[i] = b;
    p.shift[i] = shift;
    shift += b;
    if (b > p.max_digit_bits) p.max_digit_bits = b;
  }
  return p;
}

namespace {

__global__ __launch_bounds__(kRadixThreads) void radix_upsweep_kernel(const uint32_t* __restrict__ keys,
                                                                      int64_t n, int shift, int bits,
                                                                      uint32_t* __restrict__ hist,
                                                                      int64_t ntiles) {
  extern __shared__ uint32_t s_hist[];
  const int nd = 1 << bits;
  for (int i = threadIdx.x; i < nd; i += kRadixThreads) s_hist[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kRadixTile;
  const int64_t end = min(n, base + kRadixTile);
  for (int64_t p0 = base; p0 < end; p0 += kRadixThreads) {
    const int64_t p = p0 + threadIdx.x;
    const bool valid = p < end;
    radix_count_aggregated(s_hist, valid ? ((__ldg(keys + p) >> shift) & (nd - 1)) : 0u, bits, valid);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < nd; d += kRadixThreads) hist[(int64_t)d * ntiles + blockIdx.x] = s_hist[d];
}

__global__ __launch_bounds__(kRadixThreads) void radix_downsweep_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n, int shift,
    int bits, const uint32_t* __restrict__ hist, int64_t ntiles) {
  extern __shared__ uint32_t s_off[];  // [kRadixWarps][nd]
  const int nd = 1 << bits;
  const uint32_t dmask = (uint32_t)nd - 1u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kRadixWarps * nd; i += kRadixThreads) s_off[i] = 0;
  __syncthreads();

  const int64_t start = (int64_t)blockIdx.x * kRadixTile + (int64_t)warp * kRadixWarpItems;
  const int64_t end = min(n, start + kRadixWarpItems);
  uint32_t* my = s_off + warp * nd;

  // A: per-warp digit counts; one leader per distinct digit in a step updates
  // the warp-private row (input order clusters equal digits, so per-lane
  // shared atomics would serialise)
  {
    const unsigned lt = lanemask_lt();
    for (int64_t base = start; base < end; base += 32) {
      const int64_t p = base + lane;
      const bool valid = p < end;
      const uint32_t d = valid ? ((__ldg(keys_in + p) >> shift) & dmask) : 0u;
      const unsigned peers = digit_peers(d, bits, valid);
      if (valid && (peers & lt) == 0) my[d] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  // B: per-warp starting offsets = global (digit, tile) offset + counts of
  // earlier warps in this tile
  for (int d = threadIdx.x; d < nd; d += kRadixThreads) {
    uint32_t run = hist[(int64_t)d * ntiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kRadixWarps; ++w) {
      uint32_t c = s_off[w * nd + d];
      s_off[w * nd + d] = run;
      run += c;
    }
  }
  __syncthreads();

  // C: stable scatter, 32 consecutive elements per step
  const unsigned lt = lanemask_lt();
  for (int64_t base = start; base < end; base += 32) {
    const int64_t p = base + lane;
    const bool valid = p < end;
    uint32_t k = 0, v = 0;
    if (valid) {
      k = __ldg(keys_in + p);
      v = vals_in ? __ldg(vals_in + p) : (uint32_t)p;
    }
    const uint32_t d = valid ? ((k >> shift) & dmask) : 0u;
    const unsigned peers = digit_peers(d, bits, valid);
    const uint32_t rank = __popc(peers & lt);
    uint32_t pos = 0;
    if (valid) {
      pos = my[d] + rank;
      keys_out[pos] = k;
      vals_out[pos] = v;
    }
    __syncwarp();
    if (valid && rank == 0) my[d] += __popc(peers);
    __syncwarp();
  }
}

}  // namespace

int radix_sort_index(uint32_t* keys0, uint32_t* keys1, uint32_t* vals_tmp, uint32_t* vals_out,
                     int64_t n, const RadixPlan& plan, uint32_t* hist, uint32_t* scan_scratch,
                     bool hist0_ready, cudaStream_t stream, uint32_t** keys_sorted) {
  uint32_t* kbuf[2] = {keys0, keys1};
  if (keys_sorted) *keys_sorted = kbuf[plan.passes & 1];
  if (n == 0) return BFB_OK;
  const int64_t ntiles = radix_tiles(n);
  if (ntiles > 0x7fffffff) return BFB_ERR_TOO_LARGE;
  const uint32_t* vin = nullptr;  // pass 0: values are the indices
  for (int ps = 0; ps < plan.passes; ++ps) {
    const int bits = plan.digit_bits[ps], shift = plan.shift[ps];
    const int nd = 1 << bits;
    const uint32_t* kin = kbuf[ps & 1];
    uint32_t* kout = kbuf[(ps + 1) & 1];
    uint32_t* vout = ((plan.passes - 1 - ps) & 1) ? vals_tmp : vals_out;
    if (!(ps == 0 && hist0_ready)) {
      radix_upsweep_kernel<<<(unsigned)ntiles, kRadixThreads, nd * sizeof(uint32_t), stream>>>(
          kin, n, shift, bits, hist, ntiles);
      BFB_CHECK_LAUNCH();
    }
    BFB_TRY(exclusive_scan_u32(hist, hist, (int64_t)nd * ntiles, scan_scratch, nullptr, stream));
    const size_t smem = (size_t)kRadixWarps * nd * sizeof(uint32_t);
    if (smem > 48 * 1024)
      BFB_CUDA(cudaFuncSetAttribute(radix_downsweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    radix_downsweep_kernel<<<(unsigned)ntiles, kRadixThreads, smem, stream>>>(
        kin, vin, kout, vout, n, shift, bits, hist, ntiles);
    BFB_CHECK_LAUNCH();
    vin = vout;
  }
  return BFB_OK;
}

}  // namespace bfb
