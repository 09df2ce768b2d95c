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
  for (int i = threadIdx.x; i < skewed_size(nd); i += kRadixThreads) s_hist[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kRadixTile;
  const int64_t end = min(n, base + kRadixTile);
  for (int64_t p = base + threadIdx.x; p < end; p += kRadixThreads)
    atomicAdd(&s_hist[skew((int)((__ldg(keys + p) >> shift) & (nd - 1)))], 1u);
  __syncthreads();
  for (int d = threadIdx.x; d < nd; d += kRadixThreads) hist[(int64_t)d * ntiles + blockIdx.x] = s_hist[skew(d)];
}

// Stable scatter of one tile.  Each warp owns 1024 consecutive elements,
// held in registers as 32 steps of 32 lanes, and a private (skewed) row of
// digit counters.  Elements are first ranked within the tile (digit-major,
// input order within a digit) into shared memory, then every digit's run is
// written to its global slot with consecutive threads on consecutive
// addresses, so global writes are whole sectors.
__global__ __launch_bounds__(kRadixThreads, 2) void radix_downsweep_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, int64_t n, int shift,
    int bits, const uint32_t* __restrict__ hist, int64_t ntiles) {
  constexpr int kSteps = kRadixWarpItems / 32;
  extern __shared__ __align__(16) uint32_t smem_u32[];
  const int nd = 1 << bits;
  const int row = skewed_size(nd);
  uint32_t* s_off = smem_u32;                        // [kRadixWarps][row]
  uint32_t* s_key = s_off + kRadixWarps * row;       // [kRadixTile]
  uint32_t* s_val = s_key + kRadixTile;              // [kRadixTile]
  uint32_t* s_gbase = s_val + kRadixTile;            // [row] global digit start - local start
  unsigned char* s_own = reinterpret_cast<unsigned char*>(s_gbase + row);  // [kRadixWarps][row] lane per digit
  __shared__ uint32_t s_ws[kRadixWarps];
  const uint32_t dmask = (uint32_t)nd - 1u;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < kRadixWarps * row; i += kRadixThreads) s_off[i] = 0;

  const int64_t tile0 = (int64_t)blockIdx.x * kRadixTile;
  const int tile_n = (int)min((int64_t)kRadixTile, n - tile0);
  const int64_t start = tile0 + (int64_t)warp * kRadixWarpItems;
  uint32_t k[kSteps];
#pragma unroll
  for (int j = 0; j < kSteps; ++j) {
    const int64_t p = start + j * 32 + lane;
    k[j] = p < n ? __ldg(keys_in + p) : 0xffffffffu;
  }
  uint32_t* my = s_off + warp * row;
  const unsigned lt = lanemask_lt();
  __syncthreads();

  // A: per-warp digit counts (order does not matter here: shared atomics)
#pragma unroll
  for (int j = 0; j < kSteps; ++j) {
    const bool valid = start + j * 32 + lane < n;
    if (valid) atomicAdd(&my[skew((int)((k[j] >> shift) & dmask))], 1u);
  }
  __syncthreads();

  // B: tile totals per digit -> tile-local digit starts (block scan over
  // digits, up to two digits per thread) and per-warp local offsets
  constexpr int kMaxPer = ((1 << kRadixMaxBits) + kRadixThreads - 1) / kRadixThreads;
  const int per_thread = (nd + kRadixThreads - 1) / kRadixThreads;  // <= kMaxPer
  uint32_t tot[kMaxPer] = {};
  for (int q = 0; q < per_thread; ++q) {
    const int d = threadIdx.x * per_thread + q;
    if (d < nd)
      for (int w = 0; w < kRadixWarps; ++w) tot[q] += s_off[w * row + skew(d)];
  }
  {
    uint32_t mine = 0;
#pragma unroll
    for (int q = 0; q < kMaxPer; ++q) mine += tot[q];
    uint32_t x = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_ws[warp] = x;
    __syncthreads();
    uint32_t wp = 0;
    for (int w = 0; w < warp; ++w) wp += s_ws[w];
    uint32_t run = wp + x - mine;  // exclusive prefix of this thread's first digit
    for (int q = 0; q < per_thread; ++q) {
      const int d = threadIdx.x * per_thread + q;
      if (d < nd) {
        const int sd = skew(d);
        s_gbase[sd] = hist[(int64_t)d * ntiles + blockIdx.x] - run;
        uint32_t r2 = run;
        for (int w = 0; w < kRadixWarps; ++w) {
          const uint32_t c = s_off[w * row + sd];
          s_off[w * row + sd] = r2;
          r2 += c;
        }
        run += tot[q];
      }
    }
  }
  uint32_t v[kSteps];
#pragma unroll
  for (int j = 0; j < kSteps; ++j) {
    const int64_t p = start + j * 32 + lane;
    v[j] = vals_in ? (p < n ? __ldg(vals_in + p) : 0u) : (uint32_t)p;
  }
  __syncthreads();

  // C: stable rank within the tile -> shared memory.  A step whose 32 digits
  // are all different (over half the steps for keys in camera-frustum order)
  // needs no ranking: each lane claims its digit's slot in a per-warp byte
  // table and the warp checks that every lane still owns its slot.
  // Otherwise equal digits are ranked by lane with __match_any_sync.
  unsigned char* own = s_own + warp * row;
  const bool full_warp = start + kRadixWarpItems <= n;
#pragma unroll
  for (int j = 0; j < kSteps; ++j) {
    const bool valid = start + j * 32 + lane < n;
    const uint32_t d = (k[j] >> shift) & dmask;
    const int sd = skew((int)d);
    bool clash = true;
    if (full_warp) {
      own[sd] = (unsigned char)lane;
      __syncwarp();
      clash = __any_sync(0xffffffffu, own[sd] != (unsigned char)lane);
    }
    if (!clash) {
      const uint32_t pos = my[sd];
      s_key[pos] = k[j];
      s_val[pos] = v[j];
      my[sd] = pos + 1;
    } else {
      const unsigned peers = __match_any_sync(0xffffffffu, valid ? d : 0xffffffffu);
      const uint32_t rank = __popc(peers & lt);
      if (valid) {
        const uint32_t pos = my[sd] + rank;
        s_key[pos] = k[j];
        s_val[pos] = v[j];
      }
      __syncwarp();
      if (valid && rank == 0) my[sd] += __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();

  // D: digit runs to global memory, consecutive threads -> consecutive slots
  for (int i = threadIdx.x; i < tile_n; i += kRadixThreads) {
    const uint32_t key = s_key[i];
    const uint32_t pos = s_gbase[skew((int)((key >> shift) & dmask))] + (uint32_t)i;
    keys_out[pos] = key;
    vals_out[pos] = s_val[i];
  }
}

}  // namespace

int radix_sort_index(uint32_t* keys0, uint32_t* keys1, uint32_t* vals_tmp, uint32_t* vals_out,
                     int64_t n, const RadixPlan& plan, uint32_t* hist, uint32_t* scan_scratch,
                     bool hist0_ready, cudaStream_t stream, uint32_t** keys_sorted) {
  return radix_sort_pairs(keys0, keys1, nullptr, vals_tmp, vals_out, n, plan, hist, scan_scratch, hist0_ready,
                          stream, keys_sorted);
}

int radix_sort_pairs(uint32_t* keys0, uint32_t* keys1, const uint32_t* vals_in, uint32_t* vals_tmp,
                     uint32_t* vals_out, int64_t n, const RadixPlan& plan, uint32_t* hist,
                     uint32_t* scan_scratch, bool hist0_ready, cudaStream_t stream, uint32_t** keys_sorted) {
  uint32_t* kbuf[2] = {keys0, keys1};
  if (keys_sorted) *keys_sorted = kbuf[plan.passes & 1];
  if (n == 0) return BFB_OK;
  const int64_t ntiles = radix_tiles(n);
  if (ntiles > 0x7fffffff) return BFB_ERR_TOO_LARGE;
  const uint32_t* vin = vals_in;  // null: pass 0's values are the indices
  for (int ps = 0; ps < plan.passes; ++ps) {
    const int bits = plan.digit_bits[ps], shift = plan.shift[ps];
    const int nd = 1 << bits;
    const uint32_t* kin = kbuf[ps & 1];
    uint32_t* kout = kbuf[(ps + 1) & 1];
    uint32_t* vout = ((plan.passes - 1 - ps) & 1) ? vals_tmp : vals_out;
    if (!(ps == 0 && hist0_ready)) {
      radix_upsweep_kernel<<<(unsigned)ntiles, kRadixThreads, skewed_size(nd) * sizeof(uint32_t), stream>>>(
          kin, n, shift, bits, hist, ntiles);
      BFB_CHECK_LAUNCH();
    }
    BFB_TRY(exclusive_scan_u32(hist, hist, (int64_t)nd * ntiles, scan_scratch, nullptr, stream));
    const size_t smem = ((size_t)kRadixWarps * skewed_size(nd) + 2 * (size_t)kRadixTile + skewed_size(nd)) *
                            sizeof(uint32_t) +
                        (size_t)kRadixWarps * skewed_size(nd);
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
