// Dynamic scatter (per-voxel reduce of point features) for sm_100a.
//
// Reference semantics: ops/voxel/src/scatter_points_triton.py
//   :150-164  rows with any negative coordinate are invalid (_clean_coors)
//   :166-228  unique rows in ascending lexicographic order, point->voxel map
//             (-1 for invalid rows) and per-voxel counts
//   :253-314  reduce 'sum' / 'none' (sum), 'mean' (sum / count), 'max'
//   :317-424  backward: sum copies, mean divides by the count, max sends each
//             channel's gradient to the lowest point index whose feature equals
//             the reduced value
//
// Design: each valid row gets a packed lexicographic key whose per-column bit
// widths come from the grid extents (when the caller knows them) or from the
// column maxima (one device pass and one host read).  Keys of up to 31 bits
// are sorted in one stable radix sort; wider keys (up to 62 bits, e.g. batched
// (b, x, y, z) rows on a LiDAR grid) are sorted low word first and then by
// the high word carrying the first permutation, which orders them as 64-bit
// keys.  Equal rows then sit together with their points in ascending index
// order; segment heads are scanned into voxel ids, and a group of lanes per
// voxel reduces its points in that order in fp32 with 16-byte row loads (sums
// therefore follow torch.index_add_'s order exactly).
#include <algorithm>
#include <cmath>

#include "radix.cuh"
#include "scan.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_scatter)
namespace {

constexpr int kThreads = 256;
constexpr int kMaxKeyBits = 62;

struct ScatterWs {
  int32_t* dmax;       // [8]  per-column maxima
  uint32_t* status;    // [8]  [0]: rows with a coordinate past the given extent
  uint32_t* lo0;       // [n]  key (narrow) or its low word (wide)
  uint32_t* lo1;       // [n]
  uint32_t* lo_keep;   // [n]  low words in input order (wide)
  uint32_t* hi0;       // [n]  high words (wide)
  uint32_t* hi1;       // [n]
  uint32_t* vtmp;      // [n]
  uint32_t* perm1;     // [n]  order by low word (wide)
  uint32_t* perm;      // [n]  final order
  uint32_t* head;      // [n+1] segment-head flags, then voxel id of each sorted position
  uint32_t* seg;       // [n+1] sorted start of every voxel
  uint32_t* hist;
  uint32_t* scan;
};

size_t carve_ws(void* base, int64_t n, ScatterWs* w) {
  RadixPlan rp;
  rp.max_digit_bits = kRadixMaxBits;  // upper bound over every key width
  Carver c(base);
  w->dmax = c.take<int32_t>(8);
  w->status = c.take<uint32_t>(8);
  w->lo0 = c.take<uint32_t>((size_t)n);
  w->lo1 = c.take<uint32_t>((size_t)n);
  w->lo_keep = c.take<uint32_t>((size_t)n);
  w->hi0 = c.take<uint32_t>((size_t)n);
  w->hi1 = c.take<uint32_t>((size_t)n);
  w->vtmp = c.take<uint32_t>((size_t)n);
  w->perm1 = c.take<uint32_t>((size_t)n);
  w->perm = c.take<uint32_t>((size_t)n);
  w->head = c.take<uint32_t>((size_t)n + 1);
  w->seg = c.take<uint32_t>((size_t)n + 1);
  const size_t h = radix_hist_elems(n, rp);
  w->hist = c.take<uint32_t>(h);
  w->scan = c.take<uint32_t>(scan_scratch_elems((int64_t)h > n + 1 ? (int64_t)h : n + 1));
  return c.bytes();
}

__global__ void dim_max_kernel(const int32_t* __restrict__ coors, int64_t n, int ndim, int32_t* dmax) {
  __shared__ int32_t s[8];
  if (threadIdx.x < 8) s[threadIdx.x] = -1;
  __syncthreads();
  int32_t m[4] = {-1, -1, -1, -1};
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    bool ok = true;
    for (int d = 0; d < ndim; ++d) ok &= coors[i * ndim + d] >= 0;
    if (ok)
      for (int d = 0; d < ndim; ++d) m[d] = max(m[d], coors[i * ndim + d]);
  }
  for (int d = 0; d < ndim; ++d) atomicMax(&s[d], m[d]);
  __syncthreads();
  if (threadIdx.x < ndim) atomicMax(&dmax[threadIdx.x], s[threadIdx.x]);
}

struct KeySpec {
  int ndim;
  int bits;            // total key width
  bool wide;           // bits > 31: two 32-bit words
  int shift[4];        // of each column inside the 64-bit key
  uint32_t extent[4];  // 0 = unchecked
  uint32_t invalid;    // key (narrow) or high word (wide) of a row with a negative coordinate: sorts last
};

__global__ void row_keys_kernel(const int32_t* __restrict__ coors, int64_t n, KeySpec ks, uint32_t* __restrict__ lo,
                                uint32_t* __restrict__ lo_keep, uint32_t* __restrict__ hi,
                                uint32_t* __restrict__ status) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint64_t k = 0;
  bool ok = true, over = false;
  for (int d = 0; d < ks.ndim; ++d) {
    const int32_t v = coors[i * ks.ndim + d];
    ok &= v >= 0;
    over |= ks.extent[d] != 0u && v >= 0 && (uint32_t)v >= ks.extent[d];
    k |= (uint64_t)(uint32_t)v << ks.shift[d];
  }
  if (ok && over) atomicAdd(status, 1u);
  if (!ks.wide) {
    lo[i] = ok ? (uint32_t)k : ks.invalid;
  } else {
    const uint32_t l = ok ? (uint32_t)k : 0u;
    lo[i] = l;
    lo_keep[i] = l;
    hi[i] = ok ? (uint32_t)(k >> 32) : ks.invalid;
  }
}

__global__ void gather_u32_kernel(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx, int64_t n,
                                  uint32_t* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __ldg(src + __ldg(idx + i));
}

// The sorted key at position i: its primary word and, for wide keys, the low
// word (in the same final order).
struct SortedKeys {
  const uint32_t* key;
  const uint32_t* lo;  // null for narrow keys
  uint32_t invalid;
  __device__ __forceinline__ bool same(int64_t i, int64_t j) const {
    return key[i] == key[j] && (!lo || lo[i] == lo[j]);
  }
  __device__ __forceinline__ bool bad(int64_t i) const { return key[i] == invalid; }
};

__global__ void seg_head_kernel(SortedKeys sk, int64_t n, uint32_t* __restrict__ head) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  head[i] = (!sk.bad(i) && (i == 0 || !sk.same(i, i - 1))) ? 1u : 0u;
}

// head (scanned) -> voxel id per sorted position; map, unique coords, segment starts
__global__ void seg_assign_kernel(SortedKeys sk, const uint32_t* __restrict__ perm, int64_t n,
                                  const uint32_t* __restrict__ vid, const int32_t* __restrict__ coors, int ndim,
                                  int32_t* __restrict__ map, int32_t* __restrict__ out_coors,
                                  uint32_t* __restrict__ seg) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t p = perm[i];
  if (sk.bad(i)) {
    map[p] = -1;
    if (i == 0 || !sk.bad(i - 1)) seg[vid[n]] = (uint32_t)i;  // end of the last voxel
    return;
  }
  const uint32_t m = vid[i + 1] - 1;  // inclusive count of heads up to i, minus one
  if (BFB_BAD(m < (uint64_t)n)) return;
  map[p] = (int32_t)m;
  if (i == 0 || !sk.same(i, i - 1)) {
    seg[m] = (uint32_t)i;
    for (int d = 0; d < ndim; ++d) out_coors[(int64_t)m * ndim + d] = coors[(int64_t)p * ndim + d];
  }
  if (i == n - 1) seg[vid[n]] = (uint32_t)n;
}

__global__ void seg_count_kernel(const uint32_t* __restrict__ seg, const uint32_t* __restrict__ total,
                                 int32_t* __restrict__ counts) {
  const int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= (int64_t)*total) return;
  counts[m] = (int32_t)(seg[m + 1] - seg[m]);
}

// VE consecutive channels of one row, as fp32 (one 16-byte load when VE > 1).
template <class T, int VE>
__device__ __forceinline__ void load_row(const T* p, float (&f)[VE]) {
  if constexpr (VE == 1) {
    f[0] = to_f32<T>(__ldg(p));
  } else {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int q = 0; q < VE; ++q) f[q] = to_f32<T>(e[q]);
  }
}

// reduce: 0 sum, 1 mean, 2 max.  A group of 2^glog lanes per voxel; each lane
// owns channel vectors lane, lane + G, ...  Points are taken in sorted
// (ascending index) order, kU row loads in flight ahead of the adds.
template <class T, int VE>
__global__ __launch_bounds__(kThreads) void seg_reduce_kernel(const T* __restrict__ feats, int64_t c, int nvec,
                                                              int glog, const uint32_t* __restrict__ perm,
                                                              const uint32_t* __restrict__ seg,
                                                              const uint32_t* __restrict__ total, int reduce,
                                                              T* __restrict__ out) {
  constexpr int kU = 4;
  const int G = 1 << glog;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int sub = (int)(tid & (G - 1));
  const int64_t groups = ((int64_t)gridDim.x * blockDim.x) >> glog;
  const int64_t m_total = *total;
  for (int64_t m = tid >> glog; m < m_total; m += groups) {
    const uint32_t a = seg[m], b = seg[m + 1];
    for (int v = sub; v < nvec; v += G) {
      float acc[VE];
#pragma unroll
      for (int q = 0; q < VE; ++q) acc[q] = reduce == 2 ? -INFINITY : 0.f;
      for (uint32_t i = a; i < b; i += kU) {
        float r[kU][VE];
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (i + u < b) load_row<T, VE>(feats + (int64_t)__ldg(perm + i + u) * c + (int64_t)v * VE, r[u]);
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (i + u < b) {
#pragma unroll
            for (int q = 0; q < VE; ++q) acc[q] = reduce == 2 ? fmaxf(acc[q], r[u][q]) : __fadd_rn(acc[q], r[u][q]);
          }
      }
      T* dst = out + m * c + (int64_t)v * VE;
#pragma unroll
      for (int q = 0; q < VE; ++q) dst[q] = from_f32<T>(reduce == 1 ? __fdiv_rn(acc[q], (float)(b - a)) : acc[q]);
    }
  }
}

// Element kernels over n * c < 2^31 elements: 32-bit indices, the channel
// split by a precomputed divisor (no 64-bit division per element).
template <class T>
__global__ void grad_sum_kernel(const T* __restrict__ gout, const int32_t* __restrict__ map,
                                const int32_t* __restrict__ counts, uint32_t total, FastDiv cdiv, int mean,
                                T* __restrict__ gfeat) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const uint32_t i = cdiv.div(idx), ch = idx - i * cdiv.d;
  const int32_t m = __ldg(map + i);
  if (m < 0) {
    gfeat[idx] = from_f32<T>(0.f);
    return;
  }
  float g = to_f32<T>(__ldg(gout + (int64_t)m * cdiv.d + ch));
  if (mean) g = __fdiv_rn(g, (float)__ldg(counts + m));
  gfeat[idx] = from_f32<T>(g);
}

template <class T>
__global__ void grad_argmax_kernel(const T* __restrict__ feats, const T* __restrict__ reduced,
                                   const int32_t* __restrict__ map, uint32_t total, FastDiv cdiv,
                                   int32_t* __restrict__ from) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const uint32_t i = cdiv.div(idx), ch = idx - i * cdiv.d;
  const int32_t m = __ldg(map + i);
  if (m < 0) return;
  const int64_t o = (int64_t)m * cdiv.d + ch;
  if (to_f32<T>(__ldg(feats + idx)) == to_f32<T>(__ldg(reduced + o))) atomicMin(&from[o], (int32_t)i);
}

template <class T>
__global__ void grad_max_scatter_kernel(const T* __restrict__ gout, const int32_t* __restrict__ from, uint32_t total,
                                        FastDiv cdiv, int64_t n, T* __restrict__ gfeat) {
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int32_t src = __ldg(from + idx);
  const uint32_t ch = idx - cdiv.div(idx) * cdiv.d;
  if (src < n) gfeat[(int64_t)src * cdiv.d + ch] = __ldg(gout + idx);
}

int width_of(int64_t max_value) {
  int b = 0;
  while (b < 31 && ((int64_t)1 << b) <= max_value) ++b;
  return b;
}

template <class T>
int scatter_forward_t(const void* feats, const int32_t* coors, int64_t n, int64_t c, int64_t ndim, int reduce,
                      const int64_t* extents, const ScatterWs& w, void* out_feats, int32_t* out_coors, int32_t* map,
                      int32_t* counts, int64_t* m_out, cudaStream_t st) {
  KeySpec ks{};
  ks.ndim = (int)ndim;
  int width[4] = {0, 0, 0, 0};
  if (extents) {
    for (int d = 0; d < ndim; ++d) {
      if (extents[d] <= 0 || extents[d] > 0x7fffffffLL) return BFB_ERR_INVALID_ARG;
      width[d] = width_of(extents[d] - 1);
      ks.extent[d] = (uint32_t)extents[d];
    }
  } else {
    BFB_CUDA(cudaMemsetAsync(w.dmax, 0xff, 8 * sizeof(int32_t), st));
    dim_max_kernel<<<(unsigned)std::min<int64_t>(ceil_div(n, kThreads), 1184), kThreads, 0, st>>>(coors, n, (int)ndim,
                                                                                                  w.dmax);
    BFB_CHECK_LAUNCH();
    int32_t dmax[4] = {-1, -1, -1, -1};
    BFB_CUDA(cudaMemcpyAsync(dmax, w.dmax, sizeof(int32_t) * ndim, cudaMemcpyDeviceToHost, st));
    BFB_CUDA(cudaStreamSynchronize(st));
    for (int d = 0; d < ndim; ++d) width[d] = width_of(dmax[d]);
  }
  int bits = 0;
  for (int d = (int)ndim - 1; d >= 0; --d) {
    ks.shift[d] = bits;
    bits += width[d];
  }
  if (bits > kMaxKeyBits) return BFB_ERR_TOO_LARGE;
  ks.bits = bits;
  ks.wide = bits > 31;
  ks.invalid = ks.wide ? (1u << (bits - 32)) : (bits == 0 ? 1u : (1u << bits));  // above every valid key
  BFB_CUDA(cudaMemsetAsync(w.status, 0, 8 * sizeof(uint32_t), st));
  const unsigned nb = (unsigned)ceil_div(n, kThreads);
  row_keys_kernel<<<nb, kThreads, 0, st>>>(coors, n, ks, w.lo0, w.lo_keep, w.hi0, w.status);
  BFB_CHECK_LAUNCH();

  SortedKeys sk{};
  sk.invalid = ks.invalid;
  if (!ks.wide) {
    uint32_t* sorted = nullptr;
    BFB_TRY(radix_sort_index(w.lo0, w.lo1, w.vtmp, w.perm, n, make_radix_plan(ks.invalid), w.hist, w.scan, false, st,
                             &sorted));
    sk.key = sorted;
  } else {
    // low word first (all 32 bits), then the high word carrying that order
    BFB_TRY(radix_sort_index(w.lo0, w.lo1, w.vtmp, w.perm1, n, make_radix_plan(0xffffffffu), w.hist, w.scan, false,
                             st, nullptr));
    gather_u32_kernel<<<nb, kThreads, 0, st>>>(w.hi0, w.perm1, n, w.hi1);
    BFB_CHECK_LAUNCH();
    uint32_t* sorted = nullptr;
    BFB_TRY(radix_sort_pairs(w.hi1, w.hi0, w.perm1, w.vtmp, w.perm, n, make_radix_plan(ks.invalid), w.hist, w.scan,
                             false, st, &sorted));
    uint32_t* lo_final = sorted == w.hi1 ? w.hi0 : w.hi1;  // the free key buffer
    gather_u32_kernel<<<nb, kThreads, 0, st>>>(w.lo_keep, w.perm, n, lo_final);
    BFB_CHECK_LAUNCH();
    sk.key = sorted;
    sk.lo = lo_final;
  }
  seg_head_kernel<<<nb, kThreads, 0, st>>>(sk, n, w.head);
  BFB_CHECK_LAUNCH();
  // inclusive voxel ids: vid[i + 1] = heads in [0, i]; vid[n] = M
  BFB_CUDA(cudaMemsetAsync(w.head + n, 0, sizeof(uint32_t), st));
  BFB_TRY(exclusive_scan_u32(w.head, w.head, n + 1, w.scan, nullptr, st));
  seg_assign_kernel<<<nb, kThreads, 0, st>>>(sk, w.perm, n, w.head, coors, (int)ndim, map, out_coors, w.seg);
  BFB_CHECK_LAUNCH();
  seg_count_kernel<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, st>>>(w.seg, w.head + n, counts);
  BFB_CHECK_LAUNCH();
  const bool v16 = (c * (int64_t)sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(feats) & 15) == 0;
  constexpr int kVE = 16 / sizeof(T);
  const int nvec = v16 ? (int)(c / kVE) : (int)c;
  int glog = 0;
  while ((1 << glog) < nvec && glog < 5) ++glog;
  // grid sized for the worst case (one voxel per point); groups stride over the voxels
  const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div(n << glog, kThreads), 148 * 16);
  if (v16)
    seg_reduce_kernel<T, kVE><<<blocks, kThreads, 0, st>>>(static_cast<const T*>(feats), c, nvec, glog, w.perm, w.seg,
                                                          w.head + n, reduce, static_cast<T*>(out_feats));
  else
    seg_reduce_kernel<T, 1><<<blocks, kThreads, 0, st>>>(static_cast<const T*>(feats), c, nvec, glog, w.perm, w.seg,
                                                        w.head + n, reduce, static_cast<T*>(out_feats));
  BFB_CHECK_LAUNCH();
  // the one host read: the voxel count (the caller sizes its outputs by it)
  uint32_t m = 0, over = 0;
  BFB_CUDA(cudaMemcpyAsync(&m, w.head + n, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaMemcpyAsync(&over, w.status, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  *m_out = m;
  return over ? BFB_ERR_DEVICE_STATUS : BFB_OK;
}

template <class T>
int scatter_backward_t(void* gfeat, const void* gout, const void* feats, const void* reduced, const int32_t* map,
                       const int32_t* counts, int64_t n, int64_t m, int64_t c, int reduce, int32_t* from,
                       cudaStream_t st) {
  if (n == 0) return BFB_OK;
  const unsigned nb = (unsigned)ceil_div(n * c, kThreads);
  if (reduce != 2) {
    grad_sum_kernel<T><<<nb, kThreads, 0, st>>>(static_cast<const T*>(gout), map, counts, (uint32_t)(n * c),
                                                FastDiv((uint32_t)c), reduce == 1, static_cast<T*>(gfeat));
    BFB_CHECK_LAUNCH();
    return BFB_OK;
  }
  BFB_CUDA(cudaMemsetAsync(gfeat, 0, sizeof(T) * (size_t)(n * c), st));
  if (m == 0) return BFB_OK;
  // from[] = n (no source) for every voxel channel
  BFB_CUDA(cudaMemsetAsync(from, 0x7f, sizeof(int32_t) * (size_t)(m * c), st));
  grad_argmax_kernel<T><<<nb, kThreads, 0, st>>>(static_cast<const T*>(feats), static_cast<const T*>(reduced), map,
                                                 (uint32_t)(n * c), FastDiv((uint32_t)c), from);
  BFB_CHECK_LAUNCH();
  grad_max_scatter_kernel<T><<<(unsigned)ceil_div(m * c, kThreads), kThreads, 0, st>>>(
      static_cast<const T*>(gout), from, (uint32_t)(m * c), FastDiv((uint32_t)c), n, static_cast<T*>(gfeat));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

}  // namespace
}  // namespace bfb

using namespace bfb;

extern "C" int bfb_dynamic_scatter_workspace_size(int64_t n, int64_t c, int64_t ndim, size_t* bytes) {
  if (n < 0 || c <= 0 || ndim < 1 || ndim > 4 || !bytes) return BFB_ERR_INVALID_ARG;
  if (n > 0x7ffffffeLL) return BFB_ERR_TOO_LARGE;
  ScatterWs w;
  *bytes = carve_ws(nullptr, n, &w);
  return BFB_OK;
}

extern "C" int bfb_dynamic_scatter_forward(const void* feats, int dtype, const int32_t* coors, int64_t n, int64_t c,
                                           int64_t ndim, int reduce, const int64_t* extents, void* out_feats,
                                           int32_t* out_coors, int32_t* point2voxel, int32_t* counts,
                                           int64_t* num_voxels, void* ws, size_t ws_bytes, void* stream) {
  BFB_INJECT_POINT();
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (n < 0 || c <= 0 || ndim < 1 || ndim > 4 || reduce < 0 || reduce > 2 || !num_voxels) return BFB_ERR_INVALID_ARG;
  if (n > 0x7ffffffeLL) return BFB_ERR_TOO_LARGE;
  *num_voxels = 0;
  if (n == 0) return BFB_OK;
  if (!feats || !coors || !out_feats || !out_coors || !point2voxel || !counts) return BFB_ERR_INVALID_ARG;
  ScatterWs w;
  if (!ws || carve_ws(nullptr, n, &w) > ws_bytes) return BFB_ERR_WORKSPACE;
  carve_ws(ws, n, &w);
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case BFB_F32:
      return scatter_forward_t<float>(feats, coors, n, c, ndim, reduce, extents, w, out_feats, out_coors, point2voxel,
                                      counts, num_voxels, st);
    case BFB_F16:
      return scatter_forward_t<__half>(feats, coors, n, c, ndim, reduce, extents, w, out_feats, out_coors,
                                       point2voxel, counts, num_voxels, st);
    default:
      return scatter_forward_t<__nv_bfloat16>(feats, coors, n, c, ndim, reduce, extents, w, out_feats, out_coors,
                                              point2voxel, counts, num_voxels, st);
  }
}

extern "C" int bfb_dynamic_scatter_backward(void* grad_feats, const void* grad_out, const void* feats,
                                            const void* reduced, const int32_t* point2voxel, const int32_t* counts,
                                            int dtype, int64_t n, int64_t m, int64_t c, int reduce, int32_t* argmax_ws,
                                            size_t argmax_ws_bytes, void* stream) {
  BFB_INJECT_POINT();
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (n < 0 || m < 0 || c <= 0 || reduce < 0 || reduce > 2) return BFB_ERR_INVALID_ARG;
  if (n * c > 0x7ffffffeLL || m * c > 0x7ffffffeLL) return BFB_ERR_TOO_LARGE;
  if (n > 0 && (!grad_feats || !point2voxel)) return BFB_ERR_INVALID_ARG;
  if (reduce == 2 && m > 0 && (!argmax_ws || argmax_ws_bytes < sizeof(int32_t) * (size_t)(m * c)))
    return BFB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case BFB_F32:
      return scatter_backward_t<float>(grad_feats, grad_out, feats, reduced, point2voxel, counts, n, m, c, reduce,
                                       argmax_ws, st);
    case BFB_F16:
      return scatter_backward_t<__half>(grad_feats, grad_out, feats, reduced, point2voxel, counts, n, m, c, reduce,
                                        argmax_ws, st);
    default:
      return scatter_backward_t<__nv_bfloat16>(grad_feats, grad_out, feats, reduced, point2voxel, counts, n, m, c,
                                               reduce, argmax_ws, st);
  }
}
