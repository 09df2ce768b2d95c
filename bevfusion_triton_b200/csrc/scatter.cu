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
// Design: each valid row gets a packed lexicographic key (bit widths from the
// per-dimension maxima), the stable radix sort groups equal rows with points in
// ascending index order, segment heads are scanned into voxel ids, and a warp
// per voxel reduces its points in that order in fp32 (sums therefore follow
// torch.index_add_'s order exactly).
#include <algorithm>
#include <cmath>

#include "radix.cuh"
#include "scan.cuh"

namespace bfb {
namespace {

constexpr int kThreads = 256;

struct ScatterWs {
  int32_t* dmax;    // [8]   per-dimension maxima, then status
  uint32_t* keys0;  // [n]
  uint32_t* keys1;  // [n]
  uint32_t* vtmp;   // [n]
  uint32_t* perm;   // [n]
  uint32_t* head;   // [n+1] segment-head flags, then voxel id of each sorted position
  uint32_t* seg;    // [n+1] sorted start of every voxel
  uint32_t* hist;
  uint32_t* scan;
};

size_t carve_ws(void* base, int64_t n, ScatterWs* w) {
  RadixPlan rp;
  rp.max_digit_bits = kRadixMaxBits;  // upper bound over every key width
  Carver c(base);
  w->dmax = c.take<int32_t>(8);
  w->keys0 = c.take<uint32_t>((size_t)n);
  w->keys1 = c.take<uint32_t>((size_t)n);
  w->vtmp = c.take<uint32_t>((size_t)n);
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
  int shift[4];
  uint32_t invalid;  // key of rows with a negative coordinate (sorts last)
};

__global__ void row_keys_kernel(const int32_t* __restrict__ coors, int64_t n, KeySpec ks, uint32_t* __restrict__ keys) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t k = 0;
  bool ok = true;
  for (int d = 0; d < ks.ndim; ++d) {
    const int32_t v = coors[i * ks.ndim + d];
    ok &= v >= 0;
    k |= (uint32_t)v << ks.shift[d];
  }
  keys[i] = ok ? k : ks.invalid;
}

__global__ void seg_head_kernel(const uint32_t* __restrict__ keys, int64_t n, uint32_t invalid, uint32_t* __restrict__ head) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t k = keys[i];
  head[i] = (k != invalid && (i == 0 || keys[i - 1] != k)) ? 1u : 0u;
}

// head (scanned) -> voxel id per sorted position; map, unique coords, segment starts
__global__ void seg_assign_kernel(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ perm, int64_t n,
                                  uint32_t invalid, const uint32_t* __restrict__ vid, const int32_t* __restrict__ coors,
                                  int ndim, int32_t* __restrict__ map, int32_t* __restrict__ out_coors,
                                  uint32_t* __restrict__ seg) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t k = keys[i];
  const uint32_t p = perm[i];
  if (k == invalid) {
    map[p] = -1;
    if (i == 0 || keys[i - 1] != invalid) seg[vid[n]] = (uint32_t)i;  // end of the last voxel
    return;
  }
  const uint32_t m = vid[i + 1] - 1;  // inclusive count of heads up to i, minus one
  map[p] = (int32_t)m;
  if (i == 0 || keys[i - 1] != k) {
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

// reduce: 0 sum, 1 mean, 2 max.  Warp per voxel, lanes over channels.
template <class T>
__global__ void seg_reduce_kernel(const T* __restrict__ feats, int64_t c, const uint32_t* __restrict__ perm,
                                  const uint32_t* __restrict__ seg, const uint32_t* __restrict__ total, int reduce,
                                  T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t m_total = *total;
  for (int64_t m = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < m_total; m += warps) {
    const uint32_t a = seg[m], b = seg[m + 1];
    for (int64_t ch = lane; ch < c; ch += 32) {
      float acc = reduce == 2 ? -INFINITY : 0.f;
      for (uint32_t i = a; i < b; ++i) {
        const float v = to_f32<T>(feats[(int64_t)perm[i] * c + ch]);
        acc = reduce == 2 ? fmaxf(acc, v) : acc + v;
      }
      if (reduce == 1) acc = acc / (float)(b - a);
      out[m * c + ch] = from_f32<T>(acc);
    }
  }
}

template <class T>
__global__ void grad_sum_kernel(const T* __restrict__ gout, const int32_t* __restrict__ map,
                                const int32_t* __restrict__ counts, int64_t n, int64_t c, int mean,
                                T* __restrict__ gfeat) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * c) return;
  const int64_t i = idx / c, ch = idx - i * c;
  const int32_t m = map[i];
  if (m < 0) {
    gfeat[idx] = from_f32<T>(0.f);
    return;
  }
  float g = to_f32<T>(gout[(int64_t)m * c + ch]);
  if (mean) g = g / (float)counts[m];
  gfeat[idx] = from_f32<T>(g);
}

template <class T>
__global__ void grad_argmax_kernel(const T* __restrict__ feats, const T* __restrict__ reduced,
                                   const int32_t* __restrict__ map, int64_t n, int64_t c, int32_t* __restrict__ from) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n * c) return;
  const int64_t i = idx / c, ch = idx - i * c;
  const int32_t m = map[i];
  if (m < 0) return;
  if (to_f32<T>(feats[idx]) == to_f32<T>(reduced[(int64_t)m * c + ch])) atomicMin(&from[(int64_t)m * c + ch], (int32_t)i);
}

template <class T>
__global__ void grad_max_scatter_kernel(const T* __restrict__ gout, const int32_t* __restrict__ from, int64_t m_total,
                                        int64_t c, int64_t n, T* __restrict__ gfeat) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= m_total * c) return;
  const int32_t src = from[idx];
  const int64_t ch = idx % c;
  if (src < n) gfeat[(int64_t)src * c + ch] = gout[idx];
}

template <class T>
int scatter_forward_t(const void* feats, const int32_t* coors, int64_t n, int64_t c, int64_t ndim, int reduce,
                      const ScatterWs& w, void* out_feats, int32_t* out_coors, int32_t* map, int32_t* counts,
                      int64_t* m_out, cudaStream_t st) {
  BFB_CUDA(cudaMemsetAsync(w.dmax, 0xff, 8 * sizeof(int32_t), st));
  dim_max_kernel<<<(unsigned)std::min<int64_t>(ceil_div(n, kThreads), 1184), kThreads, 0, st>>>(coors, n, (int)ndim, w.dmax);
  BFB_CHECK_LAUNCH();
  int32_t dmax[4] = {-1, -1, -1, -1};
  BFB_CUDA(cudaMemcpyAsync(dmax, w.dmax, sizeof(int32_t) * ndim, cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  KeySpec ks;
  ks.ndim = (int)ndim;
  int bits = 0;
  for (int d = (int)ndim - 1; d >= 0; --d) {
    int b = 0;
    while (b < 31 && ((int64_t)1 << b) <= (int64_t)dmax[d]) ++b;
    ks.shift[d] = bits;
    bits += b;
  }
  if (bits > 31) return BFB_ERR_TOO_LARGE;
  ks.invalid = bits == 0 ? 1u : (1u << bits);  // above every valid key
  const unsigned nb = (unsigned)ceil_div(n, kThreads);
  row_keys_kernel<<<nb, kThreads, 0, st>>>(coors, n, ks, w.keys0);
  BFB_CHECK_LAUNCH();
  const RadixPlan rp = make_radix_plan(ks.invalid);
  uint32_t* sorted = nullptr;
  BFB_TRY(radix_sort_index(w.keys0, w.keys1, w.vtmp, w.perm, n, rp, w.hist, w.scan, false, st, &sorted));
  seg_head_kernel<<<nb, kThreads, 0, st>>>(sorted, n, ks.invalid, w.head);
  BFB_CHECK_LAUNCH();
  // inclusive voxel ids: vid[i + 1] = heads in [0, i]; vid[n] = M
  BFB_CUDA(cudaMemsetAsync(w.head + n, 0, sizeof(uint32_t), st));
  BFB_TRY(exclusive_scan_u32(w.head, w.head, n + 1, w.scan, nullptr, st));
  seg_assign_kernel<<<nb, kThreads, 0, st>>>(sorted, w.perm, n, ks.invalid, w.head, coors, (int)ndim, map, out_coors,
                                             w.seg);
  BFB_CHECK_LAUNCH();
  uint32_t m = 0;
  BFB_CUDA(cudaMemcpyAsync(&m, w.head + n, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  *m_out = m;
  if (m == 0) return BFB_OK;
  seg_count_kernel<<<(unsigned)ceil_div(m, kThreads), kThreads, 0, st>>>(w.seg, w.head + n, counts);
  BFB_CHECK_LAUNCH();
  seg_reduce_kernel<T><<<(unsigned)std::min<int64_t>(ceil_div((int64_t)m * 32, kThreads), 148 * 16), kThreads, 0, st>>>(
      static_cast<const T*>(feats), c, w.perm, w.seg, w.head + n, reduce, static_cast<T*>(out_feats));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

template <class T>
int scatter_backward_t(void* gfeat, const void* gout, const void* feats, const void* reduced, const int32_t* map,
                       const int32_t* counts, int64_t n, int64_t m, int64_t c, int reduce, int32_t* from,
                       cudaStream_t st) {
  if (n == 0) return BFB_OK;
  const unsigned nb = (unsigned)ceil_div(n * c, kThreads);
  if (reduce != 2) {
    grad_sum_kernel<T><<<nb, kThreads, 0, st>>>(static_cast<const T*>(gout), map, counts, n, c, reduce == 1,
                                                static_cast<T*>(gfeat));
    BFB_CHECK_LAUNCH();
    return BFB_OK;
  }
  BFB_CUDA(cudaMemsetAsync(gfeat, 0, sizeof(T) * (size_t)(n * c), st));
  if (m == 0) return BFB_OK;
  // from[] = n (no source) for every voxel channel
  BFB_CUDA(cudaMemsetAsync(from, 0x7f, sizeof(int32_t) * (size_t)(m * c), st));
  grad_argmax_kernel<T><<<nb, kThreads, 0, st>>>(static_cast<const T*>(feats), static_cast<const T*>(reduced), map, n,
                                                 c, from);
  BFB_CHECK_LAUNCH();
  grad_max_scatter_kernel<T><<<(unsigned)ceil_div(m * c, kThreads), kThreads, 0, st>>>(
      static_cast<const T*>(gout), from, m, c, n, static_cast<T*>(gfeat));
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
                                           int64_t ndim, int reduce, void* out_feats, int32_t* out_coors,
                                           int32_t* point2voxel, int32_t* counts, int64_t* num_voxels, void* ws,
                                           size_t ws_bytes, void* stream) {
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
      return scatter_forward_t<float>(feats, coors, n, c, ndim, reduce, w, out_feats, out_coors, point2voxel, counts,
                                      num_voxels, st);
    case BFB_F16:
      return scatter_forward_t<__half>(feats, coors, n, c, ndim, reduce, w, out_feats, out_coors, point2voxel, counts,
                                       num_voxels, st);
    default:
      return scatter_forward_t<__nv_bfloat16>(feats, coors, n, c, ndim, reduce, w, out_feats, out_coors, point2voxel,
                                              counts, num_voxels, st);
  }
}

extern "C" int bfb_dynamic_scatter_backward(void* grad_feats, const void* grad_out, const void* feats,
                                            const void* reduced, const int32_t* point2voxel, const int32_t* counts,
                                            int dtype, int64_t n, int64_t m, int64_t c, int reduce, int32_t* argmax_ws,
                                            size_t argmax_ws_bytes, void* stream) {
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
