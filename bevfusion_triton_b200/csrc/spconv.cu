// Sparse-convolution rulebook (indice pairs) for sm_100a.
//
// Reference semantics: ops/spconv/src/spconv_triton.py
//   :655-749  _get_indice_pairs_impl (the sequential algorithm; its
//             cuda_ordering=True branch is what the Triton path returns)
//   :792-915  get_indice_pairs_triton: candidates (input j, kernel offset k)
//             in j-major order, output sites = the distinct candidate cells in
//             ascending flat order (regular / transposed conv) or the inputs
//             themselves (submanifold), rule k's pairs in ascending j
//   :90-198   candidate cell of (j, k):
//               regular:    out = (in + pad - k*dil) / stride, exact division
//               transposed: out = in*stride - pad + k*dil
//             kept when every coordinate lies in the output shape
//   :298-318  output shape (host side)
//
// Pipeline (flat cell = b * volume + row-major spatial index, < 2^32):
//   spc_candidates  thread per (j, k): the candidate's cell, valid flag in the
//                   rule-major flag array flags[k * n + j]
//   submanifold:  spc_insert_inputs (hash: cell -> largest j holding it, as
//                 the sequential loop's last write wins), spc_lookup
//                 (candidate -> output j, or dropped)
//   regular:      spc_mark (one bit per grid cell), spc_popc + scan (output
//                 ids are the ranks of the set bits, i.e. the distinct cells in
//                 ascending order), spc_rank (candidate -> output id)
//   scan of flags -> rule k's pairs at [base_k, base_k + count_k) in ascending j;
//   spc_pack writes indice_pairs[k, 0/1, slot] and spc_counts indice_num.
//   spc_outids (regular only, second call once the caller knows the count)
//   decodes the set bits into [b, c0, .., c{ndim-1}] rows.
#include <algorithm>

#include "scan.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_spconv)
namespace {

constexpr uint32_t kSpEmpty = 0xffffffffu;
constexpr int kSpMaxDims = 4;
constexpr int kSpThreads = 256;

struct SpGeom {
  int ndim;
  int64_t ks[kSpMaxDims], st[kSpMaxDims], pad[kSpMaxDims], dil[kSpMaxDims], out[kSpMaxDims];
  int64_t volume;  // product of out[]
  int64_t K;       // product of ks[]
  int64_t batch;   // rows with a batch column outside [0, batch) are ignored
  bool transpose;
  FastDiv vol_div, out_div[kSpMaxDims];  // flat cells fit 32 bits
};

struct SpSlot {
  uint32_t key;  // kSpEmpty when free
  int32_t val;
};

uint64_t sp_table_cap(int64_t inserts) {
  uint64_t cap = 1024;
  while (cap < (uint64_t)(2 * inserts)) cap *= 2;
  return cap;
}

__device__ __forceinline__ uint32_t sp_hash(uint32_t k) {
  k ^= k >> 16; k *= 0x7feb352du; k ^= k >> 15; k *= 0x846ca68bu; k ^= k >> 16;
  return k;
}

// Slot of `key`, inserting it if absent; -1 only if the table is full
// (cannot happen: the capacity is at least twice the insertions).
__device__ __forceinline__ int64_t sp_insert(SpSlot* tb, uint64_t cap, uint32_t key) {
  const uint64_t mask = cap - 1;
  uint64_t h = sp_hash(key) & mask;
  for (uint64_t probe = 0; probe < cap; ++probe) {
    uint32_t k = tb[h].key;
    if (k == kSpEmpty) k = atomicCAS(&tb[h].key, kSpEmpty, key);
    if (k == kSpEmpty || k == key) return (int64_t)h;
    h = (h + 1) & mask;
  }
  return -1;
}

__device__ __forceinline__ int64_t sp_find(const SpSlot* tb, uint64_t cap, uint32_t key) {
  const uint64_t mask = cap - 1;
  uint64_t h = sp_hash(key) & mask;
  for (uint64_t probe = 0; probe < cap; ++probe) {
    const uint32_t k = tb[h].key;
    if (k == key) return (int64_t)h;
    if (k == kSpEmpty) return -1;
    h = (h + 1) & mask;
  }
  return -1;
}

__device__ __forceinline__ uint32_t flat_of(const int32_t* row, const SpGeom& g) {
  uint64_t f = 0;
  for (int d = 0; d < g.ndim; ++d) f = f * (uint64_t)g.out[d] + (uint64_t)row[1 + d];
  return (uint32_t)((uint64_t)row[0] * (uint64_t)g.volume + f);
}

// Rule-major launches: blockIdx.y = kernel offset k, threads stride over
// the sites j; every per-candidate array is indexed k * n + j, so no thread
// divides by K or n.
__device__ __forceinline__ void kernel_offset(int k, const SpGeom& g, int (&kd)[kSpMaxDims]) {
  for (int d = g.ndim - 1; d >= 0; --d) {  // last dimension fastest
    const int ks = (int)g.ks[d];
    kd[d] = k % ks;
    k /= ks;
  }
}

// 32-bit coordinate arithmetic: coordinates, offsets and output extents are
// below 2^31 and every flat cell below 2^32 (checked on the host).
template <int NDIM>
__global__ void spc_candidates_kernel(const int32_t* __restrict__ idx, int64_t n, SpGeom g,
                                      uint32_t* __restrict__ cell, uint32_t* __restrict__ flags) {
  const int k = blockIdx.y;
  int kd[kSpMaxDims];
  kernel_offset(k, g, kd);
  int base[kSpMaxDims], st[kSpMaxDims];
  uint32_t out[kSpMaxDims];
#pragma unroll
  for (int d = 0; d < NDIM; ++d) {  // out = (in + base) / st  or  in * st + base
    base[d] = g.transpose ? (int)(kd[d] * g.dil[d] - g.pad[d]) : (int)(g.pad[d] - kd[d] * g.dil[d]);
    st[d] = (int)g.st[d];
    out[d] = (uint32_t)g.out[d];
  }
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    const int32_t* row = idx + j * (NDIM + 1);
    bool ok = (uint32_t)__ldg(row) < (uint32_t)g.batch;  // a bad batch index would address past the bitmap
    uint32_t f = 0;
#pragma unroll
    for (int d = 0; d < NDIM; ++d) {
      const int in = __ldg(row + 1 + d);
      int o;
      if (g.transpose) {
        o = in * st[d] + base[d];
      } else {
        const int num = in + base[d];
        if (st[d] == 1) {
          o = num;
        } else {
          ok = ok && num % st[d] == 0;
          o = num / st[d];
        }
      }
      ok = ok && o >= 0 && (uint32_t)o < out[d];
      f = f * out[d] + (ok ? (uint32_t)o : 0u);
    }
    const int64_t t = (int64_t)k * n + j;
    cell[t] = (uint32_t)__ldg(row) * (uint32_t)g.volume + f;
    flags[t] = ok ? 1u : 0u;
  }
}

// submanifold: cell of every input -> the largest input index holding it
__global__ void spc_insert_inputs_kernel(const int32_t* __restrict__ idx, int64_t n, SpGeom g, SpSlot* tb,
                                         uint64_t cap) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= n) return;
  const int32_t* row = idx + j * (g.ndim + 1);
  bool ok = (uint32_t)row[0] < (uint32_t)g.batch;
  for (int d = 0; d < g.ndim; ++d) ok = ok && (uint32_t)row[1 + d] < (uint32_t)g.out[d];
  if (!ok) return;  // a site outside the grid can be nobody's neighbour
  const int64_t s = sp_insert(tb, cap, flat_of(row, g));
  if (s >= 0) atomicMax(&tb[s].val, (int32_t)j);
}

// regular / transposed: one bit per grid cell that some candidate reaches
__global__ void spc_mark_kernel(const uint32_t* __restrict__ cell, const uint32_t* __restrict__ flags, int64_t c,
                                uint32_t* __restrict__ bits) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < c; t += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[t]) continue;
    const uint32_t x = cell[t];
    const uint32_t m = 1u << (x & 31);
    if (!(bits[x >> 5] & m)) atomicOr(bits + (x >> 5), m);  // skip the atomic once the bit is seen set
  }
}

__global__ void spc_popc_kernel(const uint32_t* __restrict__ bits, int64_t words, uint32_t* __restrict__ cnt) {
  const int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (w < words) cnt[w] = (uint32_t)__popc(bits[w]);
}

// regular: output id of a candidate = rank of its cell's bit
__global__ void spc_rank_kernel(const uint32_t* __restrict__ cell, const uint32_t* __restrict__ flags, int64_t c,
                                const uint32_t* __restrict__ bits, const uint32_t* __restrict__ prefix,
                                int32_t* __restrict__ out_of) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < c; t += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[t]) continue;
    const uint32_t x = cell[t], w = x >> 5;
    out_of[t] = (int32_t)(__ldg(prefix + w) + (uint32_t)__popc(__ldg(bits + w) & ((1u << (x & 31)) - 1u)));
  }
}

// submanifold: candidate -> the input at its cell, dropped when there is none
__global__ void spc_lookup_kernel(const uint32_t* __restrict__ cell, uint32_t* __restrict__ flags, int64_t c,
                                  const SpSlot* __restrict__ tb, uint64_t cap, int32_t* __restrict__ out_of) {
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < c; t += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[t]) continue;
    const int64_t s = sp_find(tb, cap, cell[t]);
    if (s < 0) {
      flags[t] = 0u;
      continue;
    }
    out_of[t] = tb[s].val;
  }
}

// pos = exclusive scan of the rule-major flags (pos[n*K] = total): rule k's
// pairs occupy [pos[k*n], pos[(k+1)*n]) in ascending j
__global__ void spc_pack_kernel(const uint32_t* __restrict__ pos, int64_t n, const int32_t* __restrict__ out_of,
                                int32_t* __restrict__ pairs) {
  const int64_t k = blockIdx.y;
  const uint32_t base = pos[k * n];
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = k * n + j;
    const uint32_t p = pos[t];
    if (pos[t + 1] == p) continue;  // flag was 0
    const int64_t slot = (int64_t)(p - base);
    if (BFB_BAD(slot < n)) continue;
    pairs[(k * 2 + 0) * n + slot] = (int32_t)j;
    pairs[(k * 2 + 1) * n + slot] = out_of[t];
  }
}

__global__ void spc_counts_kernel(const uint32_t* __restrict__ pos, int64_t n, int64_t K,
                                  int32_t* __restrict__ num) {
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  num[k] = (int32_t)(pos[(k + 1) * n] - pos[k * n]);
}

// regular: set bits -> output rows, thread per bitmap word
__global__ void spc_outids_kernel(const uint32_t* __restrict__ bits, const uint32_t* __restrict__ prefix,
                                  int64_t words, SpGeom g, int32_t* __restrict__ outids) {
  const int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= words) return;
  uint32_t m = bits[w];
  if (!m) return;
  uint32_t pos = prefix[w];
  while (m) {
    const int b = __ffs(m) - 1;
    m &= m - 1;
    const uint32_t flat = (uint32_t)w * 32u + (uint32_t)b;
    int32_t* row = outids + (int64_t)pos * (g.ndim + 1);
    const uint32_t bi = g.vol_div.div(flat);
    uint32_t f = flat - bi * g.vol_div.d;
    row[0] = (int32_t)bi;
    for (int d = g.ndim - 1; d >= 0; --d) {
      const uint32_t q = g.out_div[d].div(f);
      row[1 + d] = (int32_t)(f - q * g.out_div[d].d);
      f = q;
    }
    ++pos;
  }
}

__global__ void spc_set_count_kernel(int32_t* __restrict__ total, int32_t v) { *total = v; }

__global__ void spc_total_kernel(const uint32_t* __restrict__ prefix, int64_t words, int32_t* __restrict__ total) {
  *total = (int32_t)prefix[words];
}

struct SpWork {
  uint32_t* cell;    // [K*n] candidate cell, rule-major
  uint32_t* flags;   // [K*n + 1] rule-major flags, then their exclusive scan
  int32_t* out_of;   // [K*n] output index per candidate
  SpSlot* table;     // [cap] submanifold: cell -> input
  uint32_t* bits;    // [words] regular: reached cells
  uint32_t* prefix;  // [words + 1] regular: set bits before each word
  uint32_t* scan;
  uint64_t cap;
  int64_t words;
};

size_t carve_work(void* base, int64_t n, int64_t K, int64_t cells, bool subm, SpWork* w) {
  const int64_t c = n * K;
  Carver cv(base);
  w->cell = cv.take<uint32_t>((size_t)c);
  w->flags = cv.take<uint32_t>((size_t)c + 1);
  w->out_of = cv.take<int32_t>((size_t)c);
  w->cap = subm ? sp_table_cap(n) : 0;
  w->table = cv.take<SpSlot>((size_t)w->cap);
  w->words = subm ? 0 : ceil_div(cells, 32);
  w->bits = cv.take<uint32_t>((size_t)w->words);
  w->prefix = cv.take<uint32_t>((size_t)w->words + 1);
  const size_t sa = scan_scratch_elems(c + 1), sb = scan_scratch_elems(w->words + 1);
  w->scan = cv.take<uint32_t>(sa > sb ? sa : sb);
  return cv.bytes();
}

int make_sp_geom(int ndim, int64_t batch, const int64_t* out_shape, const int64_t* ksize, const int64_t* stride,
                 const int64_t* padding, const int64_t* dilation, int transpose, SpGeom* g) {
  if (ndim < 1 || ndim > kSpMaxDims || batch < 1) return BFB_ERR_INVALID_ARG;
  if (!out_shape || !ksize || !stride || !padding || !dilation) return BFB_ERR_INVALID_ARG;
  g->ndim = ndim;
  g->batch = batch;
  g->transpose = transpose != 0;
  g->volume = 1;
  g->K = 1;
  for (int d = 0; d < ndim; ++d) {
    if (out_shape[d] <= 0 || ksize[d] <= 0 || stride[d] <= 0 || dilation[d] <= 0) return BFB_ERR_INVALID_ARG;
    g->ks[d] = ksize[d]; g->st[d] = stride[d]; g->pad[d] = padding[d]; g->dil[d] = dilation[d];
    g->out[d] = out_shape[d];
    if (g->volume > (int64_t(1) << 40) / out_shape[d] || g->K > 4096 / ksize[d]) return BFB_ERR_TOO_LARGE;
    g->volume *= out_shape[d];
    g->K *= ksize[d];
  }
  if ((uint64_t)batch * (uint64_t)g->volume >= 0xffffffffull) return BFB_ERR_TOO_LARGE;  // cells fit 32 bits
  for (int d = 0; d < ndim; ++d) {
    const int64_t reach = (ksize[d] - 1) * dilation[d] + (padding[d] < 0 ? -padding[d] : padding[d]);
    if (reach > 0x3fffffffLL || stride[d] > 0x3fffffffLL || out_shape[d] > 0x3fffffffLL)
      return BFB_ERR_TOO_LARGE;  // 32-bit coordinate arithmetic
    g->out_div[d] = FastDiv((uint32_t)out_shape[d]);
  }
  g->vol_div = FastDiv((uint32_t)g->volume);
  return BFB_OK;
}

}  // namespace
}  // namespace bfb

using namespace bfb;

extern "C" int bfb_indice_pairs_workspace_size(int64_t n, int ndim, int64_t batch, const int64_t* out_shape,
                                               const int64_t* ksize, int subm, size_t* bytes) {
  if (n < 0 || !bytes || !ksize || !out_shape) return BFB_ERR_INVALID_ARG;
  const int64_t ones[kSpMaxDims] = {1, 1, 1, 1};
  SpGeom g;
  BFB_TRY(make_sp_geom(ndim, batch, out_shape, ksize, ones, ones, ones, 0, &g));
  if (n * g.K >= 0x7fffffffLL) return BFB_ERR_TOO_LARGE;
  SpWork w;
  *bytes = carve_work(nullptr, n, g.K, batch * g.volume, subm != 0, &w);
  return BFB_OK;
}

extern "C" int bfb_get_indice_pairs(const int32_t* indices, int64_t n, int ndim, int64_t batch,
                                    const int64_t* out_shape, const int64_t* ksize, const int64_t* stride,
                                    const int64_t* padding, const int64_t* dilation, int subm, int transpose,
                                    int32_t* indice_pairs, int32_t* indice_num, int32_t* num_out_dev,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  SpGeom g;
  BFB_TRY(make_sp_geom(ndim, batch, out_shape, ksize, stride, padding, dilation, transpose, &g));
  if (n < 0 || (n > 0 && (!indices || !indice_pairs)) || !indice_num || !num_out_dev) return BFB_ERR_INVALID_ARG;
  if (n * g.K >= 0x7fffffffLL) return BFB_ERR_TOO_LARGE;
  SpWork w;
  if (!workspace || carve_work(nullptr, n, g.K, batch * g.volume, subm != 0, &w) > workspace_bytes)
    return BFB_ERR_WORKSPACE;
  carve_work(workspace, n, g.K, batch * g.volume, subm != 0, &w);
  cudaStream_t st = as_stream(stream);
  const int64_t c = n * g.K;
  if (c > 0) BFB_CUDA(cudaMemsetAsync(indice_pairs, 0xff, sizeof(int32_t) * (size_t)(2 * c), st));  // -1
  BFB_CUDA(cudaMemsetAsync(indice_num, 0, sizeof(int32_t) * (size_t)g.K, st));
  BFB_CUDA(cudaMemsetAsync(num_out_dev, 0, sizeof(int32_t), st));
  if (n == 0) return BFB_OK;
  const unsigned nbc = (unsigned)std::min<int64_t>(ceil_div(c, kSpThreads), 148 * 32);  // grid-stride over t
  // each thread walks ~8 sites of one offset (the per-offset setup is amortised)
  const dim3 grid_kj((unsigned)std::min<int64_t>(ceil_div(n, kSpThreads * 8), 1024), (unsigned)g.K);
  switch (ndim) {
    case 1: spc_candidates_kernel<1><<<grid_kj, kSpThreads, 0, st>>>(indices, n, g, w.cell, w.flags); break;
    case 2: spc_candidates_kernel<2><<<grid_kj, kSpThreads, 0, st>>>(indices, n, g, w.cell, w.flags); break;
    case 3: spc_candidates_kernel<3><<<grid_kj, kSpThreads, 0, st>>>(indices, n, g, w.cell, w.flags); break;
    default: spc_candidates_kernel<4><<<grid_kj, kSpThreads, 0, st>>>(indices, n, g, w.cell, w.flags); break;
  }
  BFB_CHECK_LAUNCH();
  if (subm) {
    BFB_CUDA(cudaMemsetAsync(w.table, 0xff, sizeof(SpSlot) * (size_t)w.cap, st));  // key free, val -1
    spc_insert_inputs_kernel<<<(unsigned)ceil_div(n, kSpThreads), kSpThreads, 0, st>>>(indices, n, g, w.table,
                                                                                      w.cap);
    BFB_CHECK_LAUNCH();
    spc_lookup_kernel<<<nbc, kSpThreads, 0, st>>>(w.cell, w.flags, c, w.table, w.cap, w.out_of);
    BFB_CHECK_LAUNCH();
    spc_set_count_kernel<<<1, 1, 0, st>>>(num_out_dev, (int32_t)n);
    BFB_CHECK_LAUNCH();
  } else {
    BFB_CUDA(cudaMemsetAsync(w.bits, 0, sizeof(uint32_t) * (size_t)w.words, st));
    spc_mark_kernel<<<nbc, kSpThreads, 0, st>>>(w.cell, w.flags, c, w.bits);
    BFB_CHECK_LAUNCH();
    spc_popc_kernel<<<(unsigned)ceil_div(w.words, kSpThreads), kSpThreads, 0, st>>>(w.bits, w.words, w.prefix);
    BFB_CHECK_LAUNCH();
    BFB_TRY(exclusive_scan_u32(w.prefix, w.prefix, w.words, w.scan, w.prefix + w.words, st));
    spc_rank_kernel<<<nbc, kSpThreads, 0, st>>>(w.cell, w.flags, c, w.bits, w.prefix, w.out_of);
    BFB_CHECK_LAUNCH();
    spc_total_kernel<<<1, 1, 0, st>>>(w.prefix, w.words, num_out_dev);
    BFB_CHECK_LAUNCH();
  }
  BFB_TRY(exclusive_scan_u32(w.flags, w.flags, c, w.scan, w.flags + c, st));
  spc_pack_kernel<<<grid_kj, kSpThreads, 0, st>>>(w.flags, n, w.out_of, indice_pairs);
  BFB_CHECK_LAUNCH();
  spc_counts_kernel<<<(unsigned)ceil_div(g.K, kSpThreads), kSpThreads, 0, st>>>(w.flags, n, g.K, indice_num);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

extern "C" int bfb_indice_pairs_outids(int64_t n, int ndim, int64_t batch, const int64_t* out_shape,
                                       const int64_t* ksize, const void* workspace, size_t workspace_bytes,
                                       int32_t* outids, void* stream) {
  const int64_t ones[kSpMaxDims] = {1, 1, 1, 1};
  SpGeom g;
  BFB_TRY(make_sp_geom(ndim, batch, out_shape, ksize, ones, ones, ones, 0, &g));
  SpWork w;
  if (!workspace || carve_work(nullptr, n, g.K, batch * g.volume, false, &w) > workspace_bytes)
    return BFB_ERR_WORKSPACE;
  if (n == 0) return BFB_OK;
  if (!outids) return BFB_ERR_INVALID_ARG;
  carve_work(const_cast<void*>(workspace), n, g.K, batch * g.volume, false, &w);
  spc_outids_kernel<<<(unsigned)ceil_div(w.words, kSpThreads), kSpThreads, 0, as_stream(stream)>>>(
      w.bits, w.prefix, w.words, g, outids);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}
