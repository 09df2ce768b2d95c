// Hard and dynamic voxelisation for sm_100a.
//
// Reference semantics (the sequential CPU algorithm is the authority):
//   ops/voxel/src/voxelization_triton.py:23-39   grid size, argument checks
//   ops/voxel/src/voxelization_triton.py:328-349 cell = floor((p - min) / size) in fp32,
//                                                 (-1, -1, -1) when out of range
//   ops/voxel/src/voxelization_triton.py:466-513 voxel ids in first-occurrence order,
//                                                 at most max_voxels voxels, each keeps
//                                                 its first max_points points in input
//                                                 order, buffers zero-filled
//
// Fast pipeline (max_points <= kFastMaxP), five launches for a whole batch:
//   vox_fast_insert   cell + 64-bit key (sample, cell) per point; warp-aggregated insert
//                     into the open-addressing table (first point by atomicMin); the
//                     thread that creates a slot takes a dense voxel number d from a
//                     counter and empties row d of the member table
//   vox_fast_members  per point: d and the "first point" flag; the point index goes into
//                     row d of the member table, which keeps the P smallest indices of
//                     the voxel in ascending order (an atomicMin insertion chain: each
//                     slot keeps the smaller of what it holds and what arrives and passes
//                     the larger on, so slot j ends with the (j+1)-th smallest index
//                     whatever the arrival order); per-tile flag counts, per-sample
//                     voxel counts
//   vox_fast_scan     one CTA: exclusive scans of the tile counts and the sample counts,
//                     voxel_num
//   vox_fast_assign   per tile: the exclusive scan of the flags numbers every voxel by
//                     its first point, which writes the voxel's coords and count, notes
//                     its output row and frees its table slot
//   vox_fast_copy     a thread per output element of the kept voxels: the P rows
//                     gathered through the member table, zero padding, written in order
// General pipeline (any max_points, including -1), one launch per stage:
//   vox_insert   cell + 64-bit key (sample, cell) per point; warp-aggregated insert into
//                an open-addressing table that records the voxel's first point
//                (atomicMin) and its point count
//   vox_flags    flag = the point is its voxel's first point; exclusive scan over the
//                flags numbers voxels in first-occurrence order (per sample by offset)
//   vox_assign   per first point: keep / drop against max_voxels, write coors and
//                num_points, record the voxel's table slot and member count
//   vox_fill     bucket every kept point by voxel (slots from a scan of the counts)
//   vox_rank     a thread per kept point: its slot = number of smaller point indices in
//                its voxel's bucket (input order); slots below max_points get its row;
//                rank 0 frees the table slot
//   vox_pad      a thread per (voxel, slot): zero the slots past the voxel's points
//   vox_order    a lane per voxel: voxels above 4096 points are ordered and written by
//                a whole warp (repeated minimum); dropped voxels free their slot in
//                vox_assign
// The table therefore stays clean between calls: it is initialised once
// (bfb_hard_voxelize_table_init) and every successful call leaves it clean.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "scan.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_vox)
namespace {

constexpr uint64_t kEmptyKey = ~0ull;
constexpr uint32_t kNoFirst = 0xffffffffu;
constexpr int kLinBits = 40;  // cell index bits inside a key; the rest hold the sample
constexpr int kVoxThreads = 256;

// One voxel per slot, one 32-byte sector per slot: a probe, the first-point
// minimum, the count and the id of a voxel all touch the same sector.
struct __align__(32) VoxSlot {
  unsigned long long key;  // kEmptyKey when free
  uint32_t first;          // smallest point index (kNoFirst when free)
  uint32_t cnt;            // points
  int32_t gvid;            // voxel id over the batch, -1 when dropped by max_voxels
  uint32_t pad[3];
};
static_assert(sizeof(VoxSlot) == 32, "one sector per slot");

struct TableView {
  VoxSlot* slots;
  uint64_t cap;  // power of two
};

size_t carve_table(void* base, uint64_t cap, TableView* t) {
  Carver c(base);
  t->slots = c.take<VoxSlot>(cap);
  t->cap = cap;
  return c.bytes();
}

uint64_t table_cap_for_bytes(size_t bytes) {
  uint64_t cap = 1;
  TableView t;
  while (carve_table(nullptr, cap * 2, &t) <= bytes) cap *= 2;
  return carve_table(nullptr, cap, &t) <= bytes ? cap : 0;
}

uint64_t table_cap_for_points(int64_t n) {
  uint64_t cap = 1024;
  while (cap < (uint64_t)(2 * n)) cap *= 2;
  return cap;
}

struct VoxScratch {
  int64_t* offs;     // [batch + 1]
  int32_t* slot_of;  // [n]   table slot per point, -1 when out of range
  uint32_t* excl;    // [n+1] first-point flags, then their exclusive scan
  uint32_t* gcnt;    // [n+1] members per voxel (0 when dropped)
  uint32_t* cursor;  // [n+1] bucket offsets (scan of gcnt), advanced to bucket ends by vox_fill
  int32_t* gslot;    // [n]   table slot per voxel
  int2* vinfo;       // [n]   (sample, voxel id within the sample)
  uint32_t* members; // [n]   point index per bucket slot
  int32_t* mvox;     // [n]   voxel id per bucket slot
  uint32_t* scan;
  uint32_t* err;     // [4]   0: table full (insert gave up)
};

size_t carve_scratch(void* base, int64_t n, int64_t batch, VoxScratch* v) {
  Carver c(base);
  v->offs = c.take<int64_t>((size_t)batch + 1);
  v->slot_of = c.take<int32_t>((size_t)n);
  v->excl = c.take<uint32_t>((size_t)n + 1);
  v->gcnt = c.take<uint32_t>((size_t)n + 1);
  v->cursor = c.take<uint32_t>((size_t)n + 1);
  v->gslot = c.take<int32_t>((size_t)n);
  v->vinfo = c.take<int2>((size_t)n);
  v->members = c.take<uint32_t>((size_t)n);
  v->mvox = c.take<int32_t>((size_t)n);
  v->scan = c.take<uint32_t>(scan_scratch_elems(n + 1));
  v->err = c.take<uint32_t>(4);
  return c.bytes();
}

constexpr int kFastMaxP = 64;              // the member table holds up to 64 indices per voxel
constexpr uint32_t kEmptyMember = 0xffffffffu;
constexpr int kFastThreads = 256;          // one point per thread; a tile is one CTA's points

// Member-table row stride (uint32): P rounded up to whole 16-byte vectors.
inline int64_t member_stride(int64_t P) { return (P + 3) / 4 * 4; }

struct FastScratch {
  uint32_t* hdr;           // [16] zeroed per call: 0 dense-voxel counter, 1 table full
  int64_t* offs;           // [batch + 1] sample offsets, then
  int64_t* tpre;           // [batch + 1] first tile of every sample (tpre[batch] = tiles): one upload
  uint32_t* bsum;          // [tiles + 1] first points per tile, then their exclusive scan
  int32_t* did;            // [n] table slot of every point, -1 out of range
  int32_t* sd;             // [n] table slot of dense voxel d
  int4* rec;               // [n] (tile, rank among the tile's first points, points) of dense voxel d
  uint32_t* fill;          // [n] member slots claimed in a voxel of at most P points
  uint32_t* mem;           // [n * member_stride(P)] member table
};

// Tiles of the fast pipeline: every sample cut into runs of kFastThreads
// points, so at most one partial tile per sample.
int64_t fast_tiles_bound(int64_t n, int64_t batch) { return n / kFastThreads + batch; }

size_t carve_fast(void* base, int64_t n, int64_t batch, int64_t P, FastScratch* v) {
  const int64_t tiles = fast_tiles_bound(n, batch);
  Carver c(base);
  v->hdr = c.take<uint32_t>(16);
  v->offs = c.take<int64_t>(2 * ((size_t)batch + 1));
  v->tpre = v->offs ? v->offs + batch + 1 : nullptr;
  v->bsum = c.take<uint32_t>((size_t)tiles + 1);
  v->did = c.take<int32_t>((size_t)n);
  v->sd = c.take<int32_t>((size_t)n);
  v->rec = c.take<int4>((size_t)n);
  v->fill = c.take<uint32_t>((size_t)n);
  v->mem = c.take<uint32_t>((size_t)n * (size_t)member_stride(P));
  return c.bytes();
}

bool fast_path(int64_t max_points, int64_t batch) {
  (void)batch;
  return max_points > 0 && max_points <= kFastMaxP;
}

struct Grid {
  float vs[3];
  float mn[3];
  int64_t g[3];
};

int make_grid(const float* vsize, const float* range, Grid* gr) {
  if (!vsize || !range) return BFB_ERR_INVALID_ARG;
  for (int i = 0; i < 3; ++i) {
    gr->vs[i] = vsize[i];
    gr->mn[i] = range[i];
    const double v = ((double)range[3 + i] - (double)range[i]) / (double)vsize[i];
    if (!(v == v) || v > 1e15 || v < -1e15) return BFB_ERR_INVALID_ARG;
    gr->g[i] = (int64_t)std::nearbyint(v);  // Python round(): half to even
  }
  return BFB_OK;
}

// floor((p - min) / size) in IEEE fp32 (no contraction); false when outside.
__device__ __forceinline__ bool cell_of(const float p[3], const Grid& gr, int32_t c[3]) {
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float f = floorf(__fdiv_rn(__fsub_rn(p[j], gr.mn[j]), gr.vs[j]));
    if (!(f >= 0.f) || !(f < (float)gr.g[j])) return false;
    c[j] = (int32_t)f;
  }
  return true;
}

template <class T>
__device__ __forceinline__ void load_xyz(const T* pts, int64_t p, int64_t f, float out[3]) {
  const T* r = pts + p * f;
  out[0] = to_f32<T>(r[0]);
  out[1] = to_f32<T>(r[1]);
  out[2] = to_f32<T>(r[2]);
}

__device__ __forceinline__ uint64_t mix64(uint64_t k) {
  k ^= k >> 33; k *= 0xff51afd7ed558ccdull; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ull; k ^= k >> 33;
  return k;
}

// Sample of point p: offs is ascending with offs[0] = 0, offs[batch] = n.
__device__ __forceinline__ int sample_of(const int64_t* offs, int batch, int64_t p) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offs + mid) <= p) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Host -> device upload of the small per-call tables (sample offsets, tile
// prefix) through kernel parameters: no pageable cudaMemcpyAsync, which may
// wait for the stream before it returns and so stalls the launching thread
// behind earlier work on the stream (and is not capturable into a graph).
// The first launch also zeroes `nzero` words at `zero` (the call's
// counters), which saves a memset.
template <int W>
struct UploadChunk {
  int64_t v[W];
};

template <int W>
__global__ void upload_words_kernel(const UploadChunk<W> c, int64_t* __restrict__ dst, int count,
                                    uint32_t* __restrict__ zero, int nzero) {
  for (int i = threadIdx.x; i < count; i += blockDim.x) dst[i] = c.v[i];
  for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0u;
}

// W = 128 (1 KB of parameters) covers batches up to 63; larger tables go
// in chunks of 2048 words (16 KB of the 32 KB parameter space).
template <int W>
int upload_chunks(int64_t* dst, const int64_t* src, size_t count, uint32_t* zero, int nzero, cudaStream_t st) {
  UploadChunk<W> c;
  size_t base = 0;
  do {
    const int m = (int)std::min<size_t>(W, count - base);
    std::memcpy(c.v, src + base, sizeof(int64_t) * (size_t)m);
    upload_words_kernel<W><<<1, 256, 0, st>>>(c, dst + base, m, base == 0 ? zero : nullptr, base == 0 ? nzero : 0);
    BFB_CHECK_LAUNCH();
    base += (size_t)m;
  } while (base < count);
  return BFB_OK;
}

int upload_words(int64_t* dst, const int64_t* src, size_t count, uint32_t* zero, int nzero, cudaStream_t st) {
  return count <= 128 ? upload_chunks<128>(dst, src, count, zero, nzero, st)
                      : upload_chunks<2048>(dst, src, count, zero, nzero, st);
}

// ---------------------------------------------------------------------------
// dynamic voxelisation
// ---------------------------------------------------------------------------
template <class T>
__global__ void dyn_voxelize_kernel(const T* __restrict__ pts, int64_t n, int64_t f, Grid gr,
                                    int32_t* __restrict__ coors) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  float xyz[3];
  load_xyz<T>(pts, p, f, xyz);
  int32_t c[3];
  if (!cell_of(xyz, gr, c)) c[0] = c[1] = c[2] = -1;
  coors[3 * p + 0] = c[0];
  coors[3 * p + 1] = c[1];
  coors[3 * p + 2] = c[2];
}

// ---------------------------------------------------------------------------
// hard voxelisation stages
// ---------------------------------------------------------------------------
template <class T>
__global__ __launch_bounds__(kVoxThreads) void vox_insert_kernel(const T* __restrict__ pts, int64_t n, int64_t f,
                                                                 Grid gr, const int64_t* __restrict__ offs, int batch,
                                                                 TableView tb, int32_t* __restrict__ slot_of,
                                                                 uint32_t* err) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  bool valid = false;
  uint64_t key = kEmptyKey;
  if (p < n) {
    float xyz[3];
    load_xyz<T>(pts, p, f, xyz);
    int32_t c[3];
    if (cell_of(xyz, gr, c)) {
      valid = true;
      const uint64_t lin = ((uint64_t)c[0] * (uint64_t)gr.g[1] + (uint64_t)c[1]) * (uint64_t)gr.g[2] + (uint64_t)c[2];
      const uint64_t s = batch > 1 ? (uint64_t)sample_of(offs, batch, p) : 0ull;
      key = (s << kLinBits) | lin;
    }
  }
  // a run of neighbouring lanes on the same voxel (points in scan order)
  // inserts once; its first lane holds the run's smallest point index.  The
  // same voxel in two runs inserts twice, which the atomics make harmless.
  const uint64_t prev = __shfl_up_sync(0xffffffffu, key, 1);
  const unsigned heads = __ballot_sync(0xffffffffu, lane == 0 || prev != key);
  const int leader = 31 - __clz(heads & (lanemask_lt() | (1u << lane)));
  const unsigned later = lane < 31 ? heads >> (lane + 1) : 0u;
  const uint32_t run = later ? (uint32_t)__ffs(later) : (uint32_t)(32 - lane);
  int64_t slot = -1;
  if (valid && lane == leader) {
    const uint64_t mask = tb.cap - 1;
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe < tb.cap; ++probe) {
      uint64_t k = tb.slots[h].key;
      if (k == kEmptyKey) k = atomicCAS(&tb.slots[h].key, kEmptyKey, (unsigned long long)key);
      if (k == kEmptyKey || k == key) {
        slot = (int64_t)h;
        break;
      }
      h = (h + 1) & mask;
    }
    if (slot >= 0) {
      atomicMin(&tb.slots[slot].first, (uint32_t)p);
      atomicAdd(&tb.slots[slot].cnt, run);
    } else {
      atomicAdd(err, 1u);  // table full: cannot happen when cap >= n
    }
  }
  slot = __shfl_sync(0xffffffffu, slot, leader);
  if (p < n) slot_of[p] = valid ? (int32_t)slot : -1;
}

__global__ void vox_flags_kernel(const int32_t* __restrict__ slot_of, int64_t n, const VoxSlot* __restrict__ slots,
                                 uint32_t* __restrict__ flags) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const int32_t s = slot_of[p];
  flags[p] = (s >= 0 && slots[s].first == (uint32_t)p) ? 1u : 0u;
}

template <class T>
__global__ void vox_assign_kernel(const T* __restrict__ pts, int64_t n, int64_t f, Grid gr,
                                  const int64_t* __restrict__ offs, int batch, TableView tb,
                                  const int32_t* __restrict__ slot_of, const uint32_t* __restrict__ excl,
                                  int64_t max_points, int64_t max_voxels, int32_t* __restrict__ coors,
                                  int32_t* __restrict__ num_points, uint32_t* __restrict__ gcnt,
                                  int32_t* __restrict__ gslot, int2* __restrict__ vinfo) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const int32_t slot = slot_of[p];
  if (slot < 0 || tb.slots[slot].first != (uint32_t)p) return;
  const uint32_t g = excl[p];
  const int s = batch > 1 ? sample_of(offs, batch, p) : 0;
  const int64_t local = (int64_t)g - (int64_t)excl[offs[s]];
  const uint32_t c = tb.slots[slot].cnt;
  const bool kept = max_voxels < 0 || local < max_voxels;
  gslot[g] = slot;
  gcnt[g] = kept ? c : 0u;
  vinfo[g] = make_int2(s, (int)local);
  tb.slots[slot].gvid = kept ? (int32_t)g : -1;
  if (!kept) {  // dropped by max_voxels: no later kernel visits this slot, free it now
    tb.slots[slot].key = kEmptyKey;  // (gvid stays -1 for vox_fill)
    tb.slots[slot].first = kNoFirst;
    tb.slots[slot].cnt = 0u;
  }
  if (kept) {
    float xyz[3];
    load_xyz<T>(pts, p, f, xyz);
    int32_t cc[3];
    cell_of(xyz, gr, cc);
    const int64_t row = (int64_t)s * max_voxels + local;
    coors[3 * row + 0] = cc[0];
    coors[3 * row + 1] = cc[1];
    coors[3 * row + 2] = cc[2];
    num_points[row] = (int32_t)(max_points < 0 ? c : min((int64_t)c, max_points));
  }
}

__global__ void vox_count_kernel(const int64_t* __restrict__ offs, int batch, const uint32_t* __restrict__ excl,
                                 int64_t max_voxels, int32_t* __restrict__ voxel_num) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= batch) return;
  const int64_t tot = (int64_t)excl[offs[s + 1]] - (int64_t)excl[offs[s]];
  voxel_num[s] = (int32_t)(max_voxels < 0 ? tot : min(tot, max_voxels));
}

__global__ __launch_bounds__(kVoxThreads) void vox_fill_kernel(const int32_t* __restrict__ slot_of, int64_t n,
                                                               const VoxSlot* __restrict__ slots,
                                                               uint32_t* __restrict__ cursor,
                                                               uint32_t* __restrict__ members,
                                                               int32_t* __restrict__ mvox) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  int32_t g = -1;
  if (p < n) {
    const int32_t s = slot_of[p];
    if (s >= 0) g = slots[s].gvid;
  }
  // one cursor advance per run of neighbouring lanes in the same voxel (the
  // order inside a bucket does not matter: vox_rank orders by point index)
  const int32_t prev = __shfl_up_sync(0xffffffffu, g, 1);
  const unsigned heads = __ballot_sync(0xffffffffu, lane == 0 || prev != g);
  const int leader = 31 - __clz(heads & (lanemask_lt() | (1u << lane)));
  const unsigned later = lane < 31 ? heads >> (lane + 1) : 0u;
  const uint32_t run = later ? (uint32_t)__ffs(later) : (uint32_t)(32 - lane);
  uint32_t base = 0;
  if (g >= 0 && lane == leader) base = atomicAdd(cursor + g, run);
  base = __shfl_sync(0xffffffffu, base, leader);
  if (g >= 0) {
    const uint32_t pos = base + (uint32_t)(lane - leader);
    members[pos] = (uint32_t)p;
    mvox[pos] = g;
  }
}

constexpr int kRankMax = 4096;  // voxels with more points are ordered by a whole warp

// One thread per kept point (bucket slot): its slot within the voxel is the
// number of smaller point indices in the voxel's bucket, i.e. its rank in
// input order; points ranked below P copy their features into that slot.
// The voxel's first point (rank 0) also frees its table slot.
template <class T>
__global__ __launch_bounds__(kVoxThreads) void vox_rank_kernel(
    const T* __restrict__ pts, int64_t f, const uint32_t* __restrict__ total_dev, const uint32_t* __restrict__ gcnt,
    const uint32_t* __restrict__ cursor, const int2* __restrict__ vinfo, const uint32_t* __restrict__ members,
    const int32_t* __restrict__ mvox, const int32_t* __restrict__ gslot, TableView tb, int64_t P,
    int64_t max_voxels, T* __restrict__ voxels) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  // kept points over the batch: the bucket offset one past the last voxel
  // (vox_fill advances only the offsets of voxels that own points)
  if (i >= (int64_t)cursor[*total_dev]) return;
  const int32_t g = mvox[i];
  const uint32_t cnt = gcnt[g];
  if (cnt > (uint32_t)kRankMax) return;
  const uint32_t end = cursor[g], start = end - cnt;
  const uint32_t p = members[i];
  uint32_t r = 0;
  for (uint32_t j = start; j < end; ++j) r += __ldg(members + j) < p;
  if (r == 0) {  // leave the table clean for the next call
    VoxSlot& sl = tb.slots[gslot[g]];
    sl.key = kEmptyKey;
    sl.first = kNoFirst;
    sl.cnt = 0u;
  }
  if ((int64_t)r >= P) return;
  const int2 vi = vinfo[g];
  T* dst = voxels + (((int64_t)vi.x * max_voxels + vi.y) * P + r) * f;
  const T* src = pts + (int64_t)p * f;
  for (int64_t q = 0; q < f; ++q) dst[q] = src[q];
}

// One thread per (voxel, point slot): slots past a voxel's points get 0.
// 32-bit index arithmetic while the slots fit (always, at the configured
// sizes), 64-bit division otherwise.
template <class T>
__device__ __forceinline__ void pad_slot(uint64_t g, uint64_t j, const uint32_t* __restrict__ gcnt,
                                         const int2* __restrict__ vinfo, int64_t f, int64_t P, int64_t max_voxels,
                                         T* __restrict__ voxels) {
  const uint32_t cnt = __ldg(gcnt + g);
  if (cnt == 0 || cnt > (uint32_t)kRankMax || j < cnt) return;
  const int2 vi = __ldg(vinfo + g);
  T* dst = voxels + (((int64_t)vi.x * max_voxels + vi.y) * P + (int64_t)j) * f;
  for (int64_t q = 0; q < f; ++q) dst[q] = from_f32<T>(0.f);
}

template <class T>
__global__ __launch_bounds__(kVoxThreads) void vox_pad_kernel(const uint32_t* __restrict__ total_dev,
                                                              const uint32_t* __restrict__ gcnt,
                                                              const int2* __restrict__ vinfo, int64_t f, FastDiv P,
                                                              int64_t max_voxels, T* __restrict__ voxels) {
  const uint64_t total = (uint64_t)*total_dev * P.d;
  if (total < (1ull << 32)) {
    const uint32_t stride = gridDim.x * blockDim.x;
    for (uint32_t t = blockIdx.x * blockDim.x + threadIdx.x; t < (uint32_t)total; t += stride) {
      const uint32_t g = P.div(t);
      pad_slot<T>(g, t - g * P.d, gcnt, vinfo, f, P.d, max_voxels, voxels);
    }
  } else {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
      const uint64_t g = t / P.d;
      pad_slot<T>(g, t - g * P.d, gcnt, vinfo, f, P.d, max_voxels, voxels);
    }
  }
}

// One lane per voxel; voxels above kRankMax points are written by the whole
// warp (first P points by repeated minimum selection, input order; zero
// padding) and their table slots freed.
template <class T>
__global__ __launch_bounds__(kVoxThreads) void vox_order_kernel(
    const T* __restrict__ pts, int64_t f, const uint32_t* __restrict__ total_dev, TableView tb,
    const uint32_t* __restrict__ gcnt, const uint32_t* __restrict__ cursor, const int32_t* __restrict__ gslot,
    const int2* __restrict__ vinfo, const uint32_t* __restrict__ members, int64_t P, int64_t max_voxels,
    T* __restrict__ voxels) {
  const int lane = threadIdx.x & 31;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = *total_dev;
  if (((int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31)) >= total) return;  // whole warp out of range
  const int64_t row_len = P * f;
  uint32_t cnt = 0, end = 0;
  int2 vi = make_int2(0, 0);
  if (g < total) {
    cnt = gcnt[g];
    if (cnt > (uint32_t)kRankMax) {  // the rank kernel skipped this voxel
      const int32_t slot = gslot[g];
      tb.slots[slot].key = kEmptyKey;  // leave the table clean for the next call
      tb.slots[slot].first = kNoFirst;
      tb.slots[slot].cnt = 0u;
      end = cursor[g];
      vi = vinfo[g];
    }
  }
  unsigned big = __ballot_sync(0xffffffffu, cnt > (uint32_t)kRankMax);
  while (big) {
    const int b = __ffs(big) - 1;
    big &= big - 1;
    const uint32_t bc = __shfl_sync(0xffffffffu, cnt, b);
    const uint32_t be = __shfl_sync(0xffffffffu, end, b);
    const int bx = __shfl_sync(0xffffffffu, vi.x, b);
    const int by = __shfl_sync(0xffffffffu, vi.y, b);
    const uint32_t bs = be - bc;
    T* dst = voxels + ((int64_t)bx * max_voxels + by) * row_len;
    const int64_t keep = min((int64_t)bc, P);
    uint32_t last = 0;
    for (int64_t j = 0; j < keep; ++j) {
      uint32_t best = 0xffffffffu;
      for (uint32_t i = bs + lane; i < be; i += 32) {
        const uint32_t m = members[i];
        if ((j == 0 || m > last) && m < best) best = m;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
      last = best;
      for (int64_t q = lane; q < f; q += 32) dst[j * f + q] = pts[(int64_t)best * f + q];
    }
    for (int64_t idx = keep * f + lane; idx < row_len; idx += 32) dst[idx] = from_f32<T>(0.f);
  }
}

// rows [voxel_num[s], max_voxels) of every sample -> 0
template <class T>
__global__ void vox_zero_tail_kernel(const int32_t* __restrict__ voxel_num, int64_t max_voxels, int64_t row_len,
                                     T* __restrict__ voxels, int32_t* __restrict__ coors,
                                     int32_t* __restrict__ num_points) {
  const int s = blockIdx.y;
  const int64_t vn = voxel_num[s];
  const int64_t start = vn * row_len;
  const int64_t total = max_voxels * row_len;
  T* vb = voxels + (int64_t)s * total;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = start + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride)
    vb[i] = from_f32<T>(0.f);
  for (int64_t r = vn + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < max_voxels; r += stride) {
    const int64_t row = (int64_t)s * max_voxels + r;
    coors[3 * row + 0] = 0;
    coors[3 * row + 1] = 0;
    coors[3 * row + 2] = 0;
    num_points[row] = 0;
  }
}

// ---------------------------------------------------------------------------
// fast pipeline (max_points <= kFastMaxP)
// ---------------------------------------------------------------------------
// A tile is up to kFastThreads consecutive points of ONE sample (the host
// cuts every sample into tiles), so a CTA knows its sample without a search
// and voxel numbers, which restart at 0 in each sample, are differences of
// one global scan over the tiles.
struct FastTile {
  int64_t start;  // first point
  int32_t count;  // points
  int32_t sample;
  int32_t head;   // tile index of the sample's first tile
};

// Tile t from the sample offsets and the first tile of every sample (the
// sample is the last s with tpre[s] <= t; samples without points own no tile).
__device__ __forceinline__ FastTile tile_of(int64_t t, const int64_t* __restrict__ offs,
                                            const int64_t* __restrict__ tpre, int batch) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(tpre + mid) <= t) lo = mid; else hi = mid - 1;
  }
  FastTile tl;
  tl.sample = lo;
  tl.head = (int32_t)__ldg(tpre + lo);
  tl.start = __ldg(offs + lo) + (t - tl.head) * kFastThreads;
  tl.count = (int32_t)min((int64_t)kFastThreads, __ldg(offs + lo + 1) - tl.start);
  return tl;
}

template <class T>
__global__ __launch_bounds__(kFastThreads) void vox_fast_insert_kernel(
    const T* __restrict__ pts, int64_t f, Grid gr, const int64_t* __restrict__ offs, const int64_t* __restrict__ tpre,
    int batch, TableView tb, int64_t ps, int32_t* __restrict__ did, int32_t* __restrict__ sd, uint32_t* __restrict__ mem,
    uint32_t* __restrict__ fill, uint32_t* hdr) {
  const FastTile tl = tile_of(blockIdx.x, offs, tpre, batch);
  const int64_t p = tl.start + threadIdx.x;
  const int lane = threadIdx.x & 31;
  const bool in = (int)threadIdx.x < tl.count;
  bool valid = false;
  uint64_t key = kEmptyKey;
  if (in) {
    float xyz[3];
    load_xyz<T>(pts, p, f, xyz);
    int32_t c[3];
    if (cell_of(xyz, gr, c)) {
      valid = true;
      const uint64_t lin = ((uint64_t)c[0] * (uint64_t)gr.g[1] + (uint64_t)c[1]) * (uint64_t)gr.g[2] + (uint64_t)c[2];
      key = ((uint64_t)tl.sample << kLinBits) | lin;
    }
  }
  // a run of neighbouring lanes on the same voxel inserts once, by its first
  // (smallest) point
  const uint64_t prev = __shfl_up_sync(0xffffffffu, key, 1);
  const unsigned heads = __ballot_sync(0xffffffffu, lane == 0 || prev != key);
  const int leader = 31 - __clz(heads & (lanemask_lt() | (1u << lane)));
  int64_t slot = -1;
  bool created = false;
  if (valid && lane == leader) {
    const uint64_t mask = tb.cap - 1;
    uint64_t h = mix64(key) & mask;
    for (uint64_t probe = 0; probe < tb.cap; ++probe) {
      uint64_t k = tb.slots[h].key;
      if (k == kEmptyKey) {
        k = atomicCAS(&tb.slots[h].key, kEmptyKey, (unsigned long long)key);
        created = k == kEmptyKey;
      }
      if (k == kEmptyKey || k == key) {
        slot = (int64_t)h;
        break;
      }
      h = (h + 1) & mask;
    }
    if (slot >= 0) {
      atomicMin(&tb.slots[slot].first, (uint32_t)p);
      const unsigned later = lane < 31 ? heads >> (lane + 1) : 0u;
      const uint32_t run = later ? (uint32_t)__ffs(later) : (uint32_t)(32 - lane);
      atomicAdd(&tb.slots[slot].cnt, run);  // points of the voxel
    } else {
      atomicAdd(hdr + 1, 1u);  // table full: cannot happen when cap >= 2n
    }
  }
  // creators take dense voxel numbers: one shared atomic per warp, one
  // global atomic per block (a single global counter per point would serialise)
  __shared__ uint32_t s_new, s_base;
  if (threadIdx.x == 0) s_new = 0u;
  __syncthreads();
  const unsigned cm = __ballot_sync(0xffffffffu, created);
  uint32_t wbase = 0;
  if (lane == 0 && cm) wbase = atomicAdd(&s_new, (uint32_t)__popc(cm));
  wbase = __shfl_sync(0xffffffffu, wbase, 0);
  __syncthreads();
  if (threadIdx.x == 0 && s_new) s_base = atomicAdd(hdr, s_new);
  __syncthreads();
  if (created) {  // number the voxel and empty its member row
    const uint32_t d = s_base + wbase + (uint32_t)__popc(cm & lanemask_lt());
    tb.slots[slot].gvid = (int32_t)d;
    sd[d] = (int32_t)slot;
    uint4* row = reinterpret_cast<uint4*>(mem + (int64_t)d * ps);
    for (int64_t q = 0; q < ps / 4; ++q) row[q] = make_uint4(kEmptyMember, kEmptyMember, kEmptyMember, kEmptyMember);
    fill[d] = 0u;
  }
  slot = __shfl_sync(0xffffffffu, slot, leader);
  if (in) did[p] = valid ? (int32_t)slot : -1;
}

// Insert point index v into a voxel's member row (ascending, kEmptyMember
// past the filled slots).  Slot j keeps min(held, arriving) and passes the
// larger on, so after every insertion the row holds the P smallest indices
// in order, whatever the order of arrival.  Row values only ever decrease, so
// a slot whose value (read before the chain) is already below v is passed
// without an atomic.
__device__ __forceinline__ void insert_smallest(uint32_t* __restrict__ row, int P, uint32_t v) {
  const uint4* row4 = reinterpret_cast<const uint4*>(row);
  for (int q0 = 0; 4 * q0 < P; q0 += 4) {
    uint32_t a[16];  // up to four row vectors read together (L2, where the atomics act)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 w = 4 * (q0 + u) < P ? __ldcg(row4 + q0 + u) : make_uint4(0u, 0u, 0u, 0u);
      a[4 * u] = w.x; a[4 * u + 1] = w.y; a[4 * u + 2] = w.z; a[4 * u + 3] = w.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = 4 * q0 + i;
      if (j >= P) return;
      if (a[i] < v) continue;  // slot j keeps a smaller index
      const uint32_t old = atomicMin(row + j, v);
      if (old == kEmptyMember) return;
      v = max(old, v);
    }
  }
}

// Per point: its voxel's dense number d.  A voxel with at most P points
// keeps all of them: each point claims a member slot with one atomicAdd, in
// any order (the copy kernel ranks them).  A larger voxel keeps its P
// smallest point indices, in order (insert_smallest).  The voxel's first
// point records (tile, rank among the tile's first points, point count, sample) for
// the copy kernel.  Per tile: the number of first points.
__global__ __launch_bounds__(kFastThreads) void vox_fast_members_kernel(
    const int32_t* __restrict__ did, const VoxSlot* __restrict__ slots, uint32_t* __restrict__ mem,
    uint32_t* __restrict__ fill, int64_t ps, int P, const int64_t* __restrict__ offs, const int64_t* __restrict__ tpre,
    int batch, uint32_t* __restrict__ bsum, int4* __restrict__ rec) {
  __shared__ uint32_t s_ws[kFastThreads / 32];
  const FastTile tl = tile_of(blockIdx.x, offs, tpre, batch);
  const int64_t p = tl.start + threadIdx.x;
  int32_t d = -1;
  uint32_t cnt = 0;
  bool first = false;
  if ((int)threadIdx.x < tl.count) {
    const int32_t sl = __ldg(did + p);
    if (sl >= 0) {
      const VoxSlot v = slots[sl];
      d = v.gvid;
      cnt = v.cnt;
      first = v.first == (uint32_t)p;
    }
  }
  uint32_t total;
  const uint32_t excl = block_exclusive_scan(first ? 1u : 0u, s_ws, &total);
  if (first) rec[d] = make_int4((int)blockIdx.x, (int)excl, (int)cnt, tl.sample);
  if (threadIdx.x == 0) bsum[blockIdx.x] = total;
  uint32_t* row = mem + (int64_t)d * ps;
  if (d >= 0 && cnt <= (uint32_t)P) {
    const uint32_t slot = atomicAdd(fill + d, 1u);
    if (!BFB_BAD(slot < (uint32_t)P)) row[slot] = (uint32_t)p;  // more claims than the count said
  }
  // a larger voxel: at most P points of it per warp can be among its P smallest
  const int32_t big = (d >= 0 && cnt > (uint32_t)P) ? d : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, big);
  if (big >= 0 && __popc(peers & lanemask_lt()) < P) insert_smallest(row, P, (uint32_t)p);
}

// One CTA: bsum -> exclusive scan over all tiles; voxel_num of every sample =
// its tiles' first points (difference of the scan at its last and first tile),
// capped at max_voxels.
constexpr int kFastScanThreads = 1024;
__global__ __launch_bounds__(kFastScanThreads) void vox_fast_scan_kernel(uint32_t* __restrict__ bsum, int64_t ntiles,
                                                                         const int64_t* __restrict__ tpre,
                                                                         int batch, int64_t max_voxels,
                                                                         int32_t* __restrict__ voxel_num) {
  __shared__ uint32_t ws[kFastScanThreads / 32];
  constexpr int kItems = 8;
  uint32_t carry = 0;
  for (int64_t b0 = 0; b0 <= ntiles; b0 += (int64_t)kFastScanThreads * kItems) {  // bsum[ntiles] = grand total
    uint32_t v[kItems];
    uint32_t s = 0;
    const int64_t q0 = b0 + (int64_t)threadIdx.x * kItems;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      v[i] = q0 + i < ntiles ? bsum[q0 + i] : 0u;
      s += v[i];
    }
    uint32_t total;
    uint32_t pre = block_exclusive_scan(s, ws, &total) + carry;
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      if (q0 + i <= ntiles) bsum[q0 + i] = pre;
      pre += v[i];
    }
    carry += total;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < batch; s += kFastScanThreads) {
    const int64_t c = (int64_t)bsum[tpre[s + 1]] - (int64_t)bsum[tpre[s]];
    voxel_num[s] = (int32_t)(max_voxels < 0 ? c : min(c, max_voxels));
  }
}

// A thread per (voxel, point slot) over the voxels' dense numbers: the voxel's
// number within its sample comes from its first point's record and the tile
// scan.  For a kept voxel, slot j's thread takes member j: in a voxel of at
// most P points the members are unordered, so it moves to position = number of
// smaller members; a larger voxel's members are already the P smallest in
// order.  Positions past the voxel's points are zero.  Slot 0 writes the
// coords (decoded from the table key) and the count, then frees the table
// slot, dropped voxels included.
template <class T>
__global__ __launch_bounds__(kFastThreads) void vox_fast_copy_kernel(
    const T* __restrict__ pts, int64_t f, Grid gr, const uint32_t* __restrict__ mem, int64_t ps, int P,
    const int4* __restrict__ rec, const int64_t* __restrict__ tpre, const uint32_t* __restrict__ bsum,
    const int32_t* __restrict__ sd, const uint32_t* __restrict__ hdr, TableView tb, int64_t max_voxels,
    T* __restrict__ voxels, int32_t* __restrict__ coors, int32_t* __restrict__ num_points) {
  const uint64_t items = (uint64_t)hdr[0] * (uint64_t)P;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
    const uint32_t d = (uint32_t)(i / (uint64_t)P);
    const int j = (int)(i - (uint64_t)d * (uint64_t)P);
    const int4 rc = __ldg(rec + d);
    const int64_t local = (int64_t)__ldg(bsum + rc.x) - (int64_t)__ldg(bsum + __ldg(tpre + rc.w)) + rc.y;
    const bool kept = max_voxels < 0 || local < max_voxels;
    const int64_t r = (int64_t)rc.w * max_voxels + local;
    const uint32_t* row = mem + (int64_t)d * ps;
    const int cnt = min(rc.z, P);
    if (kept) {
      T* dst = voxels + r * P * f;
      if (j < cnt) {
        const uint32_t m = __ldg(row + j);
        int pos = j;
        if (rc.z <= P) {  // unordered members: rank among them
          pos = 0;
          for (int q = 0; q < cnt; ++q) pos += __ldg(row + q) < m ? 1 : 0;
        }
        if (BFB_BAD(pos < P)) pos = j;
        const T* src = pts + (int64_t)m * f;
        for (int64_t q = 0; q < f; ++q) dst[pos * f + q] = __ldg(src + q);
      } else {
        for (int64_t q = 0; q < f; ++q) dst[j * f + q] = from_f32<T>(0.f);
      }
    }
    if (j == 0) {
      VoxSlot& sl = tb.slots[__ldg(sd + d)];
      if (kept) {
        num_points[r] = cnt;
        const uint64_t lin = sl.key & ((1ull << kLinBits) - 1ull);
        const uint64_t yz = (uint64_t)gr.g[1] * (uint64_t)gr.g[2];
        coors[3 * r + 0] = (int32_t)(lin / yz);
        coors[3 * r + 1] = (int32_t)((lin % yz) / (uint64_t)gr.g[2]);
        coors[3 * r + 2] = (int32_t)(lin % (uint64_t)gr.g[2]);
      }
      sl.key = kEmptyKey;  // leave the table clean for the next call
      sl.first = kNoFirst;
      sl.cnt = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// mean epilogue: voxel rows of every sample -> packed [M, F] means,
// (b, x, y, z) coords and counts
// ---------------------------------------------------------------------------
constexpr int kEpiMaxBatch = 4096;  // prefix of voxel_num kept in shared memory

// A thread per (voxel row, feature) over batch * max_voxels rows; row `local`
// of sample s (local < voxel_num[s]) lands at packed row prefix(s) + local.
// The mean sums the row's P point slots in slot order in fp32 (unused slots
// hold zeros) and divides once by the count.
template <class T>
__global__ __launch_bounds__(256) void vox_mean_epilogue_kernel(
    const T* __restrict__ voxels, const int32_t* __restrict__ coors, const int32_t* __restrict__ num_points,
    const int32_t* __restrict__ voxel_num, int batch, int64_t max_voxels, int64_t P, int64_t f,
    T* __restrict__ out_feats, int32_t* __restrict__ out_coords, int32_t* __restrict__ out_sizes,
    int32_t* __restrict__ total_dev) {
  __shared__ uint32_t s_pre[kEpiMaxBatch + 1];
  __shared__ uint32_t s_ws[8];
  uint32_t carry = 0;
  for (int b0 = 0; b0 < batch; b0 += 256) {
    const int sidx = b0 + threadIdx.x;
    const uint32_t c = sidx < batch ? (uint32_t)voxel_num[sidx] : 0u;
    uint32_t tot;
    const uint32_t pre = block_exclusive_scan(c, s_ws, &tot) + carry;
    if (sidx < batch) s_pre[sidx] = pre;
    carry += tot;
  }
  if (threadIdx.x == 0) s_pre[batch] = carry;
  __syncthreads();
  if (blockIdx.x == 0 && threadIdx.x == 0 && total_dev) *total_dev = (int32_t)carry;
  const uint64_t items = (uint64_t)batch * (uint64_t)max_voxels * (uint64_t)f;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items; i += stride) {
    const uint64_t row = i / (uint64_t)f;
    const int64_t q = (int64_t)(i - row * (uint64_t)f);
    const int s = (int)(row / (uint64_t)max_voxels);
    const int64_t local = (int64_t)(row - (uint64_t)s * (uint64_t)max_voxels);
    if (local >= (int64_t)(s_pre[s + 1] - s_pre[s])) continue;
    const int64_t k = (int64_t)s_pre[s] + local;
    const T* src = voxels + (int64_t)row * P * f + q;
    float acc = 0.f;
    for (int64_t j = 0; j < P; ++j) acc = __fadd_rn(acc, to_f32<T>(__ldg(src + j * f)));
    const int32_t cnt = __ldg(num_points + row);
    out_feats[k * f + q] = from_f32<T>(__fdiv_rn(acc, (float)cnt));
    if (q == 0) {
      out_coords[4 * k + 0] = s;
      out_coords[4 * k + 1] = __ldg(coors + 3 * row + 0);
      out_coords[4 * k + 2] = __ldg(coors + 3 * row + 1);
      out_coords[4 * k + 3] = __ldg(coors + 3 * row + 2);
      out_sizes[k] = cnt;
    }
  }
}

// every slot free: key empty, no first point, count 0
__global__ void vox_table_init_kernel(TableView tb) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tb.cap; i += stride) {
    VoxSlot s;
    s.key = kEmptyKey;
    s.first = kNoFirst;
    s.cnt = 0u;
    s.gvid = -1;
    s.pad[0] = s.pad[1] = s.pad[2] = 0u;
    tb.slots[i] = s;
  }
}

template <class T>
int hard_voxelize_impl(const void* points, int64_t n, int64_t f, const Grid& gr, const int64_t* offs_host,
                       int64_t batch, int64_t max_points, int64_t max_voxels, void* voxels, int32_t* coors,
                       int32_t* num_points, int32_t* voxel_num, int zero_tail, const TableView& tb,
                       const VoxScratch& sv, cudaStream_t st) {
  const T* pts = static_cast<const T*>(points);
  const int64_t P = max_points < 0 ? n : max_points;
  const int64_t MV = max_voxels < 0 ? n : max_voxels;
  if (int rc = upload_words(sv.offs, offs_host, (size_t)(batch + 1), sv.err, 4, st)) return rc;
  const unsigned nb = (unsigned)ceil_div(n > 0 ? n : 1, kVoxThreads);
  if (n > 0) {
    vox_insert_kernel<T><<<nb, kVoxThreads, 0, st>>>(pts, n, f, gr, sv.offs, (int)batch, tb, sv.slot_of, sv.err);
    BFB_CHECK_LAUNCH();
    vox_flags_kernel<<<nb, kVoxThreads, 0, st>>>(sv.slot_of, n, tb.slots, sv.excl);
    BFB_CHECK_LAUNCH();
  }
  // excl[n] = number of distinct voxels over the batch
  BFB_TRY(exclusive_scan_u32(sv.excl, sv.excl, n, sv.scan, sv.excl + n, st));
  if (n > 0) {
    vox_assign_kernel<T><<<nb, kVoxThreads, 0, st>>>(pts, n, f, gr, sv.offs, (int)batch, tb, sv.slot_of, sv.excl,
                                                     max_points, MV, coors, num_points, sv.gcnt, sv.gslot,
                                                     sv.vinfo);
    BFB_CHECK_LAUNCH();
  }
  vox_count_kernel<<<(unsigned)ceil_div(batch, 128), 128, 0, st>>>(sv.offs, (int)batch, sv.excl, max_voxels,
                                                                    voxel_num);
  BFB_CHECK_LAUNCH();
  if (n > 0) {
    // bucket offsets over voxel ids; entries past the voxel count are never read
    BFB_TRY(exclusive_scan_u32(sv.gcnt, sv.cursor, n + 1, sv.scan, nullptr, st));
    vox_fill_kernel<<<nb, kVoxThreads, 0, st>>>(sv.slot_of, n, tb.slots, sv.cursor, sv.members, sv.mvox);
    BFB_CHECK_LAUNCH();
    vox_rank_kernel<T><<<nb, kVoxThreads, 0, st>>>(pts, f, sv.excl + n, sv.gcnt, sv.cursor, sv.vinfo, sv.members,
                                                   sv.mvox, sv.gslot, tb, P, MV, static_cast<T*>(voxels));
    BFB_CHECK_LAUNCH();
    vox_pad_kernel<T><<<148 * 16, kVoxThreads, 0, st>>>(sv.excl + n, sv.gcnt, sv.vinfo, f, FastDiv((uint32_t)P), MV,
                                                        static_cast<T*>(voxels));
    BFB_CHECK_LAUNCH();
    vox_order_kernel<T><<<nb, kVoxThreads, 0, st>>>(pts, f, sv.excl + n, tb, sv.gcnt, sv.cursor, sv.gslot, sv.vinfo,
                                                    sv.members, P, MV, static_cast<T*>(voxels));
    BFB_CHECK_LAUNCH();
  }
  if (zero_tail) {
    dim3 grid((unsigned)std::min<int64_t>(ceil_div(MV * P * f, 256), 4096), (unsigned)batch);
    vox_zero_tail_kernel<T><<<grid, 256, 0, st>>>(voxel_num, MV, P * f, static_cast<T*>(voxels), coors, num_points);
    BFB_CHECK_LAUNCH();
  }
  return BFB_OK;
}

template <class T>
int hard_voxelize_fast(const void* points, int64_t n, int64_t f, const Grid& gr, const int64_t* offs_host,
                       int64_t batch, int64_t max_points, int64_t max_voxels, void* voxels, int32_t* coors,
                       int32_t* num_points, int32_t* voxel_num, int zero_tail, const TableView& tb,
                       const FastScratch& fv, cudaStream_t st) {
  const T* pts = static_cast<const T*>(points);
  const int P = (int)max_points;
  const int64_t ps = member_stride(P);
  const int64_t MV = max_voxels < 0 ? n : max_voxels;
  // sample offsets and the first tile of every sample, in one small upload
  std::vector<int64_t> up((size_t)(2 * (batch + 1)));
  int64_t tiles = 0;
  for (int64_t s = 0; s <= batch; ++s) {
    up[(size_t)s] = offs_host[s];
    up[(size_t)(batch + 1 + s)] = tiles;
    if (s < batch) tiles += ceil_div(offs_host[s + 1] - offs_host[s], kFastThreads);
  }
  if (int rc = upload_words(fv.offs, up.data(), up.size(), fv.hdr, 16, st)) return rc;
  if (tiles > 0) {
    vox_fast_insert_kernel<T><<<(unsigned)tiles, kFastThreads, 0, st>>>(pts, f, gr, fv.offs, fv.tpre, (int)batch, tb, ps,
                                                                        fv.did, fv.sd, fv.mem, fv.fill, fv.hdr);
    BFB_CHECK_LAUNCH();
    vox_fast_members_kernel<<<(unsigned)tiles, kFastThreads, 0, st>>>(fv.did, tb.slots, fv.mem, fv.fill, ps, P,
                                                                      fv.offs, fv.tpre, (int)batch, fv.bsum, fv.rec);
    BFB_CHECK_LAUNCH();
  }
  vox_fast_scan_kernel<<<1, kFastScanThreads, 0, st>>>(fv.bsum, tiles, fv.tpre, (int)batch, MV, voxel_num);
  BFB_CHECK_LAUNCH();
  if (tiles > 0) {
    vox_fast_copy_kernel<T><<<148 * 16, kFastThreads, 0, st>>>(pts, f, gr, fv.mem, ps, P, fv.rec, fv.tpre, fv.bsum,
                                                              fv.sd, fv.hdr, tb, MV, static_cast<T*>(voxels), coors,
                                                              num_points);
    BFB_CHECK_LAUNCH();
  }
  if (zero_tail) {
    dim3 grid((unsigned)std::min<int64_t>(ceil_div(MV * max_points * f, 256), 4096), (unsigned)batch);
    vox_zero_tail_kernel<T><<<grid, 256, 0, st>>>(voxel_num, MV, max_points * f, static_cast<T*>(voxels), coors,
                                                  num_points);
    BFB_CHECK_LAUNCH();
  }
  return BFB_OK;
}

int check_common(const void* points, int dtype, int64_t n, int64_t f) {
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (n < 0 || f < 3) return BFB_ERR_INVALID_ARG;
  if (n > 0x7ffffffeLL) return BFB_ERR_TOO_LARGE;
  if (n > 0 && !points) return BFB_ERR_INVALID_ARG;
  return BFB_OK;
}

}  // namespace
}  // namespace bfb

using namespace bfb;

extern "C" int bfb_dynamic_voxelize(const void* points, int dtype, int64_t n, int64_t f, const float* voxel_size,
                                    const float* coors_range, int32_t* coors, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_common(points, dtype, n, f));
  Grid gr;
  BFB_TRY(make_grid(voxel_size, coors_range, &gr));
  if (n == 0) return BFB_OK;
  if (!coors) return BFB_ERR_INVALID_ARG;
  cudaStream_t st = as_stream(stream);
  const unsigned nb = (unsigned)ceil_div(n, 256);
  switch (dtype) {
    case BFB_F32: dyn_voxelize_kernel<float><<<nb, 256, 0, st>>>(static_cast<const float*>(points), n, f, gr, coors); break;
    case BFB_F16: dyn_voxelize_kernel<__half><<<nb, 256, 0, st>>>(static_cast<const __half*>(points), n, f, gr, coors); break;
    default: dyn_voxelize_kernel<__nv_bfloat16><<<nb, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(points), n, f, gr, coors); break;
  }
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

// Scratch of one call: the fast pipeline's layout when max_points allows it.
size_t scratch_bytes_for(int64_t n, int64_t batch, int64_t max_points) {
  if (fast_path(max_points, batch)) {
    FastScratch fv;
    return carve_fast(nullptr, n, batch, max_points, &fv);
  }
  VoxScratch sv;
  return carve_scratch(nullptr, n, batch, &sv);
}

extern "C" int bfb_hard_voxelize_workspace_sizes(int64_t n, int64_t batch, int64_t max_points, size_t* table_bytes,
                                                 size_t* scratch_bytes) {
  if (n < 0 || batch < 1 || max_points == 0 || max_points < -1) return BFB_ERR_INVALID_ARG;
  if (n > 0x7ffffffeLL || batch >= (1LL << (64 - kLinBits))) return BFB_ERR_TOO_LARGE;
  TableView tv;
  if (table_bytes) *table_bytes = carve_table(nullptr, table_cap_for_points(n), &tv);
  if (scratch_bytes) *scratch_bytes = scratch_bytes_for(n, batch, max_points);
  return BFB_OK;
}

extern "C" int bfb_hard_voxelize_table_init(void* table, size_t table_bytes, void* stream) {
  const uint64_t cap = table_cap_for_bytes(table_bytes);
  if (!table || cap == 0) return BFB_ERR_WORKSPACE;
  TableView tv;
  carve_table(table, cap, &tv);
  vox_table_init_kernel<<<(unsigned)std::min<uint64_t>((cap + 255) / 256, 148 * 64), 256, 0, as_stream(stream)>>>(tv);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

extern "C" int bfb_hard_voxelize_batch(const void* points, int dtype, const int64_t* offsets, int64_t batch,
                                       int64_t n, int64_t f, const float* voxel_size, const float* coors_range,
                                       int64_t max_points, int64_t max_voxels, void* voxels, int32_t* coors,
                                       int32_t* num_points, int32_t* voxel_num, int zero_tail, void* table,
                                       size_t table_bytes, void* scratch, size_t scratch_bytes, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_common(points, dtype, n, f));
  if (batch < 1 || !offsets || !voxel_num) return BFB_ERR_INVALID_ARG;
  if (batch >= (1LL << (64 - kLinBits))) return BFB_ERR_TOO_LARGE;
  if (max_points == 0 || max_points < -1 || max_voxels == 0 || max_voxels < -1) return BFB_ERR_INVALID_ARG;
  if (offsets[0] != 0 || offsets[batch] != n) return BFB_ERR_INVALID_ARG;
  for (int64_t s = 0; s < batch; ++s)
    if (offsets[s + 1] < offsets[s]) return BFB_ERR_INVALID_ARG;
  if (!voxels || !coors || !num_points) return BFB_ERR_INVALID_ARG;
  Grid gr;
  BFB_TRY(make_grid(voxel_size, coors_range, &gr));
  for (int i = 0; i < 3; ++i)
    if (gr.g[i] <= 0) return BFB_ERR_INVALID_ARG;
  if (gr.g[0] > (1LL << kLinBits) / gr.g[1] / gr.g[2]) return BFB_ERR_TOO_LARGE;
  if ((max_points < 0 ? n : max_points) * f > 0x7fffffffLL) return BFB_ERR_TOO_LARGE;  // one voxel row
  const uint64_t cap = table_cap_for_bytes(table_bytes);
  if (!table || !scratch || cap < (uint64_t)(2 * n) || scratch_bytes_for(n, batch, max_points) > scratch_bytes)
    return BFB_ERR_WORKSPACE;
  TableView tv;
  carve_table(table, cap, &tv);
  cudaStream_t st = as_stream(stream);
  if (fast_path(max_points, batch)) {
    FastScratch fv;
    carve_fast(scratch, n, batch, max_points, &fv);
    switch (dtype) {
      case BFB_F32:
        return hard_voxelize_fast<float>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels, coors,
                                         num_points, voxel_num, zero_tail, tv, fv, st);
      case BFB_F16:
        return hard_voxelize_fast<__half>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels, coors,
                                          num_points, voxel_num, zero_tail, tv, fv, st);
      default:
        return hard_voxelize_fast<__nv_bfloat16>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels,
                                                 coors, num_points, voxel_num, zero_tail, tv, fv, st);
    }
  }
  VoxScratch sv;
  carve_scratch(scratch, n, batch, &sv);
  switch (dtype) {
    case BFB_F32:
      return hard_voxelize_impl<float>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels, coors,
                                       num_points, voxel_num, zero_tail, tv, sv, st);
    case BFB_F16:
      return hard_voxelize_impl<__half>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels, coors,
                                        num_points, voxel_num, zero_tail, tv, sv, st);
    default:
      return hard_voxelize_impl<__nv_bfloat16>(points, n, f, gr, offsets, batch, max_points, max_voxels, voxels,
                                               coors, num_points, voxel_num, zero_tail, tv, sv, st);
  }
}

extern "C" int bfb_hard_voxelize(const void* points, int dtype, int64_t n, int64_t f, const float* voxel_size,
                                 const float* coors_range, int64_t max_points, int64_t max_voxels, void* voxels,
                                 int32_t* coors, int32_t* num_points, int32_t* voxel_num, int zero_tail, void* table,
                                 size_t table_bytes, void* scratch, size_t scratch_bytes, void* stream) {
  const int64_t offs[2] = {0, n};
  return bfb_hard_voxelize_batch(points, dtype, offs, 1, n, f, voxel_size, coors_range, max_points, max_voxels,
                                 voxels, coors, num_points, voxel_num, zero_tail, table, table_bytes, scratch,
                                 scratch_bytes, stream);
}

extern "C" int bfb_hard_voxelize_status(const void* scratch, int64_t n, int64_t batch, int64_t max_points,
                                        int64_t* table_full, void* stream) {
  if (!scratch || !table_full || n < 0 || batch < 1) return BFB_ERR_INVALID_ARG;
  const uint32_t* err = nullptr;
  if (fast_path(max_points, batch)) {
    FastScratch fv;
    carve_fast(const_cast<void*>(scratch), n, batch, max_points, &fv);
    err = fv.hdr + 1;  // table full
  } else {
    VoxScratch sv;
    carve_scratch(const_cast<void*>(scratch), n, batch, &sv);
    err = sv.err;
  }
  uint32_t v = 0;
  cudaStream_t st = as_stream(stream);
  BFB_CUDA(cudaMemcpyAsync(&v, err, sizeof(uint32_t), cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  *table_full = v;
  return BFB_OK;
}


extern "C" int bfb_voxelize_mean_epilogue(const void* voxels, int dtype, const int32_t* coors,
                                          const int32_t* num_points, const int32_t* voxel_num, int64_t batch,
                                          int64_t max_voxels, int64_t max_points, int64_t f, void* out_feats,
                                          int32_t* out_coords, int32_t* out_sizes, int32_t* total_dev,
                                          void* stream) {
  BFB_INJECT_POINT();
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (batch < 1 || max_voxels < 1 || max_points < 1 || f < 1) return BFB_ERR_INVALID_ARG;
  if (batch > kEpiMaxBatch) return BFB_ERR_TOO_LARGE;
  if ((uint64_t)batch * (uint64_t)max_voxels > 0x7fffffffull) return BFB_ERR_TOO_LARGE;
  if (!voxels || !coors || !num_points || !voxel_num || !out_feats || !out_coords || !out_sizes)
    return BFB_ERR_INVALID_ARG;
  cudaStream_t st = as_stream(stream);
  const unsigned grid = (unsigned)std::min<int64_t>(ceil_div(batch * max_voxels * f, 256), 148 * 16);
  switch (dtype) {
    case BFB_F32:
      vox_mean_epilogue_kernel<float><<<grid, 256, 0, st>>>(
          static_cast<const float*>(voxels), coors, num_points, voxel_num, (int)batch, max_voxels, max_points, f,
          static_cast<float*>(out_feats), out_coords, out_sizes, total_dev);
      break;
    case BFB_F16:
      vox_mean_epilogue_kernel<__half><<<grid, 256, 0, st>>>(
          static_cast<const __half*>(voxels), coors, num_points, voxel_num, (int)batch, max_voxels, max_points, f,
          static_cast<__half*>(out_feats), out_coords, out_sizes, total_dev);
      break;
    default:
      vox_mean_epilogue_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(voxels), coors, num_points, voxel_num, (int)batch, max_voxels,
          max_points, f, static_cast<__nv_bfloat16*>(out_feats), out_coords, out_sizes, total_dev);
      break;
  }
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}
