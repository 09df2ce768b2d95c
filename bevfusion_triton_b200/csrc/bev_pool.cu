// bev_pool forward / backward for sm_100a.
//
// Reference semantics: ops/bev_pool/src/bev_pool_triton.py:219-227.
//   out[b, c, z, x, y] = sum over points n with coords[n] = (x, y, z, b) of feats[n, c]
// with the cell rank r = ((b * D + z) * H + x) * W + y (`_flatten_ranks`,
// bev_pool_triton.py:34-39) and out laid out [B, C, D, H, W].
//
// Design (one plan, reused by forward and backward):
//   1. bev_keys_kernel       coords -> 32-bit cell rank per point (+ first radix histogram)
//   2. stable LSD radix sort  (rank, point index) pairs, so a cell's points stay in
//                             ascending index order (the order torch.index_add_ sums in)
//   3. bev_bounds_kernel      [start, end) of every non-empty cell in the sorted order
//   4. bev_tile_plan_kernel   the grid is cut into tiles of 32 consecutive cells (one
//                             row segment of the output plane); a tile whose points
//                             exceed kPiecePoints is cut at cell boundaries into pieces
//   5. scan + bev_emit_kernel one work descriptor per piece
//   6. bev_fwd_kernel         one CTA per piece; each non-empty cell is summed by ONE
//                             warp in ascending point order with fp32 adds (16-byte
//                             row loads, the next rows' loads in flight while the
//                             current ones are added), largest cells first, into a shared
//                             [cell][channel] tile; then every channel-plane segment
//                             of the piece is written coalesced, zeros included (no
//                             memset, no permute).  fp32 results equal index_add_'s
//                             bit for bit.
//   7. bev_bwd_kernel         one CTA per piece: stage grad_out[b, :, cells] in shared
//                             memory (only 32-byte sectors that hold a non-empty
//                             cell), then a warp per cell keeps the cell's gradient
//                             row in registers and stores it to each of the cell's
//                             points with 16-byte stores; dropped points get 0 rows.
#include <mutex>

#include "radix.cuh"
#include "scan.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_bev)
namespace {

constexpr int kTileCells = 32;
constexpr int kPiecePoints = 2048;
constexpr int kPoolWarps = 4;
constexpr int kPoolThreads = kPoolWarps * 32;

// The geometry a plan was built for (points n, grid B, D, H, W).  Every
// kernel that reads a plan is given the caller's geometry and compares it
// with the one stamped into the plan header; on a mismatch it writes nothing,
// reads nothing past the header and raises `mismatch`, because the plan's
// arrays would otherwise be carved at the wrong offsets.
struct PlanGeo {
  uint32_t n, B, D, H, W;
};

struct PlanHeader {
  uint32_t n_valid;
  uint32_t total_pieces;
  uint32_t n_invalid;
  uint32_t mismatch;  // set by a kernel handed a plan of another geometry
  PlanGeo geo;
  uint32_t pad[55];
};
static_assert(sizeof(PlanHeader) == 256, "header is one aligned block");

// True when the plan was built for `g`.  Otherwise one thread of the grid
// raises the header's mismatch flag; the caller then returns.
__device__ __forceinline__ bool plan_matches(const PlanHeader* hdr, const PlanGeo& g) {
  const PlanGeo h = hdr->geo;
  const bool ok = h.n == g.n && h.B == g.B && h.D == g.D && h.H == g.H && h.W == g.W;
  if (!ok && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0)
    atomicExch(const_cast<uint32_t*>(&hdr->mismatch), 1u);
  return ok;
}

// Zeroes a new plan's header and stamps the geometry it is built for.
__global__ void plan_stamp_kernel(PlanHeader* hdr, PlanGeo g) {
  uint32_t* w = reinterpret_cast<uint32_t*>(hdr);
  for (int i = threadIdx.x; i < (int)(sizeof(PlanHeader) / 4); i += blockDim.x) w[i] = 0u;
  __syncthreads();
  if (threadIdx.x == 0) hdr->geo = g;
}

struct Geometry {
  int64_t n, B, D, H, W;
  int64_t dhw, cells, tpb, tiles, max_pieces;
  PlanGeo geo() const { return PlanGeo{(uint32_t)n, (uint32_t)B, (uint32_t)D, (uint32_t)H, (uint32_t)W}; }
};

int make_geometry(int64_t n, int64_t B, int64_t D, int64_t H, int64_t W, Geometry* g) {
  if (n < 0 || B <= 0 || D <= 0 || H <= 0 || W <= 0) return BFB_ERR_INVALID_ARG;
  const int64_t lim = 0x7ffffffeLL;
  if (n > lim) return BFB_ERR_TOO_LARGE;
  if (D > lim / H || D * H > lim / W) return BFB_ERR_TOO_LARGE;
  const int64_t dhw = D * H * W;
  if (B > lim / dhw) return BFB_ERR_TOO_LARGE;
  g->n = n; g->B = B; g->D = D; g->H = H; g->W = W;
  g->dhw = dhw;
  g->cells = B * dhw;
  g->tpb = ceil_div(dhw, kTileCells);
  g->tiles = B * g->tpb;
  g->max_pieces = g->tiles + 2 * ceil_div(n, kPiecePoints) + 1;
  if (g->max_pieces > 0x7fffffffLL) return BFB_ERR_TOO_LARGE;
  return BFB_OK;
}

// Kept between forward and backward: the point permutation (points sorted by
// cell, ascending index within a cell), every cell's [start, end) in it, and
// the work list.
struct PlanView {
  PlanHeader* hdr;
  uint32_t* perm;
  uint32_t* pkey;  // cell rank of every point in input order (sentinel = dropped)
  int2* cell_se;
  int4* pieces;
};

struct ScratchView {
  uint32_t* keys0;
  uint32_t* keys1;
  uint32_t* vtmp;
  uint32_t* hist;
  uint32_t* scan;
  uint32_t* tile_np;
  uint32_t* tile_mask;
};

size_t carve_plan(void* base, const Geometry& g, PlanView* v) {
  Carver c(base);
  v->hdr = c.take<PlanHeader>(1);
  v->perm = c.take<uint32_t>((size_t)g.n);
  v->pkey = c.take<uint32_t>((size_t)g.n);
  v->cell_se = c.take<int2>((size_t)g.cells + 1);
  v->pieces = c.take<int4>((size_t)g.max_pieces);
  return c.bytes();
}

size_t carve_scratch(void* base, const Geometry& g, ScratchView* v) {
  const RadixPlan rp = make_radix_plan((uint32_t)g.cells);
  Carver c(base);
  v->keys0 = c.take<uint32_t>((size_t)g.n);
  v->keys1 = c.take<uint32_t>((size_t)g.n);
  v->vtmp = c.take<uint32_t>((size_t)g.n);
  const size_t hist = radix_hist_elems(g.n, rp);
  v->hist = c.take<uint32_t>(hist);
  size_t scan_n = scan_scratch_elems((int64_t)hist);
  size_t scan_t = scan_scratch_elems(g.tiles + 1);
  v->scan = c.take<uint32_t>(scan_n > scan_t ? scan_n : scan_t);
  v->tile_np = c.take<uint32_t>((size_t)g.tiles + 1);
  v->tile_mask = c.take<uint32_t>((size_t)g.tiles);
  return c.bytes();
}


// ---------------------------------------------------------------------------
// 1. cell ranks
// ---------------------------------------------------------------------------
template <class IT>
__device__ __forceinline__ void load_coord(const IT* coords, int64_t p, int64_t& x, int64_t& y,
                                           int64_t& z, int64_t& b);
template <>
__device__ __forceinline__ void load_coord<int32_t>(const int32_t* coords, int64_t p, int64_t& x,
                                                    int64_t& y, int64_t& z, int64_t& b) {
  const int4 c = __ldg(reinterpret_cast<const int4*>(coords) + p);
  x = c.x; y = c.y; z = c.z; b = c.w;
}
template <>
__device__ __forceinline__ void load_coord<int64_t>(const int64_t* coords, int64_t p, int64_t& x,
                                                    int64_t& y, int64_t& z, int64_t& b) {
  const longlong2* q = reinterpret_cast<const longlong2*>(coords) + 2 * p;
  const longlong2 c0 = __ldg(q), c1 = __ldg(q + 1);
  x = c0.x; y = c0.y; z = c1.x; b = c1.y;
}

// Cell of point p from its (x, y, z, b) coordinates.
template <class IT>
struct CoordCells {
  const IT* coords;
  int64_t B, D, H, W;
  struct Cache {};
  __device__ __forceinline__ bool cell(int64_t p, uint32_t* r, Cache&) const {
    int64_t x, y, z, b;
    load_coord<IT>(coords, p, x, y, z, b);
    const bool ok = (uint64_t)x < (uint64_t)H && (uint64_t)y < (uint64_t)W && (uint64_t)z < (uint64_t)D &&
                    (uint64_t)b < (uint64_t)B;
    *r = (uint32_t)(((b * D + z) * H + x) * W + y);
    return ok;
  }
};

// Cell of frustum point p straight from the camera parameters: the LSS
// geometry (models/vtransforms/base.py:82-126) followed by the quantisation
// and in-grid test of its bev_pool caller (base.py:131-158), so no coordinate
// tensor is formed.  Points are ordered (b, cam, d, h, w) as the caller
// flattens them.  Each row of a 3x3 product is (a0*p0 fused-added to a1*p1)
// plus a2*p2 rounded separately, the association that reproduces torch's
// CUDA broadcast matmul of these shapes on all but a few in a million
// values (measured on the B200); `.long()` truncates toward zero.
struct CameraCells {
  const float* frustum;      // [D, fH, fW, 3] (u, v, depth)
  const float* post_rots;    // [B*N, 3, 3]
  const float* post_trans;   // [B*N, 3]
  const float* combine;      // [B*N, 3, 3]  camera2lidar_rot @ intrins^-1
  const float* trans;        // [B*N, 3]     camera2lidar translation
  const float* extra_rots;   // [B, 3, 3] or null
  const float* extra_trans;  // [B, 3] or null
  FastDiv frustum_pts;       // D * fH * fW
  FastDiv ncam;              // N
  float lower[3], dx[3];     // bx - dx / 2 and dx
  int64_t nz, nx, ny;        // grid cells along z, x, y

  // The parameters of the camera a thread is on, reloaded only when its next
  // point belongs to another camera (a keys tile spans one or two cameras).
  struct Cache {
    uint32_t bn = 0xffffffffu, b = 0;
    float pt[3], pr[9], cm[9], tr[3], er[9], et[3];
  };

  // one row of a 3x3 product: fma(a1, p1, a0 * p0) + a2 * p2
  static __device__ __forceinline__ float row3(float a0, float a1, float a2, const float (&v)[3]) {
    return __fadd_rn(__fmaf_rn(a1, v[1], __fmul_rn(a0, v[0])), __fmul_rn(a2, v[2]));
  }

  __device__ __forceinline__ void load(uint32_t bn, Cache& c) const {
    c.bn = bn;
    c.b = ncam.div(bn);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      c.pt[i] = __ldg(post_trans + 3 * bn + i);
      c.tr[i] = __ldg(trans + 3 * bn + i);
      c.et[i] = extra_trans ? __ldg(extra_trans + 3 * c.b + i) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 9; ++i) {
      c.pr[i] = __ldg(post_rots + 9 * bn + i);
      c.cm[i] = __ldg(combine + 9 * bn + i);
      c.er[i] = extra_rots ? __ldg(extra_rots + 9 * c.b + i) : 0.f;
    }
  }

  __device__ __forceinline__ bool cell(int64_t p, uint32_t* r, Cache& c) const {
    const uint32_t bn = frustum_pts.div((uint32_t)p);
    const uint32_t f = (uint32_t)p - bn * frustum_pts.d;
    if (bn != c.bn) load(bn, c);
    float t[3], u[3], v[3], q[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) t[i] = __fsub_rn(__ldg(frustum + 3 * f + i), c.pt[i]);
#pragma unroll
    for (int i = 0; i < 3; ++i) u[i] = row3(c.pr[i], c.pr[3 + i], c.pr[6 + i], t);  // post_rots^T @ t
    v[0] = __fmul_rn(u[0], u[2]);
    v[1] = __fmul_rn(u[1], u[2]);
    v[2] = u[2];
#pragma unroll
    for (int i = 0; i < 3; ++i) q[i] = __fadd_rn(row3(c.cm[3 * i], c.cm[3 * i + 1], c.cm[3 * i + 2], v), c.tr[i]);
    if (extra_rots) {
      float e[3];
#pragma unroll
      for (int i = 0; i < 3; ++i) e[i] = row3(c.er[3 * i], c.er[3 * i + 1], c.er[3 * i + 2], q);
#pragma unroll
      for (int i = 0; i < 3; ++i) q[i] = e[i];
    }
    if (extra_trans) {
#pragma unroll
      for (int i = 0; i < 3; ++i) q[i] = __fadd_rn(q[i], c.et[i]);
    }
    const int64_t lim[3] = {nx, ny, nz};
    int64_t gi[3];
    bool ok = true;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float g = truncf(__fdiv_rn(__fsub_rn(q[i], lower[i]), dx[i]));
      ok = ok && g >= 0.f && g < (float)lim[i];  // false for NaN
      gi[i] = ok ? (int64_t)g : 0;
    }
    *r = (uint32_t)((((int64_t)c.b * nz + gi[2]) * nx + gi[0]) * ny + gi[1]);
    return ok;
  }
};

// Cell rank of every point (the sentinel B*D*H*W for points outside the
// grid) into the sort's key buffer and the plan's per-point copy, plus the
// sort's first-digit histogram of this tile and the dropped-point count.
template <class Src>
__global__ __launch_bounds__(kRadixThreads) void bev_keys_kernel(
    Src src, int64_t n, uint32_t sentinel, uint32_t* __restrict__ keys, uint32_t* __restrict__ pkey, int bits0,
    uint32_t* __restrict__ hist, int64_t ntiles, PlanHeader* hdr) {
  extern __shared__ uint32_t s_hist[];
  const int nd = 1 << bits0;
  for (int i = threadIdx.x; i < skewed_size(nd); i += kRadixThreads) s_hist[i] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kRadixTile;
  const int64_t end = min(n, base + kRadixTile);
  uint32_t bad = 0;
  typename Src::Cache cache;
  for (int64_t p = base + threadIdx.x; p < end; p += kRadixThreads) {
    uint32_t k;
    const bool ok = src.cell(p, &k, cache);
    if (!ok) k = sentinel;
    bad += ok ? 0u : 1u;
    keys[p] = k;
    pkey[p] = k;
    atomicAdd(&s_hist[skew((int)(k & ((1u << bits0) - 1u)))], 1u);
  }
  // one atomic per warp for the dropped-point counter
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(&hdr->n_invalid, bad);
  __syncthreads();
  for (int d = threadIdx.x; d < nd; d += kRadixThreads) hist[(int64_t)d * ntiles + blockIdx.x] = s_hist[skew(d)];
}

// ---------------------------------------------------------------------------
// 3. per-cell [start, end) in the sorted order; number of in-grid points
// ---------------------------------------------------------------------------
// Four consecutive sorted keys per thread (one 16-byte load).
__global__ void bev_bounds_kernel(const uint32_t* __restrict__ keys, int64_t n, uint32_t sentinel,
                                  int2* __restrict__ cell_se, PlanHeader* hdr) {
  const int64_t p0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (p0 >= n) return;
  uint32_t k[6];  // k[0] = key before p0, k[1..4] = keys p0..p0+3, k[5] = key after
  k[0] = p0 > 0 ? __ldg(keys + p0 - 1) : 0xffffffffu;
  if (p0 + 4 <= n) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(keys + p0));
    k[1] = q.x; k[2] = q.y; k[3] = q.z; k[4] = q.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) k[1 + i] = p0 + i < n ? __ldg(keys + p0 + i) : 0xffffffffu;
  }
  k[5] = p0 + 4 < n ? __ldg(keys + p0 + 4) : 0xffffffffu;
#pragma unroll
  for (int i = 1; i <= 4; ++i) {
    const int64_t p = p0 + i - 1;
    if (p >= n) break;
    const bool first = (p == 0) || k[i - 1] != k[i];
    const bool last = (p == n - 1) || k[i + 1] != k[i];
    if (first) cell_se[k[i]].x = (int)p;
    if (last) cell_se[k[i]].y = (int)(p + 1);
    if (k[i] != sentinel && last && (p == n - 1 || k[i + 1] == sentinel)) hdr->n_valid = (uint32_t)(p + 1);
  }
}

// ---------------------------------------------------------------------------
// 4. tile -> pieces (greedy, cut at cell boundaries)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int tile_cells(int64_t t, int64_t tpb, int64_t dhw, int64_t* r0, int64_t* s0) {
  const int64_t b = t / tpb;
  const int64_t s = (t - b * tpb) * kTileCells;
  *s0 = s;
  *r0 = b * dhw + s;
  const int64_t rem = dhw - s;
  return rem < kTileCells ? (int)rem : kTileCells;
}

__global__ void bev_tile_plan_kernel(const int2* __restrict__ cell_se, int64_t tiles, int64_t tpb,
                                     int64_t dhw, uint32_t* __restrict__ tile_np,
                                     uint32_t* __restrict__ tile_mask) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= tiles) return;  // warp-uniform
  int64_t r0, s0;
  const int nc = tile_cells(t, tpb, dhw, &r0, &s0);
  int cnt = 0;
  if (lane < nc) {
    const int2 se = cell_se[r0 + lane];
    cnt = se.y - se.x;
  }
  uint32_t mask = 1u;
  int tot = cnt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  int run = __shfl_sync(0xffffffffu, cnt, 0);
  for (int l = tot <= kPiecePoints ? nc : 1; l < nc; ++l) {  // a tile that fits is one piece
    const int c = __shfl_sync(0xffffffffu, cnt, l);
    if (run > 0 && run + c > kPiecePoints) {
      mask |= 1u << l;
      run = c;
    } else {
      run += c;
    }
  }
  if (lane == 0) {
    tile_np[t] = __popc(mask);
    tile_mask[t] = mask;
  }
}

// ---------------------------------------------------------------------------
// 5. work descriptors: {tile, ca | cb << 8, pa, pb}
// ---------------------------------------------------------------------------
__global__ void bev_emit_kernel(const int2* __restrict__ cell_se, int64_t tiles, int64_t tpb,
                                int64_t dhw, const uint32_t* __restrict__ piece_base,
                                const uint32_t* __restrict__ tile_mask, int4* __restrict__ pieces) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= tiles) return;
  int64_t r0, s0;
  const int nc = tile_cells(t, tpb, dhw, &r0, &s0);
  int cnt = 0, start = 0x7fffffff;
  if (lane < nc) {
    const int2 se = cell_se[r0 + lane];
    cnt = se.y - se.x;
    if (cnt > 0) start = se.x;
  }
  int tile_pa = start;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tile_pa = min(tile_pa, __shfl_xor_sync(0xffffffffu, tile_pa, o));
  if (tile_pa == 0x7fffffff) tile_pa = 0;
  int incl = cnt;  // inclusive prefix of counts over cells
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t mask = tile_mask[t];
  const bool is_start = lane < nc && ((mask >> lane) & 1u);
  // piece [ca, cb): cb = next start after ca, or nc
  const uint32_t later = lane < 31 ? (mask & (0xfffffffeu << lane)) : 0u;
  const int cb = later ? __ffs(later) - 1 : nc;
  const int cb_clamped = cb < nc ? cb : nc;
  const int pref_cb = __shfl_sync(0xffffffffu, incl, (cb_clamped - 1) & 31);
  const int pref_ca = incl - cnt;  // exclusive prefix at this lane
  if (is_start) {
    const uint32_t idx = piece_base[t] + __popc(mask & ((1u << lane) - 1u));
    pieces[idx] = make_int4((int)t, lane | (cb_clamped << 8), tile_pa + pref_ca, tile_pa + pref_cb);
  }
}

// ---------------------------------------------------------------------------
// vector helpers: VE elements of T per lane, 16-byte loads/stores when VE*sizeof(T) == 16
// ---------------------------------------------------------------------------
template <class T, int VE>
struct VecIO;

template <class T>
struct VecIO<T, 1> {
  static __device__ __forceinline__ void load(const T* p, float (&f)[1]) { f[0] = to_f32<T>(__ldg(p)); }
};
template <>
struct VecIO<float, 4> {
  static __device__ __forceinline__ void load(const float* p, float (&f)[4]) {
    const uint4 r = ld_stream16(p);
    f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
  }
};
template <>
struct VecIO<__half, 8> {
  static __device__ __forceinline__ void load(const __half* p, float (&f)[8]) {
    const uint4 r = ld_stream16(p);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
};
template <>
struct VecIO<__nv_bfloat16, 8> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 r = ld_stream16(p);
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
};

// Shared row stride (bytes) for a [cell][channel] tile: a multiple of 16 that is
// 16 mod 128, so 16-byte accesses of 32 consecutive cells use every bank group.
__host__ __device__ inline int tile_row_bytes(int chs, int elem) {
  int s = (chs * elem + 15) / 16 * 16;
  while (s % 128 != 16) s += 16;
  return s;
}

// ---------------------------------------------------------------------------
// Piece prologue (warp 0): the piece's non-empty cells, largest first.
// s_cell[i] = local cell, s_beg[i] = its first sorted position minus pa,
// s_cnt[i] = its point count; *s_m = number of non-empty cells.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void order_piece_cells(const int2* __restrict__ cell_se, uint32_t r0, int ca, int cb,
                                                  int pa, int* s_cell, int* s_beg, int* s_cnt, int* s_m) {
  const int lane = threadIdx.x & 31;
  const int cell = ca + lane;
  int2 se = make_int2(0, 0);
  if (cell < cb) se = cell_se[r0 + cell];
  const int cnt = (cell < cb) ? se.y - se.x : 0;
  int rank = 0;
#pragma unroll 8
  for (int o = 0; o < 32; ++o) {
    const int co = __shfl_sync(0xffffffffu, cnt, o);
    rank += (co > cnt) || (co == cnt && o < lane);
  }
  if (cnt > 0) {
    s_cell[rank] = cell;
    s_beg[rank] = se.x - pa;
    s_cnt[rank] = cnt;
  }
  const unsigned nz = __ballot_sync(0xffffffffu, cnt > 0);
  if (lane == 0) *s_m = __popc(nz);
}

// Streams the permutation range [wa, wb) of one warp in 32-entry chunks with
// the next chunk prefetched, so perm loads never sit on the critical path.
struct PermStream {
  const uint32_t* perm;
  int wa, wb, chunk;
  uint32_t cur, nxt;
  __device__ __forceinline__ void init(const uint32_t* p, int a, int b, int lane) {
    perm = p; wa = a; wb = b; chunk = 0;
    cur = (a + lane < b) ? __ldg(p + a + lane) : 0u;
    nxt = (a + 32 + lane < b) ? __ldg(p + a + 32 + lane) : 0u;
  }
  // point index at sorted position q (warp-uniform, non-decreasing q)
  __device__ __forceinline__ uint32_t at(int q, int lane) {
    const int k = q - wa;
    if ((k >> 5) != chunk) {
      chunk = k >> 5;
      cur = nxt;
      const int r = wa + (chunk + 1) * 32 + lane;
      nxt = r < wb ? __ldg(perm + r) : 0u;
    }
    return __shfl_sync(0xffffffffu, cur, k & 31);
  }
};

// Row sources of the forward gather.  DenseRows reads feats[pid, slice];
// DepthContextRows forms depth[pid] * context[pixel(pid), slice] on the fly
// (product rounded to fp32 exactly as a materialised feature tensor would be),
// reading the context from its transposed [pixel, C] copy.
template <class T, int VE>
struct DenseRows {
  const T* feats;
  int64_t C;
  const T* base;
  __device__ __forceinline__ void bind(int v0, int lane) { base = feats + (int64_t)(v0 + lane) * VE; }
  __device__ __forceinline__ void load(uint32_t pid, uint32_t /*pos*/, float (&v)[VE]) const {
    VecIO<T, VE>::load(base + (int64_t)pid * C, v);
  }
};

// The permutation handed to this source holds the PIXEL of each sorted point
// and `depth` is in sorted order too (both written by dc_stream_kernel), so a
// row is one context vector times one scalar with no index arithmetic.
struct DepthContextRows {
  const float* depth;   // [n] depth of the sorted points
  const float* ctx_t;   // [pixels, C]
  int64_t C;
  const float* base;
  __device__ __forceinline__ void bind(int v0, int lane) { base = ctx_t + (int64_t)(v0 + lane) * 4; }
  __device__ __forceinline__ void load(uint32_t pix, uint32_t pos, float (&v)[4]) const {
    // context rows are shared by a pixel's depth bins: keep them in L1
    const float4 q = __ldg(reinterpret_cast<const float4*>(base + (int64_t)pix * C));
    const float d = __ldg(depth + pos);
    v[0] = __fmul_rn(d, q.x); v[1] = __fmul_rn(d, q.y); v[2] = __fmul_rn(d, q.z); v[3] = __fmul_rn(d, q.w);
  }
};

// Sum of one cell's rows in ascending point order, software-pipelined: the
// loads of the next U rows are in flight while the current U are added.
// `steps` bounds the loop for the whole warp, `cnt` is this lane's count
// (lane groups summing different cells keep one loop and stay converged).
template <int VE, int U, class Src>
__device__ __forceinline__ void sum_cell_pipelined(const uint32_t* __restrict__ pids, uint32_t pos0, int steps, int cnt,
                                                   const Src& src, bool active, float (&acc)[VE]) {
  float va[U][VE], vb[U][VE];
  auto load = [&](int k, float (&v)[U][VE]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (k + u < cnt && active) {
        src.load(pids[k + u], pos0 + k + u, v[u]);
      } else {
#pragma unroll
        for (int q = 0; q < VE; ++q) v[u][q] = 0.f;
      }
    }
  };
  auto add = [&](int k, const float (&v)[U][VE]) {
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (k + u < cnt) {
#pragma unroll
        for (int q = 0; q < VE; ++q) acc[q] = __fadd_rn(acc[q], v[u][q]);
      }
  };
  load(0, va);
  for (int k = 0; k < steps; k += 2 * U) {
    if (k + U < steps) load(k + U, vb);
    add(k, va);
    if (k + U >= steps) break;
    if (k + 2 * U < steps) load(k + 2 * U, va);
    add(k + U, vb);
  }
}

// Sum of a cell larger than a piece: its permutation slice is streamed from
// global memory by the whole warp (PermStream), PU rows at a time.
template <int VE, int PU, class Src>
__device__ __forceinline__ void sum_cell_streamed(const uint32_t* __restrict__ perm, int a, int cnt, int lane,
                                                  const Src& src, bool active, float (&acc)[VE]) {
  PermStream ps;
  ps.init(perm, a, a + cnt, lane);
  for (int k = 0; k < cnt; k += PU) {
    float v[PU][VE];
#pragma unroll
    for (int u = 0; u < PU; ++u) {
      const uint32_t pid = ps.at(a + k + u, lane);
      if (k + u < cnt && active) {
        src.load(pid, (uint32_t)(a + k + u), v[u]);
      } else {
#pragma unroll
        for (int q = 0; q < VE; ++q) v[u][q] = 0.f;
      }
    }
    // ascending point order, one fp32 add per element per point
#pragma unroll
    for (int u = 0; u < PU; ++u) {
      if (k + u < cnt) {
#pragma unroll
        for (int q = 0; q < VE; ++q) acc[q] = __fadd_rn(acc[q], v[u][q]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// 6. forward: one CTA per (piece, channel slice of 32 vectors)
// ---------------------------------------------------------------------------
template <class T, int VE, int PU, class Src, bool kGroups>
__global__ __launch_bounds__(kPoolThreads) void bev_fwd_kernel(
    Src src, int64_t C, int nvec, int64_t dhw, int64_t tpb,
    const uint32_t* __restrict__ perm, const int2* __restrict__ cell_se,
    const int4* __restrict__ pieces, const PlanHeader* __restrict__ hdr, PlanGeo geo, T* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_cell[kTileCells], s_beg[kTileCells], s_cnt[kTileCells];
  __shared__ int s_m, s_next;
  if (!plan_matches(hdr, geo)) return;
  const int e = blockIdx.x;
  if (e >= (int)hdr->total_pieces) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v0 = blockIdx.y * 32;
  const int nvs = min(32, nvec - v0);                // vectors in this slice
  const int chs_full = min(32, nvec) * VE;           // channel capacity per row
  const int chs = nvs * VE;                           // channels in this slice
  const int row_f = tile_row_bytes(chs_full, 4) / 4;  // floats per acc row
  float* acc_s = reinterpret_cast<float*>(smem);      // [32][row_f]
  uint32_t* s_perm = reinterpret_cast<uint32_t*>(smem + kTileCells * row_f * 4);  // [kPiecePoints]

  const int4 pc = pieces[e];
  const int64_t t = pc.x;
  const int ca = pc.y & 0xff, cb = pc.y >> 8;
  const int pa = pc.z, np = pc.w - pc.z;
  const bool staged = np <= kPiecePoints;  // else: one cell larger than a piece
  const int64_t b = t / tpb;
  const int64_t s0 = (t - b * tpb) * kTileCells;
  const uint32_t r0 = (uint32_t)(b * dhw + s0);

  for (int i = threadIdx.x; i < kTileCells * row_f / 4; i += kPoolThreads)
    reinterpret_cast<float4*>(acc_s)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (staged)
    for (int i = threadIdx.x; i < np; i += kPoolThreads) {
      uint32_t v = __ldg(perm + pa + i);
      if (BFB_BAD(v < geo.n)) v = 0u;  // a corrupt plan: read row 0 instead of out of bounds
      s_perm[i] = v;
    }
  if (warp == 0) order_piece_cells(cell_se, r0, ca, cb, pa, s_cell, s_beg, s_cnt, &s_m);
  if (threadIdx.x == 0) s_next = 0;
  __syncthreads();

  if constexpr (kGroups) {
    // Narrow rows (at most 16 vectors, e.g. 80 fp16 channels = 10 lanes) are
    // summed by lane groups of nvs lanes, each group on its own cell, so most
    // lanes stay busy; a cell is still summed by one group in ascending point
    // order.  The warp takes ngrp consecutive cells of the largest-first
    // list: their counts are close, so one loop bound (the first, largest
    // count) keeps the groups converged.  A piece that is one cell larger
    // than a piece (not staged) is summed by the whole warp.
    const int L = staged ? nvs : 32;  // lanes per group
    const int grp = lane / L, gl = lane - grp * L;
    const int ngrp = 32 / L;
    const bool active = grp < ngrp && gl < nvs;  // lanes past the last group only follow the loop
    src.bind(v0, gl);
    const int m = s_m;
    for (;;) {
      int i0 = 0;
      if (lane == 0) i0 = atomicAdd(&s_next, ngrp);
      i0 = __shfl_sync(0xffffffffu, i0, 0);
      if (i0 >= m) break;
      const int i = i0 + grp;
      const bool has = i < m;
      const int cell = has ? s_cell[i] : 0, beg = has ? s_beg[i] : 0, cnt = has ? s_cnt[i] : 0;
      float acc[VE];
#pragma unroll
      for (int q = 0; q < VE; ++q) acc[q] = 0.f;
      if (staged) {
        sum_cell_pipelined<VE, PU>(s_perm + beg, (uint32_t)(pa + beg), s_cnt[i0], cnt, src, active, acc);
      } else {
        sum_cell_streamed<VE, PU>(perm, pa + beg, cnt, lane, src, active, acc);
      }
      if (active && has) {
        float* dst = acc_s + cell * row_f + gl * VE;
#pragma unroll
        for (int q = 0; q < VE; ++q) dst[q] = acc[q];
      }
    }
  } else {
    const bool active = lane < nvs;
    src.bind(v0, lane);
    const int m = s_m;
    for (;;) {
      int i = 0;
      if (lane == 0) i = atomicAdd(&s_next, 1);
      i = __shfl_sync(0xffffffffu, i, 0);
      if (i >= m) break;
      const int cell = s_cell[i], beg = s_beg[i], cnt = s_cnt[i];
      float acc[VE];
#pragma unroll
      for (int q = 0; q < VE; ++q) acc[q] = 0.f;
      if (staged) {
        sum_cell_pipelined<VE, PU>(s_perm + beg, (uint32_t)(pa + beg), cnt, cnt, src, active, acc);
      } else {
        sum_cell_streamed<VE, PU>(perm, pa + beg, cnt, lane, src, active, acc);
      }
      if (active) {
        float* dst = acc_s + cell * row_f + lane * VE;
#pragma unroll
        for (int q = 0; q < VE; ++q) dst[q] = acc[q];
      }
    }
  }
  __syncthreads();

  // write channel-plane segments [ca, cb) of this slice, coalesced along cells
  const int64_t c0 = (int64_t)v0 * VE;
  T* obase = out + (b * C + c0) * dhw + s0;
  const int cell = ca + lane;
  for (int g4 = warp; g4 * 4 < chs; g4 += kPoolWarps) {
    if (cell < cb) {
      const float4 q = *reinterpret_cast<const float4*>(acc_s + cell * row_f + g4 * 4);
      const float qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = g4 * 4 + i;
        if (ch < chs) obase[(int64_t)ch * dhw + cell] = from_f32<T>(qv[i]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// 7. backward: one CTA per (piece, channel slice); extra CTAs zero dropped rows
// ---------------------------------------------------------------------------
template <class T, int VE>
struct RowIO;
template <class T>
struct RowIO<T, 1> {
  static __device__ __forceinline__ void copy(const T* s, T* d) { d[0] = s[0]; }
  static __device__ __forceinline__ void zero(T* d) { d[0] = from_f32<T>(0.f); }
};
struct RowIO16 {
  static __device__ __forceinline__ void copy(const void* s, void* d) {
    st_stream16(d, *reinterpret_cast<const uint4*>(s));
  }
  static __device__ __forceinline__ void zero(void* d) { st_stream16(d, make_uint4(0, 0, 0, 0)); }
};
template <>
struct RowIO<float, 4> : RowIO16 {};
template <>
struct RowIO<__half, 8> : RowIO16 {};
template <>
struct RowIO<__nv_bfloat16, 8> : RowIO16 {};

template <class T, int VE>
__global__ __launch_bounds__(kPoolThreads) void bev_bwd_kernel(
    const T* __restrict__ gout, int64_t C, int nvec, int64_t dhw, int64_t tpb, int64_t n,
    const uint32_t* __restrict__ perm, const int2* __restrict__ cell_se,
    const int4* __restrict__ pieces, const PlanHeader* __restrict__ hdr, PlanGeo geo, T* __restrict__ gfeat) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int s_cell[kTileCells], s_beg[kTileCells], s_cnt[kTileCells];
  __shared__ int s_m, s_next;
  if (!plan_matches(hdr, geo)) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int v0 = blockIdx.y * 32;
  const int nvs = min(32, nvec - v0);
  const bool active = lane < nvs;
  const int total = (int)hdr->total_pieces;
  const int e = blockIdx.x;
  T* gbase = gfeat + (int64_t)(v0 + lane) * VE;

  if (e >= total) {  // rows of points dropped as out of range -> 0
    const int64_t nvalid = hdr->n_valid;
    const int64_t start = nvalid + (int64_t)(e - total) * kPiecePoints;
    const int64_t end = min(n, start + kPiecePoints);
    for (int64_t p = start + warp; p < end; p += kPoolWarps) {
      const uint32_t pid = __ldg(perm + p);
      if (active) RowIO<T, VE>::zero(gbase + (int64_t)pid * C);
    }
    return;
  }

  const int chs_full = min(32, nvec) * VE;
  const int chs = nvs * VE;
  const int row_b = tile_row_bytes(chs_full, sizeof(T));
  const int4 pc = pieces[e];
  if (pc.z == pc.w) return;  // no points in this piece
  const int64_t t = pc.x;
  const int ca = pc.y & 0xff, cb = pc.y >> 8;
  const int64_t b = t / tpb;
  const int64_t s0 = (t - b * tpb) * kTileCells;
  const uint32_t r0 = (uint32_t)(b * dhw + s0);

  const int pa = pc.z, np = pc.w - pc.z;
  const bool staged = np <= kPiecePoints;
  uint32_t* s_perm = reinterpret_cast<uint32_t*>(smem + kTileCells * row_b);
  if (staged)
    for (int i = threadIdx.x; i < np; i += kPoolThreads) s_perm[i] = __ldg(perm + pa + i);
  if (warp == 0) order_piece_cells(cell_se, r0, ca, cb, pa, s_cell, s_beg, s_cnt, &s_m);
  if (threadIdx.x == 0) s_next = 0;

  // stage grad_out[b, c0 + ch, s0 + cell] -> smem[cell][ch], 4 channels per
  // access; skip 8-cell (32-byte) groups without points
  const int cell = ca + lane;
  bool need = false;
  if (cell < cb) {
    const int2 se = cell_se[r0 + cell];
    need = se.y > se.x;
  }
  const unsigned nz = __ballot_sync(0xffffffffu, need);
  const bool load = cell < cb && ((nz >> (lane & ~7)) & 0xffu);
  const int64_t c0 = (int64_t)v0 * VE;
  const T* gsrc = gout + (b * C + c0) * dhw + s0;
  for (int g4 = warp; g4 * 4 < chs; g4 += kPoolWarps) {
    if (load) {
      T q[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ch = g4 * 4 + i;
        q[i] = ch < chs ? __ldg(gsrc + (int64_t)ch * dhw + cell) : from_f32<T>(0.f);
      }
      T* dst = reinterpret_cast<T*>(smem + cell * row_b) + g4 * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[i] = q[i];
    }
  }
  __syncthreads();

  const int m = s_m;
  for (;;) {
    int i = 0;
    if (lane == 0) i = atomicAdd(&s_next, 1);
    i = __shfl_sync(0xffffffffu, i, 0);
    if (i >= m) break;
    const int cl = s_cell[i], beg = s_beg[i], cnt = s_cnt[i];
    const T* row = reinterpret_cast<const T*>(smem + cl * row_b) + lane * VE;
    if (staged) {
#pragma unroll 4
      for (int k = 0; k < cnt; ++k) {
        const uint32_t pid = s_perm[beg + k];
        if (active) RowIO<T, VE>::copy(row, gbase + (int64_t)pid * C);
      }
    } else {
      PermStream ps;
      ps.init(perm, pa + beg, pa + beg + cnt, lane);
      for (int k = 0; k < cnt; ++k) {
        const uint32_t pid = ps.at(pa + beg + k, lane);
        if (active) RowIO<T, VE>::copy(row, gbase + (int64_t)pid * C);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// 7b. backward in gather form (needs a workspace of one row per grid cell)
//
// bev_rows_kernel copies grad_out[b, :, cell] of every non-empty cell into a
// [cell][C] row buffer (a few tens of MB for a det sample, so it stays in L2);
// bev_gather_kernel then walks the points in input order, reads each point's
// cell rank (pkey, written by the plan) and its row from that buffer, and
// writes grad_feats as one contiguous stream.  Same result as bev_bwd_kernel;
// the output writes are sequential instead of 320-byte rows scattered over
// the whole buffer.
// ---------------------------------------------------------------------------
template <class T, int VE>
struct alignas(VE * sizeof(T) == 16 ? 16 : sizeof(T)) Vec {
  T e[VE];
};
template <class T, int VE>
__device__ __forceinline__ Vec<T, VE> load_vec(const Vec<T, VE>* p) {
  if constexpr (VE * sizeof(T) == 16) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    return *reinterpret_cast<const Vec<T, VE>*>(&r);
  } else {
    Vec<T, VE> v;
#pragma unroll
    for (int i = 0; i < VE; ++i) v.e[i] = __ldg(p->e + i);
    return v;
  }
}
template <class T, int VE>
__device__ __forceinline__ void store_vec(T* p, const Vec<T, VE>& v) {
  if constexpr (VE * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(v.e);
  } else {
#pragma unroll
    for (int i = 0; i < VE; ++i) p[i] = v.e[i];
  }
}

constexpr int kRowsBatch = 5;  // channel vectors loaded before the first store

// One CTA per tile of 32 cells; lane = cell.  Each warp takes kRowsBatch
// channel vectors at a time: their channel-plane segments are read coalesced
// (32-byte sectors without a non-empty cell skipped), then each non-empty
// cell stores the vectors into its row.
template <class T, int VE>
__global__ __launch_bounds__(kPoolThreads) void bev_rows_kernel(const T* __restrict__ gout, int64_t C, int nvec,
                                                                int64_t dhw, int64_t tpb,
                                                                const int2* __restrict__ cell_se,
                                                                const PlanHeader* __restrict__ hdr, PlanGeo geo,
                                                                T* __restrict__ rows) {
  if (!plan_matches(hdr, geo)) return;
  const int64_t t = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t r0, s0;
  const int nc = tile_cells(t, tpb, dhw, &r0, &s0);
  bool need = false;
  if (lane < nc) {
    const int2 se = __ldg(cell_se + r0 + lane);
    need = se.y > se.x;
  }
  const unsigned nz = __ballot_sync(0xffffffffu, need);
  if (nz == 0u) return;
  const bool load = lane < nc && ((nz >> (lane & ~7)) & 0xffu);
  const int64_t b = t / tpb;
  const T* src = gout + b * C * dhw + s0 + lane;
  T* dst = rows + (r0 + lane) * C;
  for (int j0 = warp * kRowsBatch; j0 < nvec; j0 += kPoolWarps * kRowsBatch) {
    Vec<T, VE> q[kRowsBatch];
#pragma unroll
    for (int u = 0; u < kRowsBatch; ++u) {
      const int j = j0 + u;
#pragma unroll
      for (int i = 0; i < VE; ++i)
        q[u].e[i] = (load && j < nvec) ? __ldg(src + (int64_t)(j * VE + i) * dhw) : from_f32<T>(0.f);
    }
    if (need) {
#pragma unroll
      for (int u = 0; u < kRowsBatch; ++u)
        if (j0 + u < nvec) store_vec<T, VE>(dst + (j0 + u) * VE, q[u]);
    }
  }
}

constexpr int kGatherThreads = 256;
constexpr int kGatherPoints = 256;  // points per CTA
constexpr int kGatherBatch = 5;     // loads in flight per thread

template <class T, int VE>
__global__ __launch_bounds__(kGatherThreads) void bev_gather_kernel(const T* __restrict__ rows,
                                                                    const uint32_t* __restrict__ pkey,
                                                                    uint32_t sentinel, int64_t n, int nvec,
                                                                    FastDiv dv, const PlanHeader* __restrict__ hdr,
                                                                    PlanGeo geo, T* __restrict__ gfeat) {
  using V = Vec<T, VE>;
  if (!plan_matches(hdr, geo)) return;
  const int64_t p0 = (int64_t)blockIdx.x * kGatherPoints;
  const uint32_t np = (uint32_t)min((int64_t)kGatherPoints, n - p0);
  const uint32_t total = np * (uint32_t)nvec;  // channel vectors of this CTA's points
  const V* rv = reinterpret_cast<const V*>(rows);
  V* out = reinterpret_cast<V*>(gfeat) + p0 * nvec;
  __shared__ uint32_t s_key[kGatherPoints];
  for (uint32_t i = threadIdx.x; i < np; i += kGatherThreads) s_key[i] = __ldg(pkey + p0 + i);
  __syncthreads();
  for (uint32_t l0 = threadIdx.x; l0 < total; l0 += kGatherThreads * kGatherBatch) {
    V q[kGatherBatch];
#pragma unroll
    for (int u = 0; u < kGatherBatch; ++u) {
      const uint32_t l = l0 + u * kGatherThreads;
      if (l < total) {
        const uint32_t p = dv.div(l);
        const uint32_t ch = l - p * (uint32_t)nvec;
        uint32_t k = s_key[p];
        if (BFB_BAD(k <= sentinel)) k = sentinel;  // a corrupt plan: zero row instead of out of bounds
        if (k != sentinel) {
          q[u] = load_vec<T, VE>(rv + (int64_t)k * nvec + ch);
        } else {
#pragma unroll
          for (int i = 0; i < VE; ++i) q[u].e[i] = from_f32<T>(0.f);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherBatch; ++u) {
      const uint32_t l = l0 + u * kGatherThreads;
      if (l < total) {
        if constexpr (VE * sizeof(T) == 16)
          st_stream16(out + l, *reinterpret_cast<const uint4*>(q[u].e));
        else
          out[l] = q[u];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <class T, int VE, int PU, class Src, bool G>
int launch_fwd_g(const Src& src, int64_t C, const Geometry& g, const PlanView& pv, void* out, cudaStream_t st) {
  const int nvec = (int)(C / VE);
  const int slices = (nvec + 31) / 32;
  const int chs_full = (nvec < 32 ? nvec : 32) * VE;
  const size_t smem = (size_t)kTileCells * tile_row_bytes(chs_full, 4) + kPiecePoints * sizeof(uint32_t);
  if (smem > 48 * 1024)
    BFB_CUDA(cudaFuncSetAttribute(bev_fwd_kernel<T, VE, PU, Src, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
  dim3 grid((unsigned)g.max_pieces, (unsigned)slices);
  bev_fwd_kernel<T, VE, PU, Src, G><<<grid, kPoolThreads, smem, st>>>(
      src, C, nvec, g.dhw, g.tpb, pv.perm, pv.cell_se, pv.pieces, pv.hdr, g.geo(), static_cast<T*>(out));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

// Rows of at most 16 channel vectors are summed by lane groups (several cells
// per warp at once); wider rows by whole warps.
template <class T, int VE, int PU, class Src>
int launch_fwd_v(const Src& src, int64_t C, const Geometry& g, const PlanView& pv, void* out,
               cudaStream_t st) {
  if (C / VE <= 16) return launch_fwd_g<T, VE, PU, Src, true>(src, C, g, pv, out, st);
  return launch_fwd_g<T, VE, PU, Src, false>(src, C, g, pv, out, st);
}

// Pipeline depth of the forward gather: 8 rows for 4-byte features (96
// registers), 4 for 16-bit features (8 elements per lane already).
template <class T, int VE>
int launch_fwd(const void* feats, int64_t C, const Geometry& g, const PlanView& pv, void* out, cudaStream_t st) {
  constexpr int kDepth = (sizeof(T) == 4 || VE == 1) ? 8 : 4;
  DenseRows<T, VE> src{static_cast<const T*>(feats), C, nullptr};
  return launch_fwd_v<T, VE, kDepth>(src, C, g, pv, out, st);
}

template <class T, int VE>
int launch_bwd(const void* gout, int64_t C, const Geometry& g, const PlanView& pv, void* gfeat,
               cudaStream_t st) {
  const int nvec = (int)(C / VE);
  const int slices = (nvec + 31) / 32;
  const int chs_full = (nvec < 32 ? nvec : 32) * VE;
  const size_t smem = (size_t)kTileCells * tile_row_bytes(chs_full, sizeof(T)) + kPiecePoints * sizeof(uint32_t);
  if (smem > 48 * 1024)
    BFB_CUDA(cudaFuncSetAttribute(bev_bwd_kernel<T, VE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)(g.max_pieces + ceil_div(g.n, kPiecePoints)), (unsigned)slices);
  bev_bwd_kernel<T, VE><<<grid, kPoolThreads, smem, st>>>(
      static_cast<const T*>(gout), C, nvec, g.dhw, g.tpb, g.n, pv.perm, pv.cell_se, pv.pieces, pv.hdr,
      g.geo(), static_cast<T*>(gfeat));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

template <class T, int VE>
int launch_bwd_gather(const void* gout, int64_t C, const Geometry& g, const PlanView& pv, void* rows,
                      void* gfeat, cudaStream_t st) {
  const int nvec = (int)(C / VE);
  bev_rows_kernel<T, VE><<<(unsigned)g.tiles, kPoolThreads, 0, st>>>(
      static_cast<const T*>(gout), C, nvec, g.dhw, g.tpb, pv.cell_se, pv.hdr, g.geo(), static_cast<T*>(rows));
  BFB_CHECK_LAUNCH();
  bev_gather_kernel<T, VE><<<(unsigned)ceil_div(g.n, kGatherPoints), kGatherThreads, 0, st>>>(
      static_cast<const T*>(rows), pv.pkey, (uint32_t)g.cells, g.n, nvec, FastDiv((uint32_t)nvec),
      pv.hdr, g.geo(), static_cast<T*>(gfeat));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

bool vec16_ok(const void* p, int64_t C, int esz) {
  return (C * esz) % 16 == 0 && (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

int run_fwd(int dtype, const void* feats, int64_t C, const Geometry& g, const PlanView& pv,
            void* out, cudaStream_t st) {
  switch (dtype) {
    case BFB_F32:
      return vec16_ok(feats, C, 4) ? launch_fwd<float, 4>(feats, C, g, pv, out, st)
                                   : launch_fwd<float, 1>(feats, C, g, pv, out, st);
    case BFB_F16:
      return vec16_ok(feats, C, 2) ? launch_fwd<__half, 8>(feats, C, g, pv, out, st)
                                   : launch_fwd<__half, 1>(feats, C, g, pv, out, st);
    case BFB_BF16:
      return vec16_ok(feats, C, 2) ? launch_fwd<__nv_bfloat16, 8>(feats, C, g, pv, out, st)
                                   : launch_fwd<__nv_bfloat16, 1>(feats, C, g, pv, out, st);
    default:
      return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

int run_bwd(int dtype, const void* gout, int64_t C, const Geometry& g, const PlanView& pv,
            void* gfeat, cudaStream_t st) {
  switch (dtype) {
    case BFB_F32:
      return vec16_ok(gfeat, C, 4) ? launch_bwd<float, 4>(gout, C, g, pv, gfeat, st)
                                   : launch_bwd<float, 1>(gout, C, g, pv, gfeat, st);
    case BFB_F16:
      return vec16_ok(gfeat, C, 2) ? launch_bwd<__half, 8>(gout, C, g, pv, gfeat, st)
                                   : launch_bwd<__half, 1>(gout, C, g, pv, gfeat, st);
    case BFB_BF16:
      return vec16_ok(gfeat, C, 2) ? launch_bwd<__nv_bfloat16, 8>(gout, C, g, pv, gfeat, st)
                                   : launch_bwd<__nv_bfloat16, 1>(gout, C, g, pv, gfeat, st);
    default:
      return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

int run_bwd_gather(int dtype, const void* gout, int64_t C, const Geometry& g, const PlanView& pv, void* rows,
                   void* gfeat, cudaStream_t st) {
  const bool v16 = vec16_ok(gfeat, C, dtype_size(dtype)) && vec16_ok(gout, 0, 1) && vec16_ok(rows, 0, 1);
  switch (dtype) {
    case BFB_F32:
      return v16 ? launch_bwd_gather<float, 4>(gout, C, g, pv, rows, gfeat, st)
                 : launch_bwd_gather<float, 1>(gout, C, g, pv, rows, gfeat, st);
    case BFB_F16:
      return v16 ? launch_bwd_gather<__half, 8>(gout, C, g, pv, rows, gfeat, st)
                 : launch_bwd_gather<__half, 1>(gout, C, g, pv, rows, gfeat, st);
    case BFB_BF16:
      return v16 ? launch_bwd_gather<__nv_bfloat16, 8>(gout, C, g, pv, rows, gfeat, st)
                 : launch_bwd_gather<__nv_bfloat16, 1>(gout, C, g, pv, rows, gfeat, st);
    default:
      return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

// Everything after the keys kernel: sort (its first histogram came with the
// keys), per-cell bounds, tiles, work list.
int finish_plan(const Geometry& g, const PlanView& pv, const ScratchView& sv, const RadixPlan& rp, cudaStream_t st) {
  const int64_t n = g.n;
  uint32_t* keys_sorted = sv.keys0;
  if (n > 0)
    BFB_TRY(radix_sort_index(sv.keys0, sv.keys1, sv.vtmp, pv.perm, n, rp, sv.hist, sv.scan,
                             /*hist0_ready=*/true, st, &keys_sorted));
  BFB_CUDA(cudaMemsetAsync(pv.cell_se, 0, sizeof(int2) * (size_t)(g.cells + 1), st));
  if (n > 0) {
    bev_bounds_kernel<<<(unsigned)ceil_div(ceil_div(n, 4), 256), 256, 0, st>>>(keys_sorted, n, (uint32_t)g.cells,
                                                                              pv.cell_se, pv.hdr);
    BFB_CHECK_LAUNCH();
  }
  const unsigned wblocks = (unsigned)ceil_div(g.tiles * 32, 256);
  bev_tile_plan_kernel<<<wblocks, 256, 0, st>>>(pv.cell_se, g.tiles, g.tpb, g.dhw, sv.tile_np, sv.tile_mask);
  BFB_CHECK_LAUNCH();
  BFB_TRY(exclusive_scan_u32(sv.tile_np, sv.tile_np, g.tiles, sv.scan, &pv.hdr->total_pieces, st));
  bev_emit_kernel<<<wblocks, 256, 0, st>>>(pv.cell_se, g.tiles, g.tpb, g.dhw, sv.tile_np, sv.tile_mask, pv.pieces);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

int check_channels(int64_t c) { return (c <= 0 || c > (1 << 20)) ? BFB_ERR_INVALID_ARG : BFB_OK; }

}  // namespace
}  // namespace bfb

using namespace bfb;

extern "C" int bfb_bev_pool_workspace_sizes(int64_t n, int64_t c, int64_t B, int64_t D, int64_t H,
                                            int64_t W, size_t* plan_bytes, size_t* scratch_bytes) {
  (void)c;
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  PlanView pv;
  ScratchView sv;
  if (plan_bytes) *plan_bytes = carve_plan(nullptr, g, &pv);
  if (scratch_bytes) *scratch_bytes = carve_scratch(nullptr, g, &sv);
  return BFB_OK;
}

extern "C" int bfb_bev_pool_plan(const void* coords, int itype, int64_t n, int64_t B, int64_t D,
                                 int64_t H, int64_t W, void* plan, size_t plan_bytes, void* scratch,
                                 size_t scratch_bytes, void* stream) {
  BFB_INJECT_POINT();
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  if (itype != BFB_I32 && itype != BFB_I64) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (!plan || !scratch) return BFB_ERR_WORKSPACE;
  if (n > 0 && !coords) return BFB_ERR_INVALID_ARG;
  if (n > 0 && (reinterpret_cast<uintptr_t>(coords) & 15)) return BFB_ERR_INVALID_ARG;
  PlanView pv;
  ScratchView sv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes || carve_scratch(nullptr, g, &sv) > scratch_bytes)
    return BFB_ERR_WORKSPACE;
  carve_plan(plan, g, &pv);
  carve_scratch(scratch, g, &sv);
  cudaStream_t st = as_stream(stream);
  const RadixPlan rp = make_radix_plan((uint32_t)g.cells);

  plan_stamp_kernel<<<1, 64, 0, st>>>(pv.hdr, g.geo());
  BFB_CHECK_LAUNCH();
  if (n > 0) {
    const int64_t ntiles = radix_tiles(n);
    const size_t hsm = sizeof(uint32_t) * skewed_size(1 << rp.digit_bits[0]);
    const uint32_t sentinel = (uint32_t)g.cells;
    if (itype == BFB_I32)
      bev_keys_kernel<<<(unsigned)ntiles, kRadixThreads, hsm, st>>>(
          CoordCells<int32_t>{static_cast<const int32_t*>(coords), B, D, H, W}, n, sentinel, sv.keys0, pv.pkey,
          rp.digit_bits[0], sv.hist, ntiles, pv.hdr);
    else
      bev_keys_kernel<<<(unsigned)ntiles, kRadixThreads, hsm, st>>>(
          CoordCells<int64_t>{static_cast<const int64_t*>(coords), B, D, H, W}, n, sentinel, sv.keys0, pv.pkey,
          rp.digit_bits[0], sv.hist, ntiles, pv.hdr);
    BFB_CHECK_LAUNCH();
  }
  return finish_plan(g, pv, sv, rp, st);
}

extern "C" int bfb_bev_pool_geometry_plan(const float* frustum, int64_t nd, int64_t fh, int64_t fw,
                                          const float* post_rots, const float* post_trans, const float* combine,
                                          const float* trans, const float* extra_rots, const float* extra_trans,
                                          int64_t B, int64_t ncam, const float* lower, const float* dx, int64_t D,
                                          int64_t H, int64_t W, void* plan, size_t plan_bytes, void* scratch,
                                          size_t scratch_bytes, void* stream) {
  BFB_INJECT_POINT();
  if (nd <= 0 || fh <= 0 || fw <= 0 || ncam <= 0 || B <= 0) return BFB_ERR_INVALID_ARG;
  if (nd > 0x7fffffffLL / fh / fw || B > 0x7fffffffLL / ncam) return BFB_ERR_TOO_LARGE;
  const int64_t fpts = nd * fh * fw;
  if (B * ncam > 0x7fffffffLL / fpts) return BFB_ERR_TOO_LARGE;
  const int64_t n = B * ncam * fpts;
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  if (!frustum || !post_rots || !post_trans || !combine || !trans || !lower || !dx) return BFB_ERR_INVALID_ARG;
  if (!plan || !scratch) return BFB_ERR_WORKSPACE;
  PlanView pv;
  ScratchView sv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes || carve_scratch(nullptr, g, &sv) > scratch_bytes)
    return BFB_ERR_WORKSPACE;
  carve_plan(plan, g, &pv);
  carve_scratch(scratch, g, &sv);
  cudaStream_t st = as_stream(stream);
  const RadixPlan rp = make_radix_plan((uint32_t)g.cells);
  CameraCells cc{frustum, post_rots, post_trans, combine, trans, extra_rots, extra_trans,
                 FastDiv((uint32_t)fpts), FastDiv((uint32_t)ncam), {lower[0], lower[1], lower[2]},
                 {dx[0], dx[1], dx[2]}, D, H, W};
  plan_stamp_kernel<<<1, 64, 0, st>>>(pv.hdr, g.geo());
  BFB_CHECK_LAUNCH();
  const int64_t ntiles = radix_tiles(n);
  const size_t hsm = sizeof(uint32_t) * skewed_size(1 << rp.digit_bits[0]);
  bev_keys_kernel<<<(unsigned)ntiles, kRadixThreads, hsm, st>>>(cc, n, (uint32_t)g.cells, sv.keys0, pv.pkey,
                                                                rp.digit_bits[0], sv.hist, ntiles, pv.hdr);
  BFB_CHECK_LAUNCH();
  return finish_plan(g, pv, sv, rp, st);
}

extern "C" int bfb_bev_pool_forward_planned(const void* feats, int dtype, int64_t n, int64_t c,
                                            int64_t B, int64_t D, int64_t H, int64_t W,
                                            const void* plan, size_t plan_bytes, void* out,
                                            void* stream) {
  BFB_INJECT_POINT();
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  BFB_TRY(check_channels(c));
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (!plan) return BFB_ERR_WORKSPACE;
  if (!out || (n > 0 && !feats)) return BFB_ERR_INVALID_ARG;
  PlanView pv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes) return BFB_ERR_WORKSPACE;
  carve_plan(const_cast<void*>(plan), g, &pv);
  return run_fwd(dtype, feats, c, g, pv, out, as_stream(stream));
}

extern "C" int bfb_bev_pool_forward(const void* feats, int dtype, const void* coords, int itype,
                                    int64_t n, int64_t c, int64_t B, int64_t D, int64_t H, int64_t W,
                                    void* out, void* plan, size_t plan_bytes, void* scratch,
                                    size_t scratch_bytes, void* stream) {
  BFB_TRY(check_channels(c));
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  BFB_TRY(bfb_bev_pool_plan(coords, itype, n, B, D, H, W, plan, plan_bytes, scratch, scratch_bytes, stream));
  return bfb_bev_pool_forward_planned(feats, dtype, n, c, B, D, H, W, plan, plan_bytes, out, stream);
}

extern "C" int bfb_bev_pool_backward(const void* gout, int dtype, int64_t n, int64_t c, int64_t B,
                                     int64_t D, int64_t H, int64_t W, const void* plan,
                                     size_t plan_bytes, void* gfeat, void* stream) {
  BFB_INJECT_POINT();
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  BFB_TRY(check_channels(c));
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (!plan) return BFB_ERR_WORKSPACE;
  if (n == 0) return BFB_OK;
  if (!gout || !gfeat) return BFB_ERR_INVALID_ARG;
  PlanView pv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes) return BFB_ERR_WORKSPACE;
  carve_plan(const_cast<void*>(plan), g, &pv);
  return run_bwd(dtype, gout, c, g, pv, gfeat, as_stream(stream));
}

extern "C" int bfb_bev_pool_backward_workspace_size(int64_t n, int64_t c, int64_t B, int64_t D, int64_t H,
                                                   int64_t W, int dtype, size_t* bytes) {
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  BFB_TRY(check_channels(c));
  const size_t esz = dtype_size(dtype);
  if (esz == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (!bytes) return BFB_ERR_INVALID_ARG;
  *bytes = (size_t)g.cells * (size_t)c * esz;
  return BFB_OK;
}

extern "C" int bfb_bev_pool_backward_gather(const void* gout, int dtype, int64_t n, int64_t c, int64_t B,
                                            int64_t D, int64_t H, int64_t W, const void* plan,
                                            size_t plan_bytes, void* gfeat, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  BFB_TRY(check_channels(c));
  if (dtype_size(dtype) == 0) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (!plan) return BFB_ERR_WORKSPACE;
  if (n == 0) return BFB_OK;
  if (!gout || !gfeat) return BFB_ERR_INVALID_ARG;
  size_t need = 0;
  BFB_TRY(bfb_bev_pool_backward_workspace_size(n, c, B, D, H, W, dtype, &need));
  if (!workspace || workspace_bytes < need) return BFB_ERR_WORKSPACE;
  PlanView pv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes) return BFB_ERR_WORKSPACE;
  carve_plan(const_cast<void*>(plan), g, &pv);
  return run_bwd_gather(dtype, gout, c, g, pv, workspace, gfeat, as_stream(stream));
}

// cells[p] = cell rank of point p in the plan, -1 when it was dropped
__global__ void plan_cells_kernel(const uint32_t* __restrict__ pkey, int64_t n, uint32_t sentinel,
                                  const PlanHeader* __restrict__ hdr, PlanGeo geo, int64_t* __restrict__ cells) {
  if (!plan_matches(hdr, geo)) return;
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const uint32_t k = pkey[p];
  cells[p] = k == sentinel ? -1 : (int64_t)k;
}

extern "C" int bfb_bev_pool_plan_cells(const void* plan, size_t plan_bytes, int64_t n, int64_t B, int64_t D,
                                       int64_t H, int64_t W, int64_t* cells, void* stream) {
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  if (!plan) return BFB_ERR_WORKSPACE;
  if (n > 0 && !cells) return BFB_ERR_INVALID_ARG;
  PlanView pv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes) return BFB_ERR_WORKSPACE;
  carve_plan(const_cast<void*>(plan), g, &pv);
  if (n == 0) return BFB_OK;
  plan_cells_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, as_stream(stream)>>>(pv.pkey, n, (uint32_t)g.cells, pv.hdr,
                                                                                     g.geo(), cells);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

extern "C" int bfb_bev_pool_invalid_count(const void* plan, int64_t* count, void* stream) {
  if (!plan || !count) return BFB_ERR_INVALID_ARG;
  uint32_t v = 0;
  cudaStream_t st = as_stream(stream);
  BFB_CUDA(cudaMemcpyAsync(&v, &static_cast<const PlanHeader*>(plan)->n_invalid, sizeof(v),
                           cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  *count = v;
  return BFB_OK;
}

extern "C" int bfb_bev_pool_plan_check(const void* plan, int64_t n, int64_t B, int64_t D, int64_t H, int64_t W,
                                       void* stream) {
  if (!plan) return BFB_ERR_INVALID_ARG;
  Geometry g;
  BFB_TRY(make_geometry(n, B, D, H, W, &g));
  PlanHeader h;
  cudaStream_t st = as_stream(stream);
  BFB_CUDA(cudaMemcpyAsync(&h, plan, sizeof(h), cudaMemcpyDeviceToHost, st));
  BFB_CUDA(cudaStreamSynchronize(st));
  const PlanGeo want = g.geo();
  const bool same = h.geo.n == want.n && h.geo.B == want.B && h.geo.D == want.D && h.geo.H == want.H &&
                    h.geo.W == want.W;
  return (same && h.mismatch == 0u) ? BFB_OK : BFB_ERR_PLAN_MISMATCH;
}

// ---------------------------------------------------------------------------
// Forward without any allocation, for callers that cannot call cudaMalloc.
//
// The plan and scratch live in one fixed file-scope device array of
// kNoAllocBytes (64 MiB), which every GPU that loads this library holds until
// the process exits.  Host code may not pass the array's name to a kernel (on
// the host it is only a stand-in symbol), so its device address is looked up
// with cudaGetSymbolAddress once per device, on that device's first call.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kNoAllocBytes = size_t(64) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

int noalloc_scratch_address(void** out) {
  int dev = -1;
  BFB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return BFB_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    BFB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return BFB_OK;
}
}  // namespace

extern "C" int bfb_bev_pool_forward_noalloc(const void* feats, int dtype, const void* coords, int itype,
                                            int64_t n, int64_t c, int64_t B, int64_t D, int64_t H, int64_t W,
                                            void* out, void* stream) {
  size_t plan_b = 0, scratch_b = 0;
  BFB_TRY(bfb_bev_pool_workspace_sizes(n, c, B, D, H, W, &plan_b, &scratch_b));
  plan_b = align_up(plan_b);
  if (plan_b + scratch_b > kNoAllocBytes) return BFB_ERR_TOO_LARGE;
  void* base = nullptr;
  BFB_TRY(noalloc_scratch_address(&base));
  char* p = static_cast<char*>(base);
  return bfb_bev_pool_forward(feats, dtype, coords, itype, n, c, B, D, H, W, out, p, plan_b, p + plan_b,
                              scratch_b, stream);
}

extern "C" size_t bfb_bev_pool_noalloc_capacity(void) { return kNoAllocBytes; }

// ===========================================================================
// Fused depth x context pooling (the LSS camera branch without a feature
// tensor): feats[n, c] = depth[n] * context[cam(n), c, h(n), w(n)] is formed
// on the fly inside the gather.  Forward equals bev_pool on the materialised
// product bit for bit (product and sums rounded as there).
// ===========================================================================
namespace bfb {
namespace {

// out[m][p][r] = in[m][r][p] (fp32), 32 x 32 tiles through shared memory.
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t R, int64_t P) {
  __shared__ float tile[32][33];
  const int64_t m = blockIdx.z;
  const int64_t r0 = (int64_t)blockIdx.y * 32, p0 = (int64_t)blockIdx.x * 32;
  const float* src = in + m * R * P;
  float* dst = out + m * R * P;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i, p = p0 + threadIdx.x;
    if (r < R && p < P) tile[i][threadIdx.x] = src[r * P + p];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t p = p0 + i, r = r0 + threadIdx.x;
    if (r < R && p < P) dst[p * R + r] = tile[threadIdx.x][i];
  }
}

int launch_transpose(const float* in, float* out, int64_t M, int64_t R, int64_t P, cudaStream_t st) {
  if (M == 0 || R == 0 || P == 0) return BFB_OK;
  if (M > 65535 || ceil_div(R, 32) > 65535) return BFB_ERR_TOO_LARGE;
  dim3 grid((unsigned)ceil_div(P, 32), (unsigned)ceil_div(R, 32), (unsigned)M);
  transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(in, out, R, P);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

struct DcDims {
  int64_t cams, nd, hw, c;  // cameras over the batch, depth bins, feature-map pixels, channels
  __host__ __device__ int64_t n() const { return cams * nd * hw; }
};

// Sorted-order stream of the fused forward: pixel and depth of every sorted point.
__global__ void dc_stream_kernel(const uint32_t* __restrict__ perm, int64_t n, const float* __restrict__ depth,
                                 FastDiv dhw, FastDiv hw, const PlanHeader* __restrict__ hdr, PlanGeo geo,
                                 uint32_t* __restrict__ pix, float* __restrict__ dep) {
  if (!plan_matches(hdr, geo)) return;
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= n) return;
  const uint32_t pid = perm[p];
  const uint32_t cam = dhw.div(pid);
  const uint32_t r = pid - cam * dhw.d;
  pix[p] = cam * hw.d + (r - hw.div(r) * hw.d);
  dep[p] = __ldg(depth + pid);
}

// A warp per camera pixel walks its depth bins in order:
//   grad_depth[n]          = sum_c grad[cell(n), c] * context[pixel, c]
//   grad_context[pixel, c] = sum_n depth[n] * grad[cell(n), c]   (ascending n)
// g_t is grad_out transposed to [cell, C]; lanes hold 4 channels each.  The
// 16 dot products of a chunk of 16 depth bins are finished together by a
// reduce-scatter across the lanes (16 shuffles), lane j ending with bin j.
__global__ __launch_bounds__(256) void dc_backward_kernel(const float* __restrict__ g_t, const float* __restrict__ ctx_t,
                                                         const uint32_t* __restrict__ keys, uint32_t cells,
                                                         const float* __restrict__ depth, DcDims dm,
                                                         float* __restrict__ gdepth, float* __restrict__ gctx_t) {
  constexpr int U = 8;
  const int lane = threadIdx.x & 31;
  const int64_t pix = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (pix >= dm.cams * dm.hw) return;  // warp-uniform
  const int64_t cam = pix / dm.hw, p = pix - cam * dm.hw;
  const int nv = (int)(dm.c / 4);
  const bool active = lane < nv;
  float cx[4] = {0.f, 0.f, 0.f, 0.f}, acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (active) VecIO<float, 4>::load(ctx_t + pix * dm.c + lane * 4, cx);
  // point of bin d: (cam * nd + d) * hw + p
  const int64_t n0 = cam * dm.nd * dm.hw + p;
  for (int64_t base = 0; base < dm.nd; base += 32) {
    const int cnt = (int)min((int64_t)32, dm.nd - base);
    const int64_t mine = n0 + (base + lane) * dm.hw;
    const uint32_t myk = lane < cnt ? __ldg(keys + mine) : cells;
    const float myd = lane < cnt ? __ldg(depth + mine) : 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float part[16];
#pragma unroll
      for (int k0 = 0; k0 < 16; k0 += U) {
        float v[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const uint32_t key = __shfl_sync(0xffffffffu, myk, 16 * h + k0 + u);
          if (key < cells && active) {
            VecIO<float, 4>::load(g_t + (int64_t)key * dm.c + lane * 4, v[u]);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) v[u][q] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const float dep = __shfl_sync(0xffffffffu, myd, 16 * h + k0 + u);
          float dot = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            dot = __fmaf_rn(v[u][q], cx[q], dot);  // gradients: fp32 tolerance, fused multiply-adds
            acc[q] = __fmaf_rn(dep, v[u][q], acc[q]);
          }
          part[k0 + u] = dot;
        }
      }
      // reduce-scatter within each half-warp (lane bits 3..0), then across halves
#pragma unroll
      for (int w = 8; w >= 1; w >>= 1) {
        const bool upper = (lane & w) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
          const float send = upper ? part[i] : part[i + w];
          const float keep = upper ? part[i + w] : part[i];
          part[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
        }
      }
      part[0] += __shfl_xor_sync(0xffffffffu, part[0], 16);
      const int bin = 16 * h + (lane & 15);
      if (lane < 16 && bin < cnt) gdepth[n0 + (base + bin) * dm.hw] = part[0];
    }
  }

  if (active) {
    float* dst = gctx_t + pix * dm.c + lane * 4;
    *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
}

// Forward -> backward buffer: context transposed to [pixel, C], then the cell
// of every frustum point (B*D*H*W outside the grid).
size_t dc_aux_bytes(const DcDims& dm) {
  Carver cv(nullptr);
  cv.take<float>((size_t)(dm.cams * dm.hw * dm.c));
  cv.take<uint32_t>((size_t)dm.n());
  return cv.bytes();
}

int dc_check(const DcDims& dm, const Geometry& g) {
  if (dm.cams <= 0 || dm.nd <= 0 || dm.hw <= 0 || dm.c <= 0) return BFB_ERR_INVALID_ARG;
  if (dm.c % 4 != 0 || dm.c > 128) return BFB_ERR_INVALID_ARG;  // a warp holds a 4-channel vector per lane
  if (dm.n() != g.n) return BFB_ERR_INVALID_ARG;
  return BFB_OK;
}

}  // namespace
}  // namespace bfb

extern "C" int bfb_bev_pool_dc_workspace_sizes(int64_t cams, int64_t nd, int64_t fh, int64_t fw, int64_t c,
                                               int64_t B, int64_t D, int64_t H, int64_t W, size_t* plan_bytes,
                                               size_t* scratch_bytes, size_t* aux_bytes, size_t* bwd_bytes) {
  const DcDims dm{cams, nd, fh * fw, c};
  Geometry g;
  BFB_TRY(make_geometry(dm.n(), B, D, H, W, &g));
  BFB_TRY(dc_check(dm, g));
  BFB_TRY(bfb_bev_pool_workspace_sizes(dm.n(), c, B, D, H, W, plan_bytes, scratch_bytes));
  if (aux_bytes) *aux_bytes = dc_aux_bytes(dm);
  if (bwd_bytes) {
    Carver cv(nullptr);
    cv.take<float>((size_t)(g.cells * c));        // grad table [cell, C]
    cv.take<float>((size_t)(cams * dm.hw * c));   // grad context [pixel, C]
    *bwd_bytes = cv.bytes();
  }
  return BFB_OK;
}

extern "C" int bfb_bev_pool_dc_forward_planned(const float* depth, const float* context, int64_t cams, int64_t nd,
                                               int64_t fh, int64_t fw, int64_t c, int64_t B, int64_t D, int64_t H,
                                               int64_t W, const void* plan, size_t plan_bytes, float* out,
                                               void* scratch, size_t scratch_bytes, void* aux, size_t aux_bytes,
                                               void* stream) {
  BFB_INJECT_POINT();
  const DcDims dm{cams, nd, fh * fw, c};
  Geometry g;
  BFB_TRY(make_geometry(dm.n(), B, D, H, W, &g));
  BFB_TRY(dc_check(dm, g));
  if (!depth || !context || !out) return BFB_ERR_INVALID_ARG;
  if (!plan || !scratch) return BFB_ERR_WORKSPACE;
  if (!aux || aux_bytes < dc_aux_bytes(dm)) return BFB_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(aux) & 15) || (reinterpret_cast<uintptr_t>(out) & 3)) return BFB_ERR_INVALID_ARG;
  if (nd * dm.hw > 0xffffffffLL || dm.n() > 0x7fffffffLL) return BFB_ERR_TOO_LARGE;
  PlanView pv;
  if (carve_plan(nullptr, g, &pv) > plan_bytes) return BFB_ERR_WORKSPACE;
  carve_plan(const_cast<void*>(plan), g, &pv);
  cudaStream_t st = as_stream(stream);
  Carver av(aux);
  float* ctx_t = av.take<float>((size_t)(cams * dm.hw * c));
  uint32_t* keys = av.take<uint32_t>((size_t)dm.n());
  BFB_TRY(launch_transpose(context, ctx_t, cams, c, dm.hw, st));  // [cam][C][hw] -> [cam][hw][C]
  BFB_CUDA(cudaMemcpyAsync(keys, pv.pkey, sizeof(uint32_t) * (size_t)dm.n(), cudaMemcpyDeviceToDevice, st));
  // sorted pixel / depth streams in the scratch
  Carver sc(scratch);
  uint32_t* spix = sc.take<uint32_t>((size_t)dm.n());
  float* sdep = sc.take<float>((size_t)dm.n());
  if (sc.bytes() > scratch_bytes) return BFB_ERR_WORKSPACE;
  dc_stream_kernel<<<(unsigned)ceil_div(dm.n(), 256), 256, 0, st>>>(pv.perm, dm.n(), depth,
                                                                   FastDiv((uint32_t)(nd * dm.hw)),
                                                                   FastDiv((uint32_t)dm.hw), pv.hdr, g.geo(), spix,
                                                                   sdep);
  BFB_CHECK_LAUNCH();
  PlanView sv = pv;
  sv.perm = spix;
  DepthContextRows src{sdep, ctx_t, c, nullptr};
  // the context rows come from L2 (a few MB per sample), so 4 rows in flight
  // per warp suffice; the smaller register file lets more warps in
  return launch_fwd_v<float, 4, 4>(src, c, g, sv, out, st);
}

extern "C" int bfb_bev_pool_dc_forward(const float* depth, const float* context, const void* coords, int itype,
                                       int64_t cams, int64_t nd, int64_t fh, int64_t fw, int64_t c, int64_t B,
                                       int64_t D, int64_t H, int64_t W, float* out, void* plan, size_t plan_bytes,
                                       void* scratch, size_t scratch_bytes, void* aux, size_t aux_bytes,
                                       void* stream) {
  const DcDims dm{cams, nd, fh * fw, c};
  Geometry g;
  BFB_TRY(make_geometry(dm.n(), B, D, H, W, &g));
  BFB_TRY(dc_check(dm, g));
  if (!depth || !context || !out) return BFB_ERR_INVALID_ARG;
  if (itype != BFB_I32 && itype != BFB_I64) return BFB_ERR_UNSUPPORTED_DTYPE;
  BFB_TRY(bfb_bev_pool_plan(coords, itype, dm.n(), B, D, H, W, plan, plan_bytes, scratch, scratch_bytes, stream));
  return bfb_bev_pool_dc_forward_planned(depth, context, cams, nd, fh, fw, c, B, D, H, W, plan, plan_bytes, out,
                                         scratch, scratch_bytes, aux, aux_bytes, stream);
}

extern "C" int bfb_bev_pool_dc_backward(const float* grad_out, const float* depth, const void* coords, int itype,
                                        int64_t cams, int64_t nd, int64_t fh, int64_t fw, int64_t c, int64_t B,
                                        int64_t D, int64_t H, int64_t W, const void* aux, size_t aux_bytes,
                                        void* ws, size_t ws_bytes, float* grad_depth, float* grad_context,
                                        void* stream) {
  BFB_INJECT_POINT();
  const DcDims dm{cams, nd, fh * fw, c};
  Geometry g;
  BFB_TRY(make_geometry(dm.n(), B, D, H, W, &g));
  BFB_TRY(dc_check(dm, g));
  (void)coords;  // the cells come from aux
  (void)itype;
  if (!grad_out || !depth || !grad_depth || !grad_context) return BFB_ERR_INVALID_ARG;
  if (!aux || aux_bytes < dc_aux_bytes(dm)) return BFB_ERR_WORKSPACE;
  size_t need = 0;
  BFB_TRY(bfb_bev_pool_dc_workspace_sizes(cams, nd, fh, fw, c, B, D, H, W, nullptr, nullptr, nullptr, &need));
  if (!ws || ws_bytes < need) return BFB_ERR_WORKSPACE;
  Carver av(const_cast<void*>(aux));
  const float* ctx_t = av.take<float>((size_t)(cams * dm.hw * c));
  const uint32_t* keys = av.take<uint32_t>((size_t)dm.n());
  Carver cv(ws);
  float* g_t = cv.take<float>((size_t)(g.cells * c));
  float* gctx_t = cv.take<float>((size_t)(cams * dm.hw * c));
  cudaStream_t st = as_stream(stream);
  BFB_TRY(launch_transpose(grad_out, g_t, B, c, g.dhw, st));  // [B][C][DHW] -> [B][DHW][C]
  dc_backward_kernel<<<(unsigned)ceil_div(cams * dm.hw * 32, 256), 256, 0, st>>>(g_t, ctx_t, keys, (uint32_t)g.cells, depth, dm,
                                                                                 grad_depth, gctx_t);
  BFB_CHECK_LAUNCH();
  BFB_TRY(launch_transpose(gctx_t, grad_context, cams, dm.hw, c, st));    // [cam][hw][C] -> [cam][C][hw]
  return BFB_OK;
}
