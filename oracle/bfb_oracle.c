/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the parity tests, smoke()
 * and bench.py's CPU baseline.  Nothing in the product path links or calls
 * this file.
 *
 * A plain-C restatement of the reference's CPU semantics for the hot path of
 * ziyangyeh/bevfusion-triton:
 *   - bev_pool            ops/bev_pool/src/bev_pool_triton.py:34-48 (`_flatten_ranks`,
 *                         `_bev_pool_cpu`: zeros().index_add_(0, ranks, feats) then
 *                         permute to [B, C, D, H, W], :227) and the backward gather
 *                         :102-150 / :188-216.
 *   - dynamic_voxelize    ops/voxel/src/voxelization_triton.py:328-349
 *                         (`_dynamic_voxelize_cpu_fallback`).
 *   - hard_voxelize       ops/voxel/src/voxelization_triton.py:466-513
 *                         (`_hard_voxelize_cpu_fallback`).
 *   - dynamic scatter     ops/voxel/src/scatter_points_triton.py:150-250 (`_clean_coors`,
 *                         `_unique_with_inverse_and_counts`, forward) and :317-345 (backward).
 *   - indice pairs        ops/spconv/src/spconv_triton.py:321-334 (`_row_array_idx`),
 *                         :528-605 (`_valid_out_pos`, `_valid_out_pos_transpose`),
 *                         :655-749 (`_get_indice_pairs_impl`, cuda_ordering=True: the
 *                         order of the reference's GPU path).
 *
 * Compiled with -O2 -ffp-contract=off and without fast-math so every fp32
 * operation rounds exactly as in the reference (SSE fp32, one rounding per op).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ----------------------------------------------------------------------- */
/* bev_pool                                                                */
/* ----------------------------------------------------------------------- */

/* out [B, C, D, H, W] fp32.  Each cell's sum is accumulated in fp32 in
 * ascending point order (index_add_ walks the index sequentially).  Returns
 * the number of points whose coordinates fall outside the grid (skipped; the
 * reference raises for those). */
int64_t oracle_bev_pool_fwd(const float* feats, const int64_t* coords, int64_t n, int64_t c,
                            int64_t B, int64_t D, int64_t H, int64_t W, float* out) {
  const int64_t dhw = D * H * W;
  int64_t bad = 0;
  memset(out, 0, sizeof(float) * (size_t)(B * c * dhw));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t x = coords[4 * i + 0], y = coords[4 * i + 1], z = coords[4 * i + 2],
                  b = coords[4 * i + 3];
    if (x < 0 || x >= H || y < 0 || y >= W || z < 0 || z >= D || b < 0 || b >= B) {
      ++bad;
      continue;
    }
    const int64_t s = (z * H + x) * W + y;
    float* o = out + b * c * dhw + s;
    const float* f = feats + i * c;
    for (int64_t ch = 0; ch < c; ++ch) o[ch * dhw] += f[ch];
  }
  return bad;
}

/* grad_feats[n, :] = grad_out[b, :, z, x, y]; rows of out-of-grid points = 0. */
void oracle_bev_pool_bwd(const float* grad_out, const int64_t* coords, int64_t n, int64_t c,
                         int64_t B, int64_t D, int64_t H, int64_t W, float* grad_feats) {
  const int64_t dhw = D * H * W;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t x = coords[4 * i + 0], y = coords[4 * i + 1], z = coords[4 * i + 2],
                  b = coords[4 * i + 3];
    float* g = grad_feats + i * c;
    if (x < 0 || x >= H || y < 0 || y >= W || z < 0 || z >= D || b < 0 || b >= B) {
      for (int64_t ch = 0; ch < c; ++ch) g[ch] = 0.f;
      continue;
    }
    const float* o = grad_out + b * c * dhw + (z * H + x) * W + y;
    for (int64_t ch = 0; ch < c; ++ch) g[ch] = o[ch * dhw];
  }
}

/* ----------------------------------------------------------------------- */
/* voxelisation                                                            */
/* ----------------------------------------------------------------------- */

/* grid = int(round((max - min) / size)) in double (voxelization_triton.py:36-38;
 * Python's round is half-to-even, as is nearbyint in the default mode). */
void oracle_grid_size(const float* vsize, const float* range, int64_t* grid) {
  for (int i = 0; i < 3; ++i) {
    double v = ((double)range[3 + i] - (double)range[i]) / (double)vsize[i];
    grid[i] = (int64_t)nearbyint(v);
  }
}

/* One point: cell = floor((p - min) / size) in fp32, all three -1 when any axis
 * is out of range (voxelization_triton.py:337-349). */
static int cell_of(const float* p, const float* vsize, const float* range, const int64_t* grid,
                   int32_t* cxyz) {
  for (int j = 0; j < 3; ++j) {
    volatile float d = p[j] - range[j];
    volatile float q = d / vsize[j];
    const float f = floorf(q);
    if (!(f >= 0.f) || f >= (float)grid[j]) { /* NaN-safe */
      cxyz[0] = cxyz[1] = cxyz[2] = -1;
      return 0;
    }
    cxyz[j] = (int32_t)f;
  }
  return 1;
}

void oracle_dynamic_voxelize(const float* points, int64_t n, int64_t f, const float* vsize,
                             const float* range, int32_t* coors) {
  int64_t grid[3];
  oracle_grid_size(vsize, range, grid);
  for (int64_t i = 0; i < n; ++i) cell_of(points + i * f, vsize, range, grid, coors + 3 * i);
}

/* open-addressing map: linear key -> voxel id */
typedef struct {
  int64_t* keys;
  int32_t* vals;
  uint64_t mask;
} omap;

static int omap_init(omap* m, int64_t n) {
  uint64_t cap = 16;
  while (cap < (uint64_t)(2 * n + 1)) cap <<= 1;
  m->keys = (int64_t*)malloc(sizeof(int64_t) * cap);
  m->vals = (int32_t*)malloc(sizeof(int32_t) * cap);
  if (!m->keys || !m->vals) return 0;
  for (uint64_t i = 0; i < cap; ++i) m->keys[i] = -1;
  m->mask = cap - 1;
  return 1;
}
static void omap_free(omap* m) {
  free(m->keys);
  free(m->vals);
}
static uint64_t mix64(uint64_t k) {
  k ^= k >> 33; k *= 0xff51afd7ed558ccdULL; k ^= k >> 33; k *= 0xc4ceb9fe1a85ec53ULL; k ^= k >> 33;
  return k;
}
/* returns slot; *found tells whether the key existed */
static uint64_t omap_find(omap* m, int64_t key, int* found) {
  uint64_t s = mix64((uint64_t)key) & m->mask;
  while (m->keys[s] != -1 && m->keys[s] != key) s = (s + 1) & m->mask;
  *found = m->keys[s] == key;
  return s;
}

/* The sequential first-occurrence algorithm.  Output buffers are
 * zero-filled in full first; returns voxel_num, or -1 on allocation failure.
 * points/voxels hold fp32 values (callers convert other dtypes). */
int64_t oracle_hard_voxelize(const float* points, int64_t n, int64_t f, const float* vsize,
                             const float* range, int64_t max_points, int64_t max_voxels,
                             float* voxels, int32_t* coors, int32_t* num_points, int64_t cap_voxels) {
  int64_t grid[3];
  oracle_grid_size(vsize, range, grid);
  const int64_t mp = max_points;
  memset(voxels, 0, sizeof(float) * (size_t)(cap_voxels * (mp > 0 ? mp : 0) * f));
  memset(coors, 0, sizeof(int32_t) * (size_t)(cap_voxels * 3));
  memset(num_points, 0, sizeof(int32_t) * (size_t)cap_voxels);
  omap m;
  if (!omap_init(&m, n)) return -1;
  int64_t voxel_num = 0;
  for (int64_t i = 0; i < n; ++i) {
    int32_t c[3];
    if (!cell_of(points + i * f, vsize, range, grid, c)) continue;
    const int64_t key = ((int64_t)c[0] * grid[1] + c[1]) * grid[2] + c[2];
    int found;
    const uint64_t s = omap_find(&m, key, &found);
    int64_t vid;
    if (found) {
      vid = m.vals[s];
    } else {
      if (max_voxels != -1 && voxel_num >= max_voxels) continue;
      vid = voxel_num++;
      m.keys[s] = key;
      m.vals[s] = (int32_t)vid;
      coors[3 * vid + 0] = c[0];
      coors[3 * vid + 1] = c[1];
      coors[3 * vid + 2] = c[2];
    }
    const int32_t k = num_points[vid];
    if (mp == -1 || k < mp) {
      if (mp != -1) memcpy(voxels + (vid * mp + k) * f, points + i * f, sizeof(float) * (size_t)f);
      num_points[vid] = k + 1;
    }
  }
  omap_free(&m);
  return voxel_num;
}

/* ----------------------------------------------------------------------- */
/* dynamic scatter                                                         */
/* ----------------------------------------------------------------------- */

static const int32_t* g_rows; /* qsort context */
static int64_t g_ndim;
static int cmp_rows(const void* a, const void* b) {
  const int64_t i = *(const int64_t*)a, j = *(const int64_t*)b;
  for (int64_t d = 0; d < g_ndim; ++d) {
    const int32_t x = g_rows[i * g_ndim + d], y = g_rows[j * g_ndim + d];
    if (x != y) return x < y ? -1 : 1;
  }
  return i < j ? -1 : (i > j);
}

/* Unique rows (ascending lexicographic) of coors with every row that has a
 * negative entry removed; map[i] = unique index or -1; counts per unique row.
 * out_coors must hold n rows.  Returns m. */
int64_t oracle_unique_rows(const int32_t* coors, int64_t n, int64_t ndim, int32_t* out_coors,
                           int32_t* map, int32_t* counts) {
  int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
  int64_t nv = 0;
  for (int64_t i = 0; i < n; ++i) {
    int neg = 0;
    for (int64_t d = 0; d < ndim; ++d) neg |= coors[i * ndim + d] < 0;
    map[i] = -1;
    if (!neg) idx[nv++] = i;
  }
  g_rows = coors;
  g_ndim = ndim;
  qsort(idx, (size_t)nv, sizeof(int64_t), cmp_rows);
  int64_t m = 0;
  for (int64_t k = 0; k < nv; ++k) {
    const int64_t i = idx[k];
    int same = k > 0;
    if (same) {
      const int64_t j = idx[k - 1];
      for (int64_t d = 0; d < ndim; ++d) same &= coors[i * ndim + d] == coors[j * ndim + d];
    }
    if (!same) {
      memcpy(out_coors + m * ndim, coors + i * ndim, sizeof(int32_t) * (size_t)ndim);
      counts[m] = 0;
      ++m;
    }
    map[i] = (int32_t)(m - 1);
    counts[m - 1] += 1;
  }
  free(idx);
  return m;
}

/* reduce: 0 = sum, 1 = mean, 2 = max.  Sums run in ascending point order in
 * fp32 (index_add_); mean divides the fp32 sum by the count; max starts at
 * -inf. */
void oracle_scatter_fwd(const float* feats, int64_t n, int64_t c, const int32_t* map,
                        const int32_t* counts, int64_t m, int reduce, float* out) {
  for (int64_t k = 0; k < m * c; ++k) out[k] = reduce == 2 ? -INFINITY : 0.f;
  for (int64_t i = 0; i < n; ++i) {
    const int32_t v = map[i];
    if (v < 0) continue;
    for (int64_t ch = 0; ch < c; ++ch) {
      float* o = out + (int64_t)v * c + ch;
      const float x = feats[i * c + ch];
      if (reduce == 2) {
        if (x > *o) *o = x;
      } else {
        *o += x;
      }
    }
  }
  if (reduce == 1)
    for (int64_t k = 0; k < m; ++k)
      for (int64_t ch = 0; ch < c; ++ch) out[k * c + ch] = out[k * c + ch] / (float)counts[k];
}

/* sum: grad row copied; mean: divided by count; max: the gradient goes to the
 * lowest point index whose feature equals the reduced value (per channel). */
void oracle_scatter_bwd(const float* grad_out, const float* feats, const float* reduced, int64_t n,
                        int64_t c, const int32_t* map, const int32_t* counts, int64_t m, int reduce,
                        float* grad_feats) {
  memset(grad_feats, 0, sizeof(float) * (size_t)(n * c));
  if (reduce != 2) {
    for (int64_t i = 0; i < n; ++i) {
      const int32_t v = map[i];
      if (v < 0) continue;
      for (int64_t ch = 0; ch < c; ++ch) {
        const float g = grad_out[(int64_t)v * c + ch];
        grad_feats[i * c + ch] = reduce == 1 ? g / (float)counts[v] : g;
      }
    }
    return;
  }
  unsigned char* done = (unsigned char*)calloc((size_t)(m * c > 0 ? m * c : 1), 1);
  for (int64_t i = 0; i < n; ++i) {
    const int32_t v = map[i];
    if (v < 0) continue;
    for (int64_t ch = 0; ch < c; ++ch) {
      const int64_t o = (int64_t)v * c + ch;
      if (!done[o] && feats[i * c + ch] == reduced[o]) {
        grad_feats[i * c + ch] = grad_out[o];
        done[o] = 1;
      }
    }
  }
  free(done);
}

/* ----------------------------------------------------------------------- */
/* sparse-convolution rulebook                                             */
/* ----------------------------------------------------------------------- */

static int64_t floordiv64(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return q;
}

#define SP_MAXD 4

/* Output positions reached from input position `in` with their kernel
 * offsets, in the enumeration order of _valid_out_pos /
 * _valid_out_pos_transpose.  Returns the count. */
static int valid_out_pos(const int64_t* in, int ndim, const int64_t* ks, const int64_t* st, const int64_t* pad,
                         const int64_t* dil, const int64_t* out_shape, int transpose, int64_t* coords_out,
                         int64_t* offsets) {
  int64_t lo[SP_MAXD], up[SP_MAXD], sz[SP_MAXD];
  for (int i = 0; i < ndim; ++i) {
    if (transpose) {
      lo[i] = in[i] * st[i] - pad[i];
      up[i] = lo[i] + (ks[i] - 1) * dil[i];
    } else {
      lo[i] = floordiv64(in[i] - (ks[i] - 1) * dil[i] - 1 + st[i] + pad[i], st[i]);
      up[i] = floordiv64(in[i] + pad[i], st[i]);
    }
    sz[i] = floordiv64(up[i] - lo[i], dil[i]) + 1;
    if (sz[i] <= 0) return 0;
  }
  int64_t ctr[SP_MAXD] = {0, 0, 0, 0};
  int cnt = 0;
  for (;;) {
    int64_t off = 0, mult = 1;
    int ok = 1;
    for (int j = ndim - 1; j >= 0; --j) {
      const int64_t val = up[j] - ctr[j] * dil[j];
      coords_out[cnt * ndim + j] = val;
      if (val < 0 || val > out_shape[j] - 1) ok = 0;
      off += mult * (transpose ? floordiv64(val - lo[j], dil[j]) : floordiv64(in[j] - val * st[j] + pad[j], dil[j]));
      mult *= ks[j];
    }
    if (ok) offsets[cnt++] = off;
    int d = ndim - 1; /* itertools.product: last counter fastest */
    while (d >= 0 && ++ctr[d] == sz[d]) ctr[d--] = 0;
    if (d < 0) break;
  }
  return cnt;
}

static int cmp_i64(const void* a, const void* b) {
  const int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
  return x < y ? -1 : x > y;
}

/* pairs [K, 2, n] must be filled with -1 and num [K] with 0 by the caller;
 * outids has room for n*K rows of ndim+1 (regular) and gets the input rows
 * for submanifold.  Returns the number of output rows. */
int64_t oracle_indice_pairs(const int32_t* idx, int64_t n, int ndim, const int64_t* out_shape,
                            const int64_t* ks, const int64_t* st, const int64_t* pad, const int64_t* dil,
                            int subm, int transpose, int32_t* pairs, int32_t* num, int32_t* outids) {
  int64_t K = 1, vol = 1;
  for (int i = 0; i < ndim; ++i) {
    K *= ks[i];
    vol *= out_shape[i];
  }
  int64_t maxpts = K;
  int64_t* oc = (int64_t*)malloc(sizeof(int64_t) * (size_t)(maxpts * ndim + 1));
  int64_t* ofs = (int64_t*)malloc(sizeof(int64_t) * (size_t)(maxpts + 1));
  /* flat index of every input (submanifold map), last writer wins */
  int64_t* inflat = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n + 1) * 2);
  int64_t* pend = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n * K + 1) * 3);
  int64_t npend = 0, nout = 0;
  for (int64_t j = 0; j < n; ++j) {
    const int32_t* row = idx + j * (ndim + 1);
    int64_t f = 0;
    for (int d = 0; d < ndim; ++d) f = f * out_shape[d] + row[1 + d];
    inflat[2 * j] = f + vol * row[0];
    inflat[2 * j + 1] = j;
  }
  if (subm) {
    /* sort (flat, j) ascending; a lookup takes the last entry of a run */
    qsort(inflat, (size_t)n, 2 * sizeof(int64_t), cmp_i64);
    for (int64_t j = 0; j < n; ++j)
      for (int d = 0; d <= ndim; ++d) outids[j * (ndim + 1) + d] = idx[j * (ndim + 1) + d];
    nout = n;
  }
  for (int64_t j = 0; j < n; ++j) {
    const int32_t* row = idx + j * (ndim + 1);
    int64_t in[SP_MAXD];
    for (int d = 0; d < ndim; ++d) in[d] = row[1 + d];
    const int cnt = valid_out_pos(in, ndim, ks, st, pad, dil, out_shape, transpose, oc, ofs);
    for (int q = 0; q < cnt; ++q) {
      int64_t f = 0;
      for (int d = 0; d < ndim; ++d) f = f * out_shape[d] + oc[q * ndim + d];
      f += vol * row[0];
      const int64_t off = ofs[q];
      if (subm) {
        /* binary search for the last (flat == f) entry */
        int64_t lo = 0, hi = n;
        while (lo < hi) {
          const int64_t mid = (lo + hi) / 2;
          if (inflat[2 * mid] <= f) lo = mid + 1; else hi = mid;
        }
        if (lo == 0 || inflat[2 * (lo - 1)] != f) continue;
        /* among equal flats the sort put them in j order only if stable; take the max j */
        int64_t best = -1;
        for (int64_t e = lo - 1; e >= 0 && inflat[2 * e] == f; --e)
          if (inflat[2 * e + 1] > best) best = inflat[2 * e + 1];
        const int32_t slot = num[off]++;
        pairs[(off * 2 + 0) * n + slot] = (int32_t)j;
        pairs[(off * 2 + 1) * n + slot] = (int32_t)best;
      } else {
        pend[3 * npend] = off;
        pend[3 * npend + 1] = j;
        pend[3 * npend + 2] = f;
        ++npend;
      }
    }
  }
  if (!subm) {
    int64_t* uniq = (int64_t*)malloc(sizeof(int64_t) * (size_t)(npend + 1));
    for (int64_t i = 0; i < npend; ++i) uniq[i] = pend[3 * i + 2];
    qsort(uniq, (size_t)npend, sizeof(int64_t), cmp_i64);
    for (int64_t i = 0; i < npend; ++i)
      if (i == 0 || uniq[i] != uniq[i - 1]) uniq[nout++] = uniq[i];
    for (int64_t o = 0; o < nout; ++o) {
      int64_t f = uniq[o];
      int32_t* r = outids + o * (ndim + 1);
      r[0] = (int32_t)(f / vol);
      f %= vol;
      for (int d = ndim - 1; d >= 0; --d) {
        r[1 + d] = (int32_t)(f % out_shape[d]);
        f /= out_shape[d];
      }
    }
    for (int64_t i = 0; i < npend; ++i) {
      const int64_t off = pend[3 * i], f = pend[3 * i + 2];
      int64_t lo = 0, hi = nout;
      while (lo < hi) {
        const int64_t mid = (lo + hi) / 2;
        if (uniq[mid] < f) lo = mid + 1; else hi = mid;
      }
      const int32_t slot = num[off]++;
      pairs[(off * 2 + 0) * n + slot] = (int32_t)pend[3 * i + 1];
      pairs[(off * 2 + 1) * n + slot] = (int32_t)lo;
    }
    free(uniq);
  }
  free(oc);
  free(ofs);
  free(inflat);
  free(pend);
  return nout;
}
