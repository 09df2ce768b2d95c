"""TEST INFRASTRUCTURE ONLY: ctypes bindings to the C oracle (bfb_oracle.c).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  Every function cites the reference code it restates (see the
header of bfb_oracle.c for file:line citations).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / 'liboracle.so'

_f32p = np.ctypeslib.ndpointer(np.float32, flags='C_CONTIGUOUS')
_i64p = np.ctypeslib.ndpointer(np.int64, flags='C_CONTIGUOUS')
_i32p = np.ctypeslib.ndpointer(np.int32, flags='C_CONTIGUOUS')
_i64 = ctypes.c_int64


def build() -> Path:
    src = HERE / 'bfb_oracle.c'
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(['make', '-s', '-C', str(HERE), 'liboracle.so'], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        L.oracle_bev_pool_fwd.argtypes = [_f32p, _i64p, _i64, _i64, _i64, _i64, _i64, _i64, _f32p]
        L.oracle_bev_pool_fwd.restype = _i64
        L.oracle_bev_pool_bwd.argtypes = [_f32p, _i64p, _i64, _i64, _i64, _i64, _i64, _i64, _f32p]
        L.oracle_grid_size.argtypes = [_f32p, _f32p, _i64p]
        L.oracle_dynamic_voxelize.argtypes = [_f32p, _i64, _i64, _f32p, _f32p, _i32p]
        L.oracle_hard_voxelize.argtypes = [_f32p, _i64, _i64, _f32p, _f32p, _i64, _i64, _f32p, _i32p,
                                           _i32p, _i64]
        L.oracle_hard_voxelize.restype = _i64
        L.oracle_unique_rows.argtypes = [_i32p, _i64, _i64, _i32p, _i32p, _i32p]
        L.oracle_unique_rows.restype = _i64
        L.oracle_scatter_fwd.argtypes = [_f32p, _i64, _i64, _i32p, _i32p, _i64, ctypes.c_int, _f32p]
        L.oracle_scatter_bwd.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i32p, _i32p, _i64,
                                         ctypes.c_int, _f32p]
        L.oracle_indice_pairs.argtypes = [_i32p, _i64, ctypes.c_int, _i64p, _i64p, _i64p, _i64p, _i64p,
                                          ctypes.c_int, ctypes.c_int, _i32p, _i32p, _i32p]
        L.oracle_indice_pairs.restype = _i64
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def bev_pool(feats, coords, B, D, H, W):
    """[B, C, D, H, W] fp32 sum (ops/bev_pool/src/bev_pool_triton.py:42-48, :227)."""
    f = _f32(feats)
    c = np.ascontiguousarray(np.asarray(coords, dtype=np.int64))
    n, C = f.shape
    out = np.empty((B, C, D, H, W), np.float32)
    bad = lib().oracle_bev_pool_fwd(f, c, n, C, B, D, H, W, out)
    return out, int(bad)


def bev_pool_backward(grad_out, coords, B, D, H, W):
    """[N, C] gather (ops/bev_pool/src/bev_pool_triton.py:102-150)."""
    g = _f32(grad_out)
    c = np.ascontiguousarray(np.asarray(coords, dtype=np.int64))
    n = c.shape[0]
    C = g.shape[1]
    out = np.empty((n, C), np.float32)
    lib().oracle_bev_pool_bwd(g, c, n, C, B, D, H, W, out)
    return out


def grid_size(voxel_size, coors_range):
    g = np.zeros(3, np.int64)
    lib().oracle_grid_size(_f32(voxel_size), _f32(coors_range), g)
    return g


def dynamic_voxelize(points, voxel_size, coors_range):
    """[N, 3] int32 cells, full -1 rows when out of range
    (ops/voxel/src/voxelization_triton.py:328-349)."""
    p = _f32(points)
    out = np.empty((p.shape[0], 3), np.int32)
    lib().oracle_dynamic_voxelize(p, p.shape[0], p.shape[1], _f32(voxel_size), _f32(coors_range), out)
    return out


def hard_voxelize(points, voxel_size, coors_range, max_points, max_voxels):
    """(voxels, coors, num_points, voxel_num) with buffers of max_voxels rows
    (ops/voxel/src/voxelization_triton.py:466-513)."""
    p = _f32(points)
    n, f = p.shape
    cap = max_voxels if max_voxels != -1 else n
    mp = max_points if max_points != -1 else 0
    voxels = np.empty((cap, mp, f), np.float32)
    coors = np.empty((cap, 3), np.int32)
    num = np.empty((cap,), np.int32)
    vn = lib().oracle_hard_voxelize(p, n, f, _f32(voxel_size), _f32(coors_range), max_points,
                                    max_voxels, voxels, coors, num, cap)
    if vn < 0:
        raise MemoryError('oracle hard_voxelize allocation failed')
    return voxels, coors, num, int(vn)


_REDUCE = {'sum': 0, 'none': 0, 'mean': 1, 'max': 2}


def dynamic_scatter(feats, coors, reduce_type):
    """(voxel_feats, voxel_coors, map, counts)
    (ops/voxel/src/scatter_points_triton.py:150-250)."""
    f = _f32(feats)
    c = np.ascontiguousarray(np.asarray(coors, dtype=np.int32))
    n, C = f.shape
    ndim = c.shape[1]
    uc = np.empty((n, ndim), np.int32)
    mp = np.empty((n,), np.int32)
    cnt = np.empty((n,), np.int32)
    m = lib().oracle_unique_rows(c, n, ndim, uc, mp, cnt)
    out = np.empty((m, C), np.float32)
    lib().oracle_scatter_fwd(f, n, C, mp, cnt, m, _REDUCE[reduce_type], out)
    return out, uc[:m].copy(), mp, cnt[:m].copy()


def dynamic_scatter_backward(grad_out, feats, reduced, point2voxel, counts, reduce_type):
    """[N, C] gradient (ops/voxel/src/scatter_points_triton.py:317-345)."""
    g = _f32(grad_out)
    f = _f32(feats)
    r = _f32(reduced)
    n, C = f.shape
    out = np.empty((n, C), np.float32)
    lib().oracle_scatter_bwd(g, f, r, n, C, np.ascontiguousarray(point2voxel, np.int32),
                             np.ascontiguousarray(counts, np.int32), r.shape[0],
                             _REDUCE[reduce_type], out)
    return out


def indice_pairs(indices, out_shape, ksize, stride, padding, dilation, subm, transpose):
    """Rulebook of a sparse convolution (the reference's sequential algorithm
    with the GPU path's output order).  Returns (outids, pairs [K, 2, n],
    num [K]) as int32 arrays."""
    idx = np.ascontiguousarray(np.asarray(indices, dtype=np.int32))
    n, nd = idx.shape[0], idx.shape[1] - 1
    a = [np.ascontiguousarray(np.asarray(v, dtype=np.int64)) for v in (out_shape, ksize, stride, padding, dilation)]
    K = int(np.prod(a[1]))
    pairs = np.full((K, 2, n), -1, dtype=np.int32)
    num = np.zeros((K,), dtype=np.int32)
    outids = np.zeros((max(n * K, 1), nd + 1), dtype=np.int32)
    m = lib().oracle_indice_pairs(idx, n, nd, *a, int(bool(subm)), int(bool(transpose)), pairs, num, outids)
    return outids[:m], pairs, num


# ----------------------------------------------------- sparse convolution
# Restatements in numpy of ops/spconv/src/spconv_triton.py:967-1111 (the
# reference's CPU path: index_select gather, one matmul per rule, index_add_
# scatter, rules in ascending order).  The convolution is accumulated in
# float64 (the checker's reference value); max-pooling in the input dtype, as
# the reference's scatter_reduce / index_add_ on a tensor of that dtype.

def _rules(pairs, num, inverse):
    """(k, in_idx, out_idx) of every rule with pairs, spconv_triton.py:967-978."""
    pairs = np.asarray(pairs)
    num = np.asarray(num)
    si, so = (1, 0) if inverse else (0, 1)
    for k in range(pairs.shape[0]):
        m = int(num[k])
        if m > 0:
            yield k, pairs[k, si, :m].astype(np.int64), pairs[k, so, :m].astype(np.int64)


def indice_conv(features, filters, pairs, num, n_out, inverse=False, bias=None):
    """spconv_triton.py:981-1007 (+ :1010-1032 with ``bias``), float64."""
    x = np.asarray(features, np.float64)
    cin = x.shape[1]
    w = np.asarray(filters, np.float64).reshape(-1, cin, np.asarray(filters).shape[-1])
    out = np.zeros((n_out, w.shape[2]), np.float64)
    for k, i, o in _rules(pairs, num, inverse):
        np.add.at(out, o, x[i] @ w[k])
    if bias is not None:
        out = out + np.asarray(bias, np.float64)
    return out


def indice_conv_backward(features, filters, out_bp, pairs, num, inverse=False):
    """spconv_triton.py:1035-1061, float64: (input_grad, filters_grad)."""
    x = np.asarray(features, np.float64)
    cin = x.shape[1]
    w = np.asarray(filters, np.float64).reshape(-1, cin, np.asarray(filters).shape[-1])
    g = np.asarray(out_bp, np.float64)
    gx = np.zeros_like(x)
    gw = np.zeros_like(w)
    for k, i, o in _rules(pairs, num, inverse):
        gw[k] += x[i].T @ g[o]
        np.add.at(gx, i, g[o] @ w[k].T)
    return gx, gw.reshape(np.asarray(filters).shape)


def indice_maxpool(features, pairs, num, n_out):
    """spconv_triton.py:1064-1082: max into zeros (include_self), exact."""
    x = np.asarray(features)
    out = np.zeros((n_out, x.shape[1]), x.dtype)
    for _, i, o in _rules(pairs, num, False):
        np.maximum.at(out, o, x[i])
    return out


def indice_maxpool_backward(features, out_features, out_bp, pairs, num):
    """spconv_triton.py:1085-1111: index_add_ in the dtype, rules ascending."""
    x = np.asarray(features)
    y = np.asarray(out_features)
    g = np.asarray(out_bp)
    gx = np.zeros_like(x)
    for _, i, o in _rules(pairs, num, False):
        np.add.at(gx, i, np.where(x[i] == y[o], g[o], np.zeros_like(g[o])))
    return gx
