"""Low-level voxel ops with the reference signatures
(ops/voxel/voxel_layer.py:27-48, ops/voxel/src/voxelization_triton.py:428-463,
:674-710, ops/voxel/src/scatter_points_triton.py:253-424), on the sm_100a
kernels.  CUDA tensors only; there is no CPU path.
"""
from __future__ import annotations

from typing import Sequence

import torch

from ..._lib import ops

__all__ = ['hard_voxelize', 'dynamic_voxelize', 'hard_voxelize_batch',
           'dynamic_point_to_voxel_forward', 'dynamic_point_to_voxel_backward']


def _voxel_meta(voxel_size: Sequence[float], coors_range: Sequence[float], ndim: int = 3):
    """Argument checks and grid size of voxelization_triton.py:23-39."""
    voxel_size = [float(v) for v in voxel_size]
    coors_range = [float(v) for v in coors_range]
    if ndim != 3:
        raise NotImplementedError('Only 3D voxelization is supported')
    if len(voxel_size) != ndim:
        raise ValueError(f'voxel_size must have length {ndim}')
    if len(coors_range) != ndim * 2:
        raise ValueError(f'coors_range must have length {ndim * 2}')
    grid_size = [int(round((coors_range[3 + i] - coors_range[i]) / voxel_size[i])) for i in range(3)]
    return voxel_size, coors_range, grid_size


def _require_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError('bevfusion_triton_b200 ops run on CUDA tensors only (no CPU fallback)')


def dynamic_voxelize(points: torch.Tensor, coors: torch.Tensor, voxel_size: Sequence[float],
                     coors_range: Sequence[float], NDim: int = 3) -> None:
    """coors[i] = voxel cell of points[i] or (-1, -1, -1); writes in place.

    Out-of-range rows are -1 in all three columns (the reference CPU path;
    its GPU paths leave some columns untouched)."""
    voxel_size, coors_range, _ = _voxel_meta(voxel_size, coors_range, NDim)
    _require_cuda(points, coors)
    if points.size(0) == 0:
        return
    ops().dynamic_voxelize(points, coors, voxel_size, coors_range)


def hard_voxelize(points: torch.Tensor, voxels: torch.Tensor, coors: torch.Tensor,
                  num_points_per_voxel: torch.Tensor, voxel_size: Sequence[float],
                  coors_range: Sequence[float], max_points: int, max_voxels: int, NDim: int = 3,
                  deterministic: bool = True) -> int:
    """First-occurrence hard voxelisation into caller buffers; returns voxel_num.

    Matches the reference CPU algorithm (voxelization_triton.py:466-513) bit
    for bit: voxels are numbered by their first in-range point, each keeps its
    first ``max_points`` points in input order, all three buffers are
    zero-filled beyond what is written.  ``deterministic=False`` is accepted
    and served by the same deterministic kernel (the reference's
    non-deterministic path leaves the order unspecified)."""
    voxel_size, coors_range, _ = _voxel_meta(voxel_size, coors_range, NDim)
    _require_cuda(points, voxels, coors, num_points_per_voxel)
    del deterministic
    return int(ops().hard_voxelize(points, voxels, coors, num_points_per_voxel, voxel_size, coors_range,
                                   int(max_points), int(max_voxels), True))


def hard_voxelize_batch(points: torch.Tensor, offsets: Sequence[int], voxel_size: Sequence[float],
                        coors_range: Sequence[float], max_points: int, max_voxels: int,
                        zero_tail: bool = False):
    """Hard-voxelise ``len(offsets) - 1`` samples in one set of launches.

    Sample ``s`` owns ``points[offsets[s]:offsets[s+1]]``.  Returns
    ``(voxels [B, max_voxels, max_points, F], coors [B, max_voxels, 3],
    num_points [B, max_voxels], voxel_num [B])`` on the device; rows past a
    sample's ``voxel_num`` are left unwritten unless ``zero_tail``.  No host
    copy or synchronisation: the sample offsets travel as kernel parameters,
    so the call can be captured into a CUDA graph."""
    voxel_size, coors_range, _ = _voxel_meta(voxel_size, coors_range, 3)
    _require_cuda(points)
    offsets = [int(o) for o in offsets]
    B = len(offsets) - 1
    n, f = points.shape
    P = n if max_points == -1 else int(max_points)
    MV = n if max_voxels == -1 else int(max_voxels)
    voxels = points.new_empty((B, MV, P, f))
    coors = points.new_empty((B, MV, 3), dtype=torch.int32)
    num = points.new_empty((B, MV), dtype=torch.int32)
    vn = points.new_empty((B,), dtype=torch.int32)
    ops().hard_voxelize_batch(points, offsets, voxels, coors, num, vn, voxel_size, coors_range,
                              int(max_points), int(max_voxels), bool(zero_tail))
    return voxels, coors, num, vn


_REDUCE_MODE = {'none', 'mean', 'sum', 'max'}


def _check_scatter_args(feats: torch.Tensor, coors: torch.Tensor, reduce_type: str) -> None:
    """The argument checks of scatter_points_triton.py:258-265 (same
    exception types)."""
    if reduce_type not in _REDUCE_MODE:
        raise ValueError(f'Unsupported reduce_type: {reduce_type}')
    if feats.dim() != 2:
        raise AssertionError('feats must have shape [N, C]')
    if coors.dim() != 2:
        raise AssertionError('coors must have shape [N, ndim]')
    if feats.size(0) != coors.size(0):
        raise AssertionError('feats and coors must have the same first dimension')


def dynamic_point_to_voxel_forward(feats: torch.Tensor, coors: torch.Tensor, reduce_type: str,
                                   extents: Sequence[int] | None = None):
    """(voxel_feats, voxel_coors, point2voxel_map, voxel_points_count);
    scatter_points_triton.py:253-314.  ``extents`` (optional, not in the
    reference signature): one bound per coordinate column, which saves the
    kernel a pass over the coordinates and a host read."""
    _check_scatter_args(feats, coors, reduce_type)
    if feats.size(0) == 0:
        return (feats.clone().detach(), coors.clone().detach(),
                coors.new_empty((0,), dtype=torch.int32), coors.new_empty((0,), dtype=torch.int32))
    _require_cuda(feats, coors)
    ext = None if extents is None else [int(e) for e in extents]
    vf, vc, mp, cnt = ops().dynamic_scatter_forward(feats, coors.to(torch.int32), reduce_type, ext)
    return vf, vc, mp, cnt


def dynamic_point_to_voxel_backward(grad_feats: torch.Tensor, grad_reduced_feats: torch.Tensor,
                                    feats: torch.Tensor, reduced_feats: torch.Tensor,
                                    coors_map: torch.Tensor, reduce_count: torch.Tensor,
                                    reduce_type: str) -> None:
    """Writes grad_feats in place; scatter_points_triton.py:348-424."""
    if reduce_type not in _REDUCE_MODE:
        raise ValueError(f'Unsupported reduce_type: {reduce_type}')
    _require_cuda(grad_feats, grad_reduced_feats, feats, reduced_feats, coors_map, reduce_count)
    ops().dynamic_scatter_backward(grad_feats, grad_reduced_feats, feats, reduced_feats, coors_map,
                                   reduce_count, reduce_type)
