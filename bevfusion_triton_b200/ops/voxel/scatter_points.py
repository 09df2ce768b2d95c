"""Per-voxel reduction of point features: ``dynamic_scatter`` and the
``DynamicScatter`` module, drop-ins for ops/voxel/scatter_points.py:8-104.

Both run as ONE call of the ``bfb_b200::dynamic_scatter_forward`` custom op,
whose backward is registered on the op itself (``ops/_registry.py``), so
there is no per-sample loop and no host read of the batch size: batched rows
``(b, x, y, z)`` are keyed and sorted as whole rows, which orders the voxels
sample by sample and, inside a sample, by ``(x, y, z)`` -- the order the
reference builds by reducing every sample separately and padding its batch
index back on.  A row with any negative entry (the batch column included)
belongs to no voxel.

One difference, by design: the reference loops over samples ``0 ..
coors[-1, 0]`` and so drops rows of a larger batch index that come before
the last row; here every sample present is reduced.
"""
from __future__ import annotations

from typing import Sequence

import torch
from torch import nn

from ..._lib import ops
from .voxel_layer import _check_scatter_args, _require_cuda


def dynamic_scatter(feats: torch.Tensor, coors: torch.Tensor, reduce_type: str = 'max',
                    extents: Sequence[int] | None = None):
    """``(voxel_feats, voxel_coors)``: ``feats`` [N, C] reduced ('sum',
    'mean' or 'max') over the points of each distinct ``coors`` row
    ([N, ndim] int32), rows in ascending lexicographic order.  Differentiable
    w.r.t. ``feats``.  ``extents`` (optional, one bound per column with
    ``0 <= coors[:, d] < extents[d]``) lets the keys be packed without a pass
    over the coordinates and a host read."""
    _check_scatter_args(feats, coors, reduce_type)
    if feats.size(0) == 0:
        return feats.clone().detach(), coors.clone().detach()
    _require_cuda(feats, coors)
    ext = None if extents is None else [int(e) for e in extents]
    vf, vc, _, _ = ops().dynamic_scatter_forward(feats.contiguous(), coors.to(torch.int32).contiguous(),
                                                 reduce_type, ext)
    return vf, vc


class DynamicScatter(nn.Module):
    """Scatters the points of a dynamically voxelised cloud into their voxels
    (mean when ``average_points`` else max).  ``coors`` may be [N, 3]
    ``(x, y, z)`` rows of one cloud or [N, 4] ``(b, x, y, z)`` rows of a
    batch; both are reduced in one call.  ``coors_extents`` (optional) bounds
    each coordinate column, see ``dynamic_scatter``."""

    def __init__(self, voxel_size, point_cloud_range, average_points: bool,
                 coors_extents: Sequence[int] | None = None):
        super().__init__()
        self.voxel_size = voxel_size
        self.point_cloud_range = point_cloud_range
        self.average_points = average_points
        self.coors_extents = coors_extents

    def forward_single(self, points: torch.Tensor, coors: torch.Tensor):
        return self.forward(points, coors)

    def forward(self, points: torch.Tensor, coors: torch.Tensor):
        reduce_type = 'mean' if self.average_points else 'max'
        return dynamic_scatter(points, coors, reduce_type, self.coors_extents)

    def __repr__(self):
        return (f'{type(self).__name__}(voxel_size={self.voxel_size}, '
                f'point_cloud_range={self.point_cloud_range}, average_points={self.average_points})')
