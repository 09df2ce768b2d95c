"""``Voxelization`` / ``voxelization`` with the reference signatures
(ops/voxel/voxelize.py:10-148) on the sm_100a kernels."""
from __future__ import annotations

import torch
from torch import nn
from torch.autograd import Function
from torch.nn.modules.utils import _pair

from ..._lib import ops
from .voxel_layer import _require_cuda, _voxel_meta, dynamic_voxelize, hard_voxelize_batch


class _Voxelization(Function):
    @staticmethod
    def forward(ctx, points, voxel_size, coors_range, max_points=35, max_voxels=20000, deterministic=True):
        """voxelize.py:12-71: max_points or max_voxels == -1 selects dynamic
        voxelisation (coords only); otherwise returns (voxels, coors,
        num_points) sliced to voxel_num.  Rows past voxel_num are sliced off,
        so the buffers are allocated uninitialised and only the kept rows are
        written."""
        if max_points == -1 or max_voxels == -1:
            coors = points.new_zeros(size=(points.size(0), 3), dtype=torch.int)
            dynamic_voxelize(points, coors, voxel_size, coors_range, 3)
            return coors
        voxel_size, coors_range, _ = _voxel_meta(voxel_size, coors_range, 3)
        _require_cuda(points)
        voxels = points.new_empty(size=(max_voxels, max_points, points.size(1)))
        coors = points.new_empty(size=(max_voxels, 3), dtype=torch.int)
        num_points_per_voxel = points.new_empty(size=(max_voxels,), dtype=torch.int)
        voxel_num = ops().hard_voxelize(points, voxels, coors, num_points_per_voxel, voxel_size, coors_range,
                                        int(max_points), int(max_voxels), False)
        return voxels[:voxel_num], coors[:voxel_num], num_points_per_voxel[:voxel_num]


voxelization = _Voxelization.apply


class Voxelization(nn.Module):
    """voxelize.py:77-148."""

    def __init__(self, voxel_size, point_cloud_range, max_num_points, max_voxels=20000, deterministic=True):
        super().__init__()
        self.voxel_size = voxel_size
        self.point_cloud_range = point_cloud_range
        self.max_num_points = max_num_points
        if isinstance(max_voxels, tuple):
            self.max_voxels = max_voxels
        else:
            self.max_voxels = _pair(max_voxels)
        self.deterministic = deterministic
        point_cloud_range = torch.tensor(point_cloud_range, dtype=torch.float32)
        voxel_size = torch.tensor(voxel_size, dtype=torch.float32)
        grid_size = (point_cloud_range[3:] - point_cloud_range[:3]) / voxel_size
        grid_size = torch.round(grid_size).long()
        input_feat_shape = grid_size[:2]
        self.grid_size = grid_size
        self.pcd_shape = [*input_feat_shape, 1]

    def forward(self, input):
        max_voxels = self.max_voxels[0] if self.training else self.max_voxels[1]
        return voxelization(input, self.voxel_size, self.point_cloud_range, self.max_num_points, max_voxels,
                            self.deterministic)

    def __repr__(self):
        return (f'{self.__class__.__name__}(voxel_size={self.voxel_size}, '
                f'point_cloud_range={self.point_cloud_range}, max_num_points={self.max_num_points}, '
                f'max_voxels={self.max_voxels}, deterministic={self.deterministic})')


def voxelize_batch(points_list, voxel_size, point_cloud_range, max_num_points, max_voxels, reduce_mean=True):
    """Batched replacement of ``BEVFusion.voxelize`` (models/fusion_models/
    bevfusion.py:269-296): one set of launches for all samples instead of a
    Python loop over them.  Returns ``(feats, coords, sizes)`` as that method
    does: feats [M, F] (mean over each voxel's points when ``reduce_mean``,
    else [M, P, F]), coords [M, 4] int32 = (sample, x, y, z), sizes [M].

    With ``reduce_mean`` the packing and the mean are one epilogue launch
    (``bfb_voxelize_mean_epilogue``); the only host read is the voxel total M
    that sizes the returned tensors."""
    pts = torch.cat([p for p in points_list], 0) if len(points_list) > 1 else points_list[0]
    offs = [0]
    for p in points_list:
        offs.append(offs[-1] + int(p.size(0)))
    voxels, coors, num, vn = hard_voxelize_batch(pts, offs, voxel_size, point_cloud_range, max_num_points,
                                                 max_voxels)
    feats, coords, sizes, total = ops().voxelize_mean_epilogue(voxels, coors, num, vn)
    m = int(total.item())
    if reduce_mean:
        return feats[:m], coords[:m], sizes[:m]
    # the unreduced [M, P, F] rows: gather the packed rows (no per-sample loop)
    rows = coords[:m, 0].long() * voxels.size(1) + torch.arange(m, device=pts.device) - \
        torch.repeat_interleave(torch.cumsum(vn.long(), 0) - vn.long(), vn.long(), output_size=m)
    return voxels.flatten(0, 1)[rows], coords[:m], sizes[:m]
