from .scatter_points import DynamicScatter, dynamic_scatter
from .voxelize import Voxelization, voxelization, voxelize_batch

# the reference package's export list (ops/voxel/__init__.py); voxelize_batch,
# which has no reference counterpart, is importable from here too
__all__ = ['Voxelization', 'voxelization', 'dynamic_scatter', 'DynamicScatter']
