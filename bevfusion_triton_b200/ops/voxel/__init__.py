from .scatter_points import DynamicScatter, dynamic_scatter
from .voxelize import Voxelization, voxelization, voxelize_batch

__all__ = ['Voxelization', 'voxelization', 'dynamic_scatter', 'DynamicScatter', 'voxelize_batch']
