"""B200-native (sm_100a) grid scatter-reduce hot path of BEVFusion.

Drop-in replacements for the reference's operator modules:

* ``bevfusion_triton_b200.ops.bev_pool.bev_pool``        <- ``ops.bev_pool.bev_pool``
* ``bevfusion_triton_b200.ops.voxel.{Voxelization, voxelization,
  DynamicScatter, dynamic_scatter}``                      <- ``ops.voxel.*``
* ``bevfusion_triton_b200.ops.voxel.voxel_layer.{hard_voxelize,
  dynamic_voxelize, dynamic_point_to_voxel_forward,
  dynamic_point_to_voxel_backward}``                      <- ``ops.voxel.voxel_layer.*``

All kernels live in ``libbfb_b200.so`` (C ABI, include/bfb_b200.h); torch
custom ops in ``_bfb_torch.so`` wrap it.  There is no CPU or Triton path.
"""
from ._lib import load_native, native_paths  # noqa: F401

__all__ = ['load_native', 'native_paths']
