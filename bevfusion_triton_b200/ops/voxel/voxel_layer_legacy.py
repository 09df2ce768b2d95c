"""Drop-in for the legacy import path ops/voxel/voxel_layer_legacy.py:60-90
(``hard_voxelize``, ``dynamic_voxelize``, ``dynamic_point_to_voxel_forward``,
``dynamic_point_to_voxel_backward`` and the ``voxel_layer_ext`` namespace of
the compiled extension they wrapped).

The same positional signatures as the extension's functions
(ops/voxel/csrc/voxelization.cpp:7-10); they run this library's sm_100a ops
(``ops.voxel.voxel_layer``), whose results follow the reference's CPU
algorithms (first-occurrence voxel order, ascending point order inside a
voxel).  The legacy CPU voxeliser's indexing at non-cubic grids is not
reproduced.
"""
from __future__ import annotations

from types import SimpleNamespace

from .voxel_layer import (dynamic_point_to_voxel_backward, dynamic_point_to_voxel_forward, dynamic_voxelize,
                          hard_voxelize)

voxel_layer_ext = SimpleNamespace(hard_voxelize=hard_voxelize, dynamic_voxelize=dynamic_voxelize,
                                  dynamic_point_to_voxel_forward=dynamic_point_to_voxel_forward,
                                  dynamic_point_to_voxel_backward=dynamic_point_to_voxel_backward)

__all__ = ['dynamic_point_to_voxel_backward', 'dynamic_point_to_voxel_forward', 'dynamic_voxelize', 'hard_voxelize',
           'voxel_layer_ext']
