"""TEST / BASELINE INFRASTRUCTURE ONLY: the reference's own CPU algorithms for
the hot path, restated for timing on the host cores (bench.py's CPU
baseline and reference arm).  Never on the product path.

* bev_pool: the reference CPU path is ``zeros().index_add_(0, ranks, feats)``
  then a permute to [B, C, D, H, W] (ops/bev_pool/src/bev_pool_triton.py:34-48,
  :219-227); forward + backward go through torch autograd on CPU tensors,
  using every host thread torch is given.
* hard_voxelize: the reference CPU path is a per-point Python loop
  (ops/voxel/src/voxelization_triton.py:466-513, ~9 s per LiDAR sample); it is
  timed through its C restatement in bfb_oracle.c (same algorithm, same
  outputs), one sample per host thread.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import torch

from . import oracle


def bev_pool_cpu(feats: torch.Tensor, coords: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """bev_pool_triton.py:34-48 + :227."""
    x = coords[:, 0].long()
    y = coords[:, 1].long()
    z = coords[:, 2].long()
    b = coords[:, 3].long()
    ranks = ((b * D + z) * H + x) * W + y
    out = feats.new_zeros((B * D * H * W, feats.size(1)))
    out = out.index_add(0, ranks, feats)
    return out.view(B, D, H, W, feats.size(1)).permute(0, 4, 1, 2, 3).contiguous()


def bev_pool_fwd_bwd_cpu(feats: torch.Tensor, coords: torch.Tensor, B, D, H, W, upstream: torch.Tensor):
    x = feats.detach().requires_grad_(True)
    out = bev_pool_cpu(x, coords, B, D, H, W)
    out.backward(upstream)
    return out.detach(), x.grad


def hard_voxelize_many(clouds, voxel_size, coors_range, max_points, max_voxels, threads=None):
    """The sequential first-occurrence algorithm on each cloud, clouds in
    parallel across host threads (ctypes releases the GIL)."""
    threads = threads or os.cpu_count() or 1
    arrs = [np.ascontiguousarray(c.numpy() if isinstance(c, torch.Tensor) else c, dtype=np.float32) for c in clouds]
    with ThreadPoolExecutor(max_workers=threads) as ex:
        return list(ex.map(lambda a: oracle.hard_voxelize(a, voxel_size, coors_range, max_points, max_voxels),
                           arrs))
