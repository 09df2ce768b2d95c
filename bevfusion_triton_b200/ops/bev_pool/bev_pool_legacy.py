"""Drop-in for the legacy import path ops/bev_pool/bev_pool_legacy.py:99-108
(``bev_pool(feats, coords, B, D, H, W)``: the sort + interval-sum pooling
the Triton op replaced).

Same inputs and output ([B, C, D, H, W], a sum over each cell's points).
The legacy code argsorts a rank with an unstable sort, so its fp32 sums come
in an order that depends on the run; this runs the same sm_100a op as
``ops.bev_pool.bev_pool`` (ascending point order per cell, the reference CPU
path's ``index_add_`` order), which the legacy result equals within fp32
rounding.  Like the legacy function it asserts that feats and coords have
the same length; it takes fp16 / bf16 features too (the legacy kernel is
fp32 only).
"""
from __future__ import annotations

import torch

from .bev_pool import bev_pool as _bev_pool


def bev_pool(feats: torch.Tensor, coords: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    assert feats.shape[0] == coords.shape[0]
    return _bev_pool(feats, coords, B, D, H, W)


__all__ = ['bev_pool']
