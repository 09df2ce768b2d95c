"""``bev_pool`` with the reference signature, on the sm_100a kernels.

Reference: ops/bev_pool/src/bev_pool_triton.py:219-227 (``bev_pool``), input
checks :12-31 (``_check_inputs``: same exception types and messages),
autograd :153-216.  ``feats`` [N, C] (fp32 / fp16 / bf16), ``coords`` [N, 4]
int32 / int64 with columns (x, y, z, b); returns [B, C, D, H, W] in the
dtype of ``feats``, differentiable w.r.t. ``feats``.

Differences from the reference, by design:
* no CPU path: CPU tensors raise (the reference falls back to
  ``index_add_``);
* fp16 / bf16 inputs are summed in fp32 and rounded once (the reference's
  Triton atomics accumulate in the storage type);
* points whose coordinates fall outside the grid are dropped (and counted,
  see ``invalid_count``) instead of raising (CPU) or writing out of bounds
  (Triton).
"""
from __future__ import annotations

import torch

from ..._lib import ops


def _check_inputs(feats: torch.Tensor, coords: torch.Tensor, B: int, D: int, H: int, W: int) -> None:
    """bev_pool_triton.py:12-31."""
    if feats.dim() != 2:
        raise ValueError('feats must have shape [N, C].')
    if coords.dim() != 2 or coords.size(-1) != 4:
        raise ValueError('coords must have shape [N, 4].')
    if feats.size(0) != coords.size(0):
        raise ValueError('feats and coords must have the same number of points.')
    if coords.dtype not in (torch.int32, torch.int64):
        raise TypeError('coords must have dtype torch.int32 or torch.int64.')
    if feats.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise TypeError('feats must have dtype torch.float16, torch.float32, or torch.bfloat16.')
    if min(B, D, H, W) <= 0:
        raise ValueError('B, D, H, W must be positive integers.')


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError('bevfusion_triton_b200 ops run on CUDA tensors only (no CPU fallback)')


class _BevPoolFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, feats, coords, B, D, H, W):
        out, plan = ops().bev_pool_forward(feats, coords, B, D, H, W)
        ctx.save_for_backward(plan)
        ctx.shape = (feats.size(0), B, D, H, W)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (plan,) = ctx.saved_tensors
        n, B, D, H, W = ctx.shape
        gfeat = ops().bev_pool_backward(grad_out, plan, n, B, D, H, W)
        return gfeat, None, None, None, None, None


class _BevPoolPlannedFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, feats, plan, B, D, H, W):
        ctx.save_for_backward(plan)
        ctx.shape = (feats.size(0), B, D, H, W)
        return ops().bev_pool_forward_planned(feats, plan, B, D, H, W)

    @staticmethod
    def backward(ctx, grad_out):
        (plan,) = ctx.saved_tensors
        n, B, D, H, W = ctx.shape
        return ops().bev_pool_backward(grad_out, plan, n, B, D, H, W), None, None, None, None, None


def bev_pool(feats: torch.Tensor, coords: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """Sum-pool point features into a dense [B, C, D, H, W] grid."""
    B, D, H, W = int(B), int(D), int(H), int(W)
    _check_inputs(feats, coords, B, D, H, W)
    _require_cuda(feats, coords)
    return _BevPoolFunction.apply(feats, coords, B, D, H, W)


def bev_pool_plan(coords: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """Sort + work plan for fixed ``coords`` (e.g. a fixed camera rig), reusable
    across calls with ``bev_pool_planned``.  Returns an opaque uint8 tensor."""
    B, D, H, W = int(B), int(D), int(H), int(W)
    if coords.dim() != 2 or coords.size(-1) != 4:
        raise ValueError('coords must have shape [N, 4].')
    if coords.dtype not in (torch.int32, torch.int64):
        raise TypeError('coords must have dtype torch.int32 or torch.int64.')
    if min(B, D, H, W) <= 0:
        raise ValueError('B, D, H, W must be positive integers.')
    _require_cuda(coords)
    return ops().bev_pool_plan(coords, B, D, H, W)


def bev_pool_planned(feats: torch.Tensor, plan: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """``bev_pool`` with a plan from ``bev_pool_plan`` (same coords, same N)."""
    if feats.dim() != 2:
        raise ValueError('feats must have shape [N, C].')
    if feats.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise TypeError('feats must have dtype torch.float16, torch.float32, or torch.bfloat16.')
    _require_cuda(feats, plan)
    return _BevPoolPlannedFunction.apply(feats, plan, int(B), int(D), int(H), int(W))


def invalid_count(plan: torch.Tensor) -> int:
    """Points a plan dropped as out of range (synchronises the stream)."""
    return int(ops().bev_pool_invalid_count(plan))
