"""``bev_pool`` with the reference signature, on the sm_100a kernels.

Reference: ops/bev_pool/src/bev_pool_triton.py:219-227 (``bev_pool``), input
checks :12-31 (``_check_inputs``: same exception types and messages),
autograd :153-216 (registered on the custom op with
``torch.library.register_autograd``, see ``ops/_registry.py``).  ``feats``
[N, C] (fp32 / fp16 / bf16), ``coords`` [N, 4]
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

from ..._lib import bev_pool_plan_bytes, ops


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


def bev_pool(feats: torch.Tensor, coords: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """Sum-pool point features into a dense [B, C, D, H, W] grid."""
    B, D, H, W = int(B), int(D), int(H), int(W)
    _check_inputs(feats, coords, B, D, H, W)
    _require_cuda(feats, coords)
    return ops().bev_pool_forward(feats, coords, B, D, H, W)[0]


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


def check_plan(plan: torch.Tensor, n: int, B: int, D: int, H: int, W: int) -> None:
    """Raise ValueError unless ``plan`` has the size of a plan for (n, B, D, H,
    W).  A plan reused for another point count or grid (a fixed-rig plan
    handed a short last batch, say) would carve its arrays at the wrong
    offsets; the kernels also compare the geometry stamped in the plan and
    write nothing on a mismatch (``plan_matches`` below reads that back)."""
    if plan.dtype != torch.uint8 or plan.dim() != 1:
        raise ValueError('plan must be the uint8 tensor returned by bev_pool_plan / bev_pool_geometry_plan.')
    need = bev_pool_plan_bytes(int(n), int(B), int(D), int(H), int(W))
    if plan.numel() != need:
        raise ValueError(f'bev_pool plan was built for another geometry: it holds {plan.numel()} bytes, '
                         f'(n={n}, B={B}, D={D}, H={H}, W={W}) needs {need}.')


def plan_matches(plan: torch.Tensor, n: int, B: int, D: int, H: int, W: int) -> bool:
    """True when ``plan`` was built for (n, B, D, H, W) and no call has been
    handed it with another geometry since (reads the plan header: synchronises
    the stream)."""
    return bool(ops().bev_pool_plan_check(plan, int(n), int(B), int(D), int(H), int(W)))


def bev_pool_planned(feats: torch.Tensor, plan: torch.Tensor, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """``bev_pool`` with a plan from ``bev_pool_plan`` (same coords, same N)."""
    if feats.dim() != 2:
        raise ValueError('feats must have shape [N, C].')
    if feats.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise TypeError('feats must have dtype torch.float16, torch.float32, or torch.bfloat16.')
    check_plan(plan, feats.size(0), B, D, H, W)
    _require_cuda(feats, plan)
    return ops().bev_pool_forward_planned(feats, plan, int(B), int(D), int(H), int(W))


def plan_cells(plan: torch.Tensor, n: int, B: int, D: int, H: int, W: int) -> torch.Tensor:
    """[n] int64: the cell rank ((b*D + z)*H + x)*W + y a plan gave every
    point (input order), -1 for points it dropped."""
    return ops().bev_pool_plan_cells(plan, int(n), int(B), int(D), int(H), int(W))


def invalid_count(plan: torch.Tensor) -> int:
    """Points a plan dropped as out of range (synchronises the stream)."""
    return int(ops().bev_pool_invalid_count(plan))


def bev_pool_depth_context(depth: torch.Tensor, context: torch.Tensor, coords: torch.Tensor | None,
                           B: int, D: int, H: int, W: int, plan: torch.Tensor | None = None) -> torch.Tensor:
    """The LSS camera branch's pooling without a feature tensor.

    Equals ``bev_pool(feats[kept], coords[kept], B, D, H, W)`` with
    ``feats = rearrange(depth.unsqueeze(2) * context.unsqueeze(3), 'b n c d h w -> (b n d h w) c')``
    (models/vtransforms/depth_lss.py:91-94, base.py:136-160), forward bit for
    bit.  ``depth`` [B, N, D_bins, fH, fW] (softmaxed) or [cams, D_bins, fH,
    fW]; ``context`` [B, N, C, fH, fW] or [cams, C, fH, fW], fp32;
    ``coords`` one (x, y, z, b) row per frustum point in (b, n, d, h, w)
    order, unfiltered (points outside the grid are dropped).  With ``plan``
    (from ``bev_pool_geometry_plan`` or ``bev_pool_plan`` over those frustum
    points) ``coords`` is not needed and may be None.  Differentiable w.r.t.
    depth and context.  C must be a multiple of 4, at most 128.
    """
    if depth.dim() == 5:
        depth = depth.flatten(0, 1)
    if context.dim() == 5:
        context = context.flatten(0, 1)
    if depth.dim() != 4 or context.dim() != 4:
        raise ValueError('depth and context must be 4-D or 5-D tensors.')
    if plan is None:
        if coords is None or coords.dim() != 2 or coords.size(-1) != 4:
            raise ValueError('coords must have shape [N, 4].')
        if coords.dtype not in (torch.int32, torch.int64):
            raise TypeError('coords must have dtype torch.int32 or torch.int64.')
    if depth.dtype != torch.float32 or context.dtype != torch.float32:
        raise TypeError('depth and context must have dtype torch.float32.')
    if min(B, D, H, W) <= 0:
        raise ValueError('B, D, H, W must be positive integers.')
    if plan is not None:
        check_plan(plan, depth.size(0) * depth.size(1) * depth.size(2) * depth.size(3), B, D, H, W)
    _require_cuda(depth, context, *((coords,) if plan is None else (plan,)))
    B, D, H, W = int(B), int(D), int(H), int(W)
    if plan is None:
        return ops().bev_pool_dc_forward(depth, context, coords, B, D, H, W)[0]
    return ops().bev_pool_dc_forward_planned(depth, context, plan, B, D, H, W)[0]


def bev_grid(xbound, ybound, zbound):
    """Lower grid edge ``bx - dx / 2``, cell size ``dx`` (fp32 values, as the
    reference forms them) and cell counts ``nx`` (x, y, z); gen_dx_bx
    (models/vtransforms/base.py:19-23) and the offset of base.py:138."""
    rows = [xbound, ybound, zbound]
    dx = torch.tensor([r[2] for r in rows], dtype=torch.float32)
    bx = torch.tensor([r[0] + r[2] / 2.0 for r in rows], dtype=torch.float32)
    lower = bx - dx / 2.0
    nx = [int((r[1] - r[0]) / r[2]) for r in rows]
    return lower.tolist(), dx.tolist(), nx


def bev_pool_geometry_plan(frustum: torch.Tensor, camera2lidar_rots: torch.Tensor, camera2lidar_trans: torch.Tensor,
                           intrins: torch.Tensor, post_rots: torch.Tensor, post_trans: torch.Tensor,
                           xbound, ybound, zbound, extra_rots: torch.Tensor | None = None,
                           extra_trans: torch.Tensor | None = None):
    """bev_pool plan straight from the camera parameters (no coords tensor).

    Fuses ``BaseTransform.get_geometry`` (models/vtransforms/base.py:82-126)
    with the quantise + in-grid filter of ``BaseTransform.bev_pool``
    (base.py:131-158): ``frustum`` [D_bins, fH, fW, 3] (``create_frustum``),
    ``camera2lidar_rots``, ``intrins``, ``post_rots`` [B, N, 3, 3],
    ``camera2lidar_trans``, ``post_trans`` [B, N, 3], optional
    ``extra_rots`` [B, 3, 3] / ``extra_trans`` [B, 3] (lidar augmentation).
    ``camera2lidar_rots @ intrins^-1`` is formed with ``torch.linalg.solve`` as
    the reference does; the per-point 3x3 products run in the keys kernel
    with the association of torch's CUDA matmul for these shapes (equal on
    all but a few values in a million), so a point within rounding of a cell
    edge may still land in the neighbouring cell.

    Returns ``(plan, (B, D, H, W))``: the plan covers every frustum point in
    (b, n, d, h, w) order and drops the ones outside the grid, so
    ``bev_pool_planned(x.flatten(0, 4), plan, B, D, H, W)`` pools the
    UNFILTERED features ``x`` [B, N, D_bins, fH, fW, C] (no boolean-mask
    gather) and ``bev_pool_depth_context(depth, context, None, B, D, H, W,
    plan=plan)`` pools depth x context.
    """
    for name, t in (('camera2lidar_rots', camera2lidar_rots), ('intrins', intrins), ('post_rots', post_rots)):
        if t.dim() != 4 or t.shape[-2:] != (3, 3):
            raise ValueError(f'{name} must have shape [B, N, 3, 3].')
    if frustum.dim() != 4 or frustum.size(-1) != 3:
        raise ValueError('frustum must have shape [D, fH, fW, 3].')
    _require_cuda(frustum, camera2lidar_rots, camera2lidar_trans, intrins, post_rots, post_trans)
    # the reference's torch.linalg.solve without its host-synchronising error
    # check (same factorisation and result)
    combine = torch.linalg.solve_ex(intrins.float().transpose(-1, -2),
                                    camera2lidar_rots.float().transpose(-1, -2))[0].transpose(-1, -2)
    lower, dx, nx = bev_grid(xbound, ybound, zbound)
    B = camera2lidar_rots.size(0)
    D, H, W = nx[2], nx[0], nx[1]
    plan = ops().bev_pool_geometry_plan(frustum, post_rots, post_trans, combine, camera2lidar_trans,
                                        extra_rots, extra_trans, lower, dx, D, H, W)
    return plan, (B, D, H, W)
