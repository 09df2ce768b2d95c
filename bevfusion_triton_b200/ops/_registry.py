"""Fake (meta) kernels and autograd formulas of the ``torch.ops.bfb_b200``
custom ops.

The ops themselves are defined and implemented (CUDA only) in
``csrc/torch_ops.cpp``.  This module gives each one a shape function so that
``torch.compile`` / ``torch.export`` can trace them without running a kernel,
and registers the backward of the differentiable ones
(``torch.library.register_autograd``), so the public functions need no
``torch.autograd.Function`` of their own:

* ``bev_pool_forward`` / ``bev_pool_forward_planned`` -> ``bev_pool_backward``
  (the reference's autograd pair, ops/bev_pool/src/bev_pool_triton.py:153-216);
* ``bev_pool_dc_forward`` / ``bev_pool_dc_forward_planned`` -> ``bev_pool_dc_backward``;
* ``dynamic_scatter_forward`` -> ``dynamic_scatter_backward``
  (ops/voxel/scatter_points.py:8-50, scatter_points_triton.py:348-424);
* ``indice_conv`` -> ``indice_conv_backward`` and ``indice_maxpool`` ->
  ``indice_maxpool_backward`` (ops/spconv/functional.py:21-110).

Workspace sizes in the fake kernels come from the library's host-only size
queries, so a traced plan tensor has exactly the size the real op returns.
Data-dependent sizes (voxel and output-site counts) are unbacked symbolic
sizes.
"""
from __future__ import annotations

import ctypes

import torch

from .._lib import load_native

_done = False


def _sizes(fn, *args) -> list[int]:
    """Call a C-ABI size query taking int64 arguments and size_t* outputs."""
    lib = load_native()
    outs = [ctypes.c_size_t(0) for _ in range(fn[1])]
    st = getattr(lib, fn[0])(*[ctypes.c_int64(int(a)) for a in args], *[ctypes.byref(o) for o in outs])
    if st != 0:
        raise ValueError(f'{fn[0]} refused the sizes {args} (status {st})')
    return [o.value for o in outs]


def _concrete(*vals) -> bool:
    return all(isinstance(v, int) for v in vals)


def _plan_numel(n, B, D, H, W):
    if not _concrete(n, B, D, H, W):
        return torch.library.get_ctx().new_dynamic_size()
    return _sizes(('bfb_bev_pool_workspace_sizes', 2), n, 1, B, D, H, W)[0]


def _dc_numels(depth, context, B, D, H, W):
    cams, nd, fh, fw = depth.shape
    c = context.size(1)
    if not _concrete(cams, nd, fh, fw, c, B, D, H, W):
        ctx = torch.library.get_ctx()
        return ctx.new_dynamic_size(), ctx.new_dynamic_size()
    plan, _, aux, _ = _sizes(('bfb_bev_pool_dc_workspace_sizes', 4), cams, nd, fh, fw, c, B, D, H, W)
    return plan, aux


def _register_fakes() -> None:
    lib = 'bfb_b200::'
    reg = torch.library.register_fake

    @reg(lib + 'bev_pool_forward')
    def _(feats, coords, B, D, H, W):
        out = feats.new_empty((B, feats.size(1), D, H, W))
        return out, feats.new_empty((_plan_numel(feats.size(0), B, D, H, W),), dtype=torch.uint8)

    @reg(lib + 'bev_pool_plan')
    def _(coords, B, D, H, W):
        return coords.new_empty((_plan_numel(coords.size(0), B, D, H, W),), dtype=torch.uint8)

    @reg(lib + 'bev_pool_forward_planned')
    def _(feats, plan, B, D, H, W):
        return feats.new_empty((B, feats.size(1), D, H, W))

    @reg(lib + 'bev_pool_backward')
    def _(grad_out, plan, n, B, D, H, W):
        return grad_out.new_empty((n, grad_out.size(1)))

    @reg(lib + 'bev_pool_invalid_count')
    def _(plan):
        return torch.library.get_ctx().new_dynamic_size()

    @reg(lib + 'bev_pool_plan_check')
    def _(plan, n, B, D, H, W):
        return True  # a data-dependent check: traced as passing

    @reg(lib + 'bev_pool_plan_cells')
    def _(plan, n, B, D, H, W):
        return plan.new_empty((n,), dtype=torch.int64)

    @reg(lib + 'bev_pool_dc_forward')
    def _(depth, context, coords, B, D, H, W):
        _, aux = _dc_numels(depth, context, B, D, H, W)
        return depth.new_empty((B, context.size(1), D, H, W)), depth.new_empty((aux,), dtype=torch.uint8)

    @reg(lib + 'bev_pool_dc_forward_planned')
    def _(depth, context, plan, B, D, H, W):
        _, aux = _dc_numels(depth, context, B, D, H, W)
        return depth.new_empty((B, context.size(1), D, H, W)), depth.new_empty((aux,), dtype=torch.uint8)

    @reg(lib + 'bev_pool_geometry_plan')
    def _(frustum, post_rots, post_trans, combine, trans, extra_rots, extra_trans, lower, dx, D, H, W):
        B, ncam = post_rots.shape[:2]
        nd, fh, fw = frustum.shape[:3]
        return frustum.new_empty((_plan_numel(B * ncam * nd * fh * fw, B, D, H, W),), dtype=torch.uint8)

    @reg(lib + 'bev_pool_dc_backward')
    def _(grad_out, depth, coords, aux, C, B, D, H, W):
        cams, _, fh, fw = depth.shape
        return torch.empty_like(depth), depth.new_empty((cams, C, fh, fw))

    @reg(lib + 'dynamic_voxelize')
    def _(points, coors, voxel_size, coors_range):
        return None

    @reg(lib + 'hard_voxelize')
    def _(points, voxels, coors, num_points, voxel_size, coors_range, max_points, max_voxels, zero_tail):
        return torch.library.get_ctx().new_dynamic_size()

    @reg(lib + 'hard_voxelize_batch')
    def _(points, offsets, voxels, coors, num_points, voxel_num, voxel_size, coors_range, max_points, max_voxels,
          zero_tail):
        return None

    @reg(lib + 'voxelize_mean_epilogue')
    def _(voxels, coors, num_points, voxel_num):
        B, MV, _, F = voxels.shape
        return (voxels.new_empty((B * MV, F)), coors.new_empty((B * MV, 4)), coors.new_empty((B * MV,)),
                coors.new_empty((1,)))

    @reg(lib + 'get_indice_pairs')
    def _(indices, batch, out_shape, ksize, stride, padding, dilation, subm, transpose):
        n, k1 = indices.shape
        K = 1
        for k in ksize:
            K *= k
        pairs = indices.new_empty((K, 2, n))
        num = indices.new_empty((K,))
        if subm:
            return indices.new_empty((n, k1)), pairs, num
        return indices.new_empty((torch.library.get_ctx().new_dynamic_size(), k1)), pairs, num

    @reg(lib + 'dynamic_scatter_forward')
    def _(feats, coors, reduce, extents=None):
        m = torch.library.get_ctx().new_dynamic_size()
        n, ndim = coors.shape
        return (feats.new_empty((m, feats.size(1))), coors.new_empty((m, ndim), dtype=torch.int32),
                coors.new_empty((n,), dtype=torch.int32), coors.new_empty((m,), dtype=torch.int32))

    @reg(lib + 'dynamic_scatter_backward')
    def _(grad_feats, grad_out, feats, reduced, map, counts, reduce):
        return None

    @reg(lib + 'indice_conv')
    def _(features, filters, indice_pairs, indice_pair_num, num_activate_out, inverse=False, bias=None):
        return features.new_empty((num_activate_out, filters.size(-1)))

    @reg(lib + 'indice_conv_backward')
    def _(features, filters, out_bp, indice_pairs, indice_pair_num, inverse=False):
        return torch.empty_like(features), torch.empty_like(filters, memory_format=torch.contiguous_format)

    @reg(lib + 'indice_maxpool')
    def _(features, indice_pairs, indice_pair_num, num_activate_out):
        return features.new_empty((num_activate_out, features.size(1)))

    @reg(lib + 'indice_maxpool_backward')
    def _(features, out_features, out_bp, indice_pairs, indice_pair_num):
        return torch.empty_like(features)


def _register_autograd() -> None:
    O = torch.ops.bfb_b200

    # bev_pool: out[b, c, z, x, y] = sum of feats[n, c] over the cell's points;
    # d feats[n] = grad_out at the point's cell (0 for dropped points)
    def bev_setup(ctx, inputs, output):
        feats, _, B, D, H, W = inputs
        ctx.save_for_backward(output[1])
        ctx.geo = (feats.size(0), B, D, H, W)

    def bev_backward(ctx, grad_out, _grad_plan):
        (plan,) = ctx.saved_tensors
        return O.bev_pool_backward(grad_out.contiguous(), plan, *ctx.geo), None, None, None, None, None

    torch.library.register_autograd('bfb_b200::bev_pool_forward', bev_backward, setup_context=bev_setup)

    def planned_setup(ctx, inputs, output):
        feats, plan, B, D, H, W = inputs
        ctx.save_for_backward(plan)
        ctx.geo = (feats.size(0), B, D, H, W)

    def planned_backward(ctx, grad_out):
        (plan,) = ctx.saved_tensors
        return O.bev_pool_backward(grad_out.contiguous(), plan, *ctx.geo), None, None, None, None, None

    torch.library.register_autograd('bfb_b200::bev_pool_forward_planned', planned_backward,
                                    setup_context=planned_setup)

    # fused depth x context pooling: gradients w.r.t. depth and context
    def dc_setup(ctx, inputs, output):
        depth, context, _, B, D, H, W = inputs
        ctx.save_for_backward(depth, output[1])
        ctx.geo = (context.size(1), B, D, H, W)

    def dc_backward(ctx, grad_out, _grad_aux):
        depth, aux = ctx.saved_tensors
        none = depth.new_empty((0,), dtype=torch.int64)  # the cells come from aux
        gdepth, gctx = O.bev_pool_dc_backward(grad_out.contiguous(), depth, none, aux, *ctx.geo)
        return gdepth, gctx, None, None, None, None, None

    torch.library.register_autograd('bfb_b200::bev_pool_dc_forward', dc_backward, setup_context=dc_setup)
    torch.library.register_autograd('bfb_b200::bev_pool_dc_forward_planned', dc_backward, setup_context=dc_setup)

    # dynamic scatter: gradient w.r.t. the point features only
    def scatter_setup(ctx, inputs, output):
        feats, _, reduce, _ = inputs
        ctx.save_for_backward(feats, output[0], output[2], output[3])
        ctx.reduce = reduce

    def scatter_backward(ctx, grad_vf, _gc, _gm, _gn):
        feats, reduced, pmap, counts = ctx.saved_tensors
        grad = torch.empty_like(feats)
        O.dynamic_scatter_backward(grad, grad_vf.contiguous(), feats, reduced, pmap, counts, ctx.reduce)
        return grad, None, None, None

    torch.library.register_autograd('bfb_b200::dynamic_scatter_forward', scatter_backward,
                                    setup_context=scatter_setup)

    # sparse convolution: gradients w.r.t. features, filters and the bias
    def conv_setup(ctx, inputs, output):
        features, filters, pairs, num, _, inverse, bias = inputs
        ctx.save_for_backward(features, filters, pairs, num)
        ctx.inverse = inverse
        ctx.has_bias = bias is not None

    def conv_backward(ctx, grad):
        features, filters, pairs, num = ctx.saved_tensors
        gin, gw = O.indice_conv_backward(features, filters, grad.contiguous(), pairs, num, ctx.inverse)
        gb = grad.sum(0) if ctx.has_bias else None
        return gin, gw.view_as(filters), None, None, None, None, gb

    torch.library.register_autograd('bfb_b200::indice_conv', conv_backward, setup_context=conv_setup)

    def pool_setup(ctx, inputs, output):
        features, pairs, num, _ = inputs
        ctx.save_for_backward(features, output, pairs, num)

    def pool_backward(ctx, grad):
        features, out, pairs, num = ctx.saved_tensors
        return O.indice_maxpool_backward(features, out, grad.contiguous(), pairs, num), None, None, None

    torch.library.register_autograd('bfb_b200::indice_maxpool', pool_backward, setup_context=pool_setup)


def register() -> None:
    """Register the fake kernels and autograd formulas (once per process)."""
    global _done
    if _done:
        return
    _done = True
    _register_fakes()
    _register_autograd()
