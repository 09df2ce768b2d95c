"""Sparse-convolution rulebook (``get_indice_pairs``) and the convolution /
max-pooling over it (``indice_conv``, ``fused_indice_conv``,
``indice_conv_backward``, ``indice_maxpool``, ``indice_maxpool_backward``,
ops/spconv/ops.py:95-188) on the sm_100a kernels.

Reference: ops/spconv/ops.py:25-93 (output-size helpers, ``get_indice_pairs``)
and ops/spconv/src/spconv_triton.py:608-652 (argument checks), :792-915 (the
Triton path).  Same signature, exception types and results as the reference's
GPU path: submanifold returns the input rows as outputs; a regular or
transposed rulebook numbers its output sites in ascending (b, c0, ..) order;
within a rule the pairs are in ascending input row, unused slots -1.

Differences: CUDA tensors only (no CPU path); ``batch * prod(out_shape)``
must stay below 2**32; the optional ``grid`` scratch tensor is not needed and
is only reset to -1, as the reference leaves it.
"""
from __future__ import annotations

import torch

from ..._lib import ops


def get_conv_output_size(input_size, kernel_size, stride, padding, dilation):
    """ops/spconv/ops.py:25-37."""
    out = []
    for i in range(len(input_size)):
        size = (input_size[i] + 2 * padding[i] - dilation[i] * (kernel_size[i] - 1) - 1) // stride[i] + 1
        out.append(1 if kernel_size[i] == -1 else size)
    return out


def get_deconv_output_size(input_size, kernel_size, stride, padding, dilation, output_padding):
    """ops/spconv/ops.py:40-50."""
    out = []
    for i in range(len(input_size)):
        if kernel_size[i] == -1:
            raise ValueError("deconv don't support kernel_size < 0")
        out.append((input_size[i] - 1) * stride[i] - 2 * padding[i] + kernel_size[i] + output_padding[i])
    return out


def _nd(value, ndim: int) -> list[int]:
    if isinstance(value, (list, tuple)):
        if len(value) != ndim:
            raise ValueError(f'Expected parameter of length {ndim}, got {len(value)}')
        return [int(v) for v in value]
    return [int(value)] * ndim


def get_indice_pairs(indices: torch.Tensor, batch_size: int, spatial_shape, ksize=3, stride=1, padding=0,
                     dilation=1, out_padding=0, subm: bool = False, transpose: bool = False,
                     grid: torch.Tensor | None = None):
    """(outids [M, ndim + 1], indice_pairs [K, 2, N], indice_num [K]) of a
    sparse convolution over ``indices`` [N, ndim + 1] (b, c0, ..)."""
    if batch_size <= 0:
        raise ValueError('batch_size must be positive')
    if not indices.is_cuda:
        raise RuntimeError('bevfusion_triton_b200 ops run on CUDA tensors only (no CPU fallback)')
    if indices.numel() > 0:
        bmin, bmax = (int(v) for v in torch.aminmax(indices[:, 0]))  # one host read
        if bmin < 0:
            raise ValueError('indices batch column must be non-negative')
        if bmax >= batch_size:
            raise ValueError('indices batch column exceeds batch_size')
    ndim = indices.shape[1] - 1
    ksize, stride, padding = _nd(ksize, ndim), _nd(stride, ndim), _nd(padding, ndim)
    dilation, out_padding = _nd(dilation, ndim), _nd(out_padding, ndim)
    spatial_shape = [int(v) for v in spatial_shape]
    for d, s in zip(dilation, stride):
        assert any([s == 1, d == 1]), "don't support this."
    if subm:
        out_shape = spatial_shape
    elif transpose:
        out_shape = get_deconv_output_size(spatial_shape, ksize, stride, padding, dilation, out_padding)
    else:
        out_shape = get_conv_output_size(spatial_shape, ksize, stride, padding, dilation)
    outids, pairs, num = ops().get_indice_pairs(indices, int(batch_size), out_shape, ksize, stride, padding,
                                                dilation, bool(subm), bool(transpose))
    if grid is not None:
        grid.fill_(-1)
    if subm:
        outids = indices
    dt = indices.dtype
    return outids.to(dt), pairs.to(dt), num.to(dt)


# --------------------------------------------------------------- convolution
def _require_cuda(*ts) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError('bevfusion_triton_b200 ops run on CUDA tensors only (no CPU fallback)')


def _amp(features, *ts):
    """Operands as the convolution computes them.  Under torch.autocast the
    reference's per-rule matmul runs in the autocast dtype (fp16 / bf16, on
    the tensor cores) whatever the features' and filters' dtypes, and its
    result lands in a buffer of the features' dtype; here the features and
    the other operands are cast to the autocast dtype (a differentiable cast,
    so fp32 parameters still receive gradients) and the result is returned
    in the features' dtype.  Outside autocast the dtypes must match.
    Returns (features, operands, dtype to return the result in, or None)."""
    dev = features.device.type
    if not torch.is_autocast_enabled(dev):
        return features, ts, None
    dt = torch.get_autocast_dtype(dev)
    cast = (lambda t: None if t is None or t.dtype == dt else t.to(dt))  # noqa: E731
    keep = (lambda t, c: t if c is None else c)  # noqa: E731
    return keep(features, cast(features)), tuple(keep(t, cast(t)) for t in ts), (
        None if features.dtype == dt else features.dtype)


def indice_conv(features: torch.Tensor, filters: torch.Tensor, indice_pairs: torch.Tensor,
                indice_pair_num: torch.Tensor, num_activate_out: int, inverse: bool = False,
                subm: bool = False) -> torch.Tensor:
    """[num_activate_out, Cout]: every output row sums, over the kernel
    offsets k in ascending order, features[in] @ filters[k] for the rule-k
    pair (in, out) that names it (ops/spconv/ops.py:95-114 ->
    spconv_triton.py:981-1007).  ``inverse`` swaps the two pair slots;
    ``subm`` changes nothing here, as in the reference.  One launch over all
    rules, no host read of the rule counts; differentiable w.r.t. features and
    filters."""
    del subm
    _require_cuda(features, filters, indice_pairs, indice_pair_num)
    f, (w,), back = _amp(features, filters)
    out = ops().indice_conv(f, w, indice_pairs, indice_pair_num, int(num_activate_out), bool(inverse), None)
    return out if back is None else out.to(back)


def fused_indice_conv(features, filters, bias, indice_pairs, indice_pair_num, num_activate_out, inverse, subm):
    """indice_conv + bias, the bias added in the kernel's epilogue; as in the
    reference (spconv_triton.py:1010-1032) a submanifold convolution adds no
    bias here."""
    _require_cuda(features, filters, indice_pairs, indice_pair_num)
    f, (w, b), back = _amp(features, filters, None if subm else bias)
    out = ops().indice_conv(f, w, indice_pairs, indice_pair_num, int(num_activate_out), bool(inverse), b)
    return out if back is None else out.to(back)


def indice_conv_backward(features, filters, out_bp, indice_pairs, indice_pair_num, inverse: bool = False,
                         subm: bool = False):
    """(input_grad [N, Cin], filters_grad shaped like filters)
    (spconv_triton.py:1035-1061); the filter gradient is summed in a fixed
    order, so it is deterministic."""
    del subm
    _require_cuda(features, filters, out_bp, indice_pairs, indice_pair_num)
    f, (w, g), back = _amp(features, filters, out_bp)
    gin, gw = ops().indice_conv_backward(f, w, g, indice_pairs, indice_pair_num, bool(inverse))
    return (gin if back is None else gin.to(back)), gw.view(filters.shape).to(filters.dtype)


def indice_maxpool(features, indice_pairs, indice_pair_num, num_activate_out):
    """[num_activate_out, C]: max over each output's inputs, never below 0
    (the reference pools into zeros, spconv_triton.py:1064-1082)."""
    _require_cuda(features, indice_pairs, indice_pair_num)
    return ops().indice_maxpool(features, indice_pairs, indice_pair_num, int(num_activate_out))


def indice_maxpool_backward(features, out_features, out_bp, indice_pairs, indice_pair_num):
    """input_grad [N, C]: every input equal to its output's pooled value
    receives that output's gradient (spconv_triton.py:1085-1111)."""
    _require_cuda(features, out_features, out_bp, indice_pairs, indice_pair_num)
    return ops().indice_maxpool_backward(features, out_features, out_bp, indice_pairs, indice_pair_num)
