"""Sparse convolution modules: drop-ins for ops/spconv/conv.py:27-470
(``SparseConvolution`` and its 2-/3-/4-D regular, transposed, inverse and
submanifold forms; same constructor arguments, parameters and rulebook
caching).

A layer with an ``indice_key`` stores its rulebook in the input tensor's
``indice_dict`` as ``(outids, indices, indice_pairs, indice_pair_num,
spatial_shape)`` and reuses a stored one; an inverse convolution takes the
rulebook of the strided layer with the same key and maps that layer's
outputs back to its inputs.  The forward is one call of the
``bfb_b200::indice_conv`` op with the bias added in its epilogue (the
result is rounded before the bias is added, as the reference's
``out += bias`` does), and its backward is registered on the op.
"""
from __future__ import annotations

import math

import numpy as np
import torch
from torch import nn
from torch.nn import init

from ..._lib import ops as _native
from . import ops as spops
from .modules import SparseModule
from .structure import SparseConvTensor


def _nd(v, ndim):
    return list(v) if isinstance(v, (list, tuple)) else [v] * ndim


def _fan_in_hwio(w: torch.Tensor) -> int:
    """Fan-in of a [*kernel, Cin, Cout] filter (ops/spconv/conv.py:27-46)."""
    if w.dim() < 2:
        raise ValueError('fan in and fan out can not be computed for tensorwith fewer than 2 dimensions')
    if w.dim() == 2:
        return w.size(-2)
    return w.size(-2) * w[..., 0, 0].numel()


class SparseConvolution(SparseModule):
    def __init__(self, ndim, in_channels, out_channels, kernel_size=3, stride=1, padding=0, dilation=1, groups=1,
                 bias=True, subm=False, output_padding=0, transposed=False, inverse=False, indice_key=None,
                 fused_bn=False):
        super().__init__()
        assert groups == 1
        kernel_size, stride = _nd(kernel_size, ndim), _nd(stride, ndim)
        padding, dilation = _nd(padding, ndim), _nd(dilation, ndim)
        output_padding = _nd(output_padding, ndim)
        for d, s in zip(dilation, stride):
            assert any([s == 1, d == 1]), "don't support this."
        self.ndim = ndim
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.conv1x1 = int(np.prod(kernel_size)) == 1
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.transposed = transposed
        self.inverse = inverse
        self.output_padding = output_padding
        self.groups = groups
        self.subm = subm
        self.indice_key = indice_key
        self.fused_bn = fused_bn
        self.weight = nn.Parameter(torch.empty(*kernel_size, in_channels, out_channels))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_channels))
        else:
            self.register_parameter('bias', None)
        self.reset_parameters()

    def reset_parameters(self):
        init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1 / math.sqrt(_fan_in_hwio(self.weight))
            init.uniform_(self.bias, -bound, bound)

    def _out_shape(self, spatial_shape):
        if self.subm:
            return spatial_shape
        if self.transposed:
            return spops.get_deconv_output_size(spatial_shape, self.kernel_size, self.stride, self.padding,
                                                self.dilation, self.output_padding)
        return spops.get_conv_output_size(spatial_shape, self.kernel_size, self.stride, self.padding, self.dilation)

    def forward(self, input: SparseConvTensor) -> SparseConvTensor:
        assert isinstance(input, SparseConvTensor)
        feats, indices = input.features, input.indices
        spatial_shape, batch = input.spatial_shape, input.batch_size
        if self.conv1x1:
            out = feats @ self.weight.view(self.in_channels, self.out_channels)
            if self.bias is not None:
                out = out + self.bias
            res = SparseConvTensor(out, indices, spatial_shape, batch)
        else:
            cached = input.find_indice_pair(self.indice_key)
            if self.inverse:
                assert cached is not None and self.indice_key is not None
                _, outids, pairs, num, out_shape = cached
                assert pairs.shape[0] == np.prod(self.kernel_size), \
                    'inverse conv must have same kernel size as its couple conv'
            elif cached is not None:
                outids, _, pairs, num, _ = cached
                out_shape = self._out_shape(spatial_shape)
            else:
                out_shape = self._out_shape(spatial_shape)
                outids, pairs, num = spops.get_indice_pairs(indices, batch, spatial_shape, self.kernel_size,
                                                            self.stride, self.padding, self.dilation,
                                                            self.output_padding, self.subm, self.transposed,
                                                            grid=input.grid)
                input.indice_dict[self.indice_key] = (outids, indices, pairs, num, spatial_shape)
            # the fused (folded batch-norm) form of a submanifold layer adds no
            # bias, as the reference's fused_indice_conv
            f, (w, b), back = spops._amp(feats, self.weight,
                                         None if (self.fused_bn and self.subm) else self.bias)
            out = _native().indice_conv(f, w, pairs.to(feats.device), num.to(feats.device), int(outids.shape[0]),
                                        bool(self.inverse), b)
            if back is not None:
                out = out.to(back)
            res = SparseConvTensor(out, outids, out_shape, batch)
        res.indice_dict = input.indice_dict
        res.grid = input.grid
        return res


def _conv_class(name, ndim, **fixed):
    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1, bias=True,
                 indice_key=None):
        SparseConvolution.__init__(self, ndim, in_channels, out_channels, kernel_size, stride, padding, dilation,
                                   groups, bias, indice_key=indice_key, **fixed)
    return type(name, (SparseConvolution,), {'__init__': __init__, '__doc__': f'{ndim}-D {name} (ops/spconv/conv.py).'})


SparseConv2d = _conv_class('SparseConv2d', 2)
SparseConv3d = _conv_class('SparseConv3d', 3)
SparseConv4d = _conv_class('SparseConv4d', 4)
SparseConvTranspose2d = _conv_class('SparseConvTranspose2d', 2, transposed=True)
SparseConvTranspose3d = _conv_class('SparseConvTranspose3d', 3, transposed=True)
SubMConv2d = _conv_class('SubMConv2d', 2, subm=True)
SubMConv3d = _conv_class('SubMConv3d', 3, subm=True)
SubMConv4d = _conv_class('SubMConv4d', 4, subm=True)


class SparseInverseConv2d(SparseConvolution):
    def __init__(self, in_channels, out_channels, kernel_size, indice_key, bias=True):
        super().__init__(2, in_channels, out_channels, kernel_size, bias=bias, inverse=True, indice_key=indice_key)


class SparseInverseConv3d(SparseConvolution):
    def __init__(self, in_channels, out_channels, kernel_size, indice_key, bias=True):
        super().__init__(3, in_channels, out_channels, kernel_size, bias=bias, inverse=True, indice_key=indice_key)
