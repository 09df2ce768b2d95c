"""Sparse module containers: drop-ins for ops/spconv/modules.py:23-202
(``SparseModule``, ``SparseSequential``, ``ToDense``, ``RemoveGrid``).

``SparseSequential`` hands a ``SparseConvTensor`` to the sparse modules and
applies every other module (batch norm, activations) to its features, as
the reference does; the sparse encoder (models/backbones/sparse_encoder.py)
is built from it."""
from __future__ import annotations

from collections import OrderedDict

import torch
from torch import nn

from .structure import SparseConvTensor


class SparseModule(nn.Module):
    """Marker base class: modules of this type take and return a
    ``SparseConvTensor`` inside ``SparseSequential``."""


def is_spconv_module(module) -> bool:
    return isinstance(module, SparseModule)


def is_sparse_conv(module) -> bool:
    from .conv import SparseConvolution
    return isinstance(module, SparseConvolution)


class SparseSequential(SparseModule):
    """Sequential container over sparse and dense modules.  Accepts modules
    positionally, one ``OrderedDict``, or by keyword."""

    def __init__(self, *args, **kwargs):
        super().__init__()
        if len(args) == 1 and isinstance(args[0], OrderedDict):
            for name, m in args[0].items():
                self.add_module(name, m)
        else:
            for i, m in enumerate(args):
                self.add_module(str(i), m)
        for name, m in kwargs.items():
            if name in self._modules:
                raise ValueError('name exists.')
            self.add_module(name, m)
        self._sparity_dict = {}

    def __getitem__(self, idx):
        n = len(self)
        if not -n <= idx < n:
            raise IndexError(f'index {idx} is out of range')
        return list(self._modules.values())[idx % n]

    def __len__(self):
        return len(self._modules)

    @property
    def sparity_dict(self):
        return self._sparity_dict

    def add(self, module, name=None):
        if name is None:
            name = str(len(self._modules))
            if name in self._modules:
                raise KeyError('name exists')
        self.add_module(name, module)

    def forward(self, input):
        for name, m in self._modules.items():
            if is_spconv_module(m):
                assert isinstance(input, SparseConvTensor)
                self._sparity_dict[name] = input.sparity
                input = m(input)
            elif isinstance(input, SparseConvTensor):
                if input.indices.shape[0] != 0:  # an empty tensor keeps its features
                    input.features = m(input.features)
            else:
                input = m(input)
        return input

    def fused(self):
        """A copy in which every sparse convolution directly followed by a
        ``BatchNorm1d`` becomes one convolution with the normalisation folded
        into its filters and bias (``fused_bn``), with the reference's folding
        formula: w * gamma / (sqrt(var) + eps), (b - mean) * gamma /
        (sqrt(var) + eps) + beta."""
        from .conv import SparseConvolution
        mods = list(self._modules.values())
        out, i = [], 0
        while i < len(mods):
            m = mods[i]
            if is_sparse_conv(m) and i + 1 < len(mods) and isinstance(mods[i + 1], nn.BatchNorm1d):
                bn = mods[i + 1]
                conv = SparseConvolution(m.ndim, m.in_channels, m.out_channels, m.kernel_size, m.stride, m.padding,
                                         m.dilation, m.groups, True, m.subm, m.output_padding, m.transposed,
                                         m.inverse, m.indice_key, fused_bn=True).to(m.weight.device)
                conv.load_state_dict(m.state_dict(), strict=False)
                with torch.no_grad():
                    scale = bn.weight / (torch.sqrt(bn.running_var) + bn.eps)
                    conv.weight.mul_(scale)
                    conv.bias.copy_(-bn.running_mean * scale + bn.bias)
                out.append(conv)
                i += 2
            else:
                out.append(m)
                i += 1
        return SparseSequential(*out)


class ToDense(SparseModule):
    """SparseConvTensor -> dense [B, C, *spatial]."""

    def forward(self, x: SparseConvTensor):
        return x.dense()


class RemoveGrid(SparseModule):
    """Drops the tensor's pre-allocated grid."""

    def forward(self, x: SparseConvTensor):
        x.grid = None
        return x
