"""Sparse max-pooling modules: drop-ins for ops/spconv/pool.py:21-81.  The
rulebook is built per call (no ``indice_key``), as in the reference."""
from __future__ import annotations

from . import ops as spops
from .functional import indice_maxpool
from .modules import SparseModule
from .structure import SparseConvTensor


class SparseMaxPool(SparseModule):
    def __init__(self, ndim, kernel_size, stride=1, padding=0, dilation=1, subm=False):
        super().__init__()
        nd = lambda v: list(v) if isinstance(v, (list, tuple)) else [v] * ndim  # noqa: E731
        self.ndim = ndim
        self.kernel_size = nd(kernel_size)
        self.stride = nd(stride)
        self.padding = nd(padding)
        self.subm = subm
        self.dilation = nd(dilation)

    def forward(self, input: SparseConvTensor) -> SparseConvTensor:
        assert isinstance(input, SparseConvTensor)
        shape = input.spatial_shape
        out_shape = shape if self.subm else spops.get_conv_output_size(shape, self.kernel_size, self.stride,
                                                                       self.padding, self.dilation)
        outids, pairs, num = spops.get_indice_pairs(input.indices, input.batch_size, shape, self.kernel_size,
                                                    self.stride, self.padding, self.dilation, 0, self.subm)
        dev = input.features.device
        out = indice_maxpool(input.features, pairs.to(dev), num.to(dev), int(outids.shape[0]))
        res = SparseConvTensor(out, outids, out_shape, input.batch_size)
        res.indice_dict = input.indice_dict
        res.grid = input.grid
        return res


class SparseMaxPool2d(SparseMaxPool):
    def __init__(self, kernel_size, stride=1, padding=0, dilation=1):
        super().__init__(2, kernel_size, stride, padding, dilation)


class SparseMaxPool3d(SparseMaxPool):
    def __init__(self, kernel_size, stride=1, padding=0, dilation=1):
        super().__init__(3, kernel_size, stride, padding, dilation)
