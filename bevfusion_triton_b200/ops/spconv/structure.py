"""``SparseConvTensor`` and ``scatter_nd``: drop-ins for
ops/spconv/structure.py:5-61 (same attributes and methods, which the sparse
encoder and the convolution modules read: ``features``, ``indices``,
``spatial_shape``, ``batch_size``, ``indice_dict``, ``grid``,
``spatial_size``, ``find_indice_pair``, ``dense``, ``sparity``)."""
from __future__ import annotations

import numpy as np
import torch


def scatter_nd(indices: torch.Tensor, updates: torch.Tensor, shape) -> torch.Tensor:
    """A zero tensor of ``shape`` with ``updates`` written at ``indices``
    (the last dimension of ``indices`` addresses the leading dimensions of
    ``shape``).  Like the reference, repeated indices are not summed: one of
    the writes wins."""
    shape = list(shape)
    ret = torch.zeros(shape, dtype=updates.dtype, device=updates.device)
    nd = indices.shape[-1]
    flat = indices.reshape(-1, nd).long()
    lead = torch.tensor(shape[:nd], device=flat.device, dtype=torch.long)
    strides = torch.ones(nd, dtype=torch.long, device=flat.device)
    for d in range(nd - 2, -1, -1):
        strides[d] = strides[d + 1] * lead[d + 1]
    rows = (flat * strides).sum(1)
    ret.view(-1, *shape[nd:])[rows] = updates.reshape(-1, *shape[nd:])
    return ret


class SparseConvTensor:
    """Active sites ``indices`` [N, ndim + 1] int32 rows (b, c0, ..) with
    ``features`` [N, C] on a grid of ``spatial_shape`` for ``batch_size``
    samples.  ``indice_dict`` caches rulebooks by a layer's ``indice_key``
    so that layers sharing a key (and the inverse convolution of a strided
    one) reuse them."""

    def __init__(self, features, indices, spatial_shape, batch_size, grid=None):
        self.features = features
        self.indices = indices if indices.dtype == torch.int32 else indices.int()
        self.spatial_shape = spatial_shape
        self.batch_size = batch_size
        self.indice_dict = {}
        self.grid = grid

    @property
    def spatial_size(self):
        return np.prod(self.spatial_shape)

    def find_indice_pair(self, key):
        if key is None:
            return None
        return self.indice_dict.get(key)

    def dense(self, channels_first: bool = True) -> torch.Tensor:
        """[B, C, *spatial] (or [B, *spatial, C]) with zeros at inactive sites."""
        shape = [self.batch_size] + list(self.spatial_shape) + [self.features.shape[1]]
        res = scatter_nd(self.indices.long(), self.features, shape)
        if not channels_first:
            return res
        nd = len(self.spatial_shape)
        return res.permute(0, nd + 1, *range(1, nd + 1)).contiguous()

    @property
    def sparity(self):
        return self.indices.shape[0] / np.prod(self.spatial_shape) / self.batch_size
