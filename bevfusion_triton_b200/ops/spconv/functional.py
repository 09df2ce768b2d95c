"""Differentiable sparse convolution and pooling, drop-ins for
ops/spconv/functional.py:21-114 (``indice_conv``, ``indice_inverse_conv``,
``indice_subm_conv``, ``indice_maxpool``, same positional arguments).

The reference wraps each op in a ``torch.autograd.Function``; here the
backward is registered on the ``bfb_b200::indice_conv`` / ``indice_maxpool``
custom ops themselves, so these are plain calls that autograd,
``torch.compile`` and ``torch.export`` see through.
"""
from __future__ import annotations

import torch

from . import ops as _ops


def indice_conv(features: torch.Tensor, filters: torch.Tensor, indice_pairs: torch.Tensor,
                indice_pair_num: torch.Tensor, num_activate_out: int) -> torch.Tensor:
    return _ops.indice_conv(features, filters, indice_pairs, indice_pair_num, num_activate_out, False)


def indice_inverse_conv(features, filters, indice_pairs, indice_pair_num, num_activate_out):
    return _ops.indice_conv(features, filters, indice_pairs, indice_pair_num, num_activate_out, True)


def indice_subm_conv(features, filters, indice_pairs, indice_pair_num, num_activate_out):
    return _ops.indice_conv(features, filters, indice_pairs, indice_pair_num, num_activate_out, False, True)


def indice_maxpool(features, indice_pairs, indice_pair_num, num_activate_out):
    return _ops.indice_maxpool(features, indice_pairs, indice_pair_num, num_activate_out)
