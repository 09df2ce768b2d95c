"""Drop-in for the legacy import path ops/spconv/ops_legacy.py:72-270 (the
compiled-extension backend of ``ops.spconv.ops``: ``get_conv_output_size``,
``get_deconv_output_size``, ``get_indice_pairs``, ``indice_conv``,
``fused_indice_conv``, ``indice_conv_backward``, ``indice_maxpool``,
``indice_maxpool_backward``; same signatures).

They are this library's ops (``ops.spconv.ops``): the rulebook follows the
reference's GPU ordering (output sites in ascending (b, c0, ..) order, rule
pairs in ascending input row), the convolutions run on the sm_100a kernels.
"""
from .ops import (fused_indice_conv, get_conv_output_size, get_deconv_output_size, get_indice_pairs, indice_conv,
                  indice_conv_backward, indice_maxpool, indice_maxpool_backward)

__all__ = ['fused_indice_conv', 'get_conv_output_size', 'get_deconv_output_size', 'get_indice_pairs', 'indice_conv',
           'indice_conv_backward', 'indice_maxpool', 'indice_maxpool_backward']
