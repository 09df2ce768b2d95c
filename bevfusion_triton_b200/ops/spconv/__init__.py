"""Sparse convolution: rulebook, convolution and max-pooling ops
(``ops.py``, ``functional.py``) and the module layer the sparse encoder is
built from (``conv.py``, ``pool.py``, ``modules.py``, ``structure.py``),
drop-ins for the reference's ``ops/spconv`` package."""
from .conv import (SparseConv2d, SparseConv3d, SparseConv4d, SparseConvolution, SparseConvTranspose2d,
                   SparseConvTranspose3d, SparseInverseConv2d, SparseInverseConv3d, SubMConv2d, SubMConv3d,
                   SubMConv4d)
from .modules import RemoveGrid, SparseModule, SparseSequential, ToDense
from .ops import (fused_indice_conv, get_conv_output_size, get_deconv_output_size, get_indice_pairs, indice_conv,
                  indice_conv_backward, indice_maxpool, indice_maxpool_backward)
from .pool import SparseMaxPool2d, SparseMaxPool3d
from .structure import SparseConvTensor, scatter_nd

# the reference package's export list, in its order (ops/spconv/__init__.py);
# the ops and the 4-D / helper modules above are importable from here too
__all__ = ['SparseConv2d', 'SparseConv3d', 'SubMConv2d', 'SubMConv3d', 'SparseConvTranspose2d', 'SparseConvTranspose3d',
           'SparseInverseConv2d', 'SparseInverseConv3d', 'SparseModule', 'SparseSequential', 'SparseMaxPool2d',
           'SparseMaxPool3d', 'SparseConvTensor', 'scatter_nd']
