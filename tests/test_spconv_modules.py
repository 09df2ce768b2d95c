"""The sparse-convolution module layer on CPU: construction, parameter
initialisation, SparseSequential dispatch, SparseConvTensor helpers and the
batch-norm folding of SparseSequential.fused() (ops/spconv/conv.py,
modules.py, structure.py, pool.py of the reference).  No kernel runs here."""
import math

import numpy as np
import pytest
import torch
from torch import nn

from bevfusion_triton_b200.ops import spconv as S


def test_constructors_and_parameters():
    m = S.SubMConv3d(16, 32, 3, indice_key='subm1')
    assert m.weight.shape == (3, 3, 3, 16, 32) and m.bias.shape == (32,)
    assert m.subm and not m.transposed and not m.inverse and m.indice_key == 'subm1'
    c = S.SparseConv3d(16, 32, (1, 1, 3), stride=(1, 1, 2), padding=0, bias=False)
    assert c.bias is None and c.kernel_size == [1, 1, 3] and c.stride == [1, 1, 2] and c.padding == [0, 0, 0]
    t = S.SparseConvTranspose3d(8, 4, 3, stride=2)
    assert t.transposed and t.output_padding == [0, 0, 0]
    inv = S.SparseInverseConv3d(32, 16, 3, indice_key='spconv2')
    assert inv.inverse and inv.kernel_size == [3, 3, 3] and inv.stride == [1, 1, 1]
    assert S.SubMConv3d(4, 4, 1).conv1x1 and not m.conv1x1
    assert S.SparseConv2d(3, 5, 3).weight.shape == (3, 3, 3, 5)
    with pytest.raises(AssertionError):
        S.SparseConv3d(4, 4, 3, stride=2, dilation=2)
    # kaiming-uniform filters; bias bound 1 / sqrt(fan_in), fan_in = Cin * kernel volume
    torch.manual_seed(0)
    m = S.SubMConv3d(16, 32, 3)
    fan_in = 16 * 27
    assert float(m.bias.abs().max()) <= 1 / math.sqrt(fan_in)
    assert float(m.weight.abs().max()) <= 1 / math.sqrt(fan_in) + 1e-7


def test_sparse_conv_tensor_helpers():
    idx = torch.tensor([[0, 1, 2, 0], [1, 0, 0, 1], [0, 2, 1, 1]], dtype=torch.int64)
    f = torch.arange(6, dtype=torch.float32).view(3, 2)
    x = S.SparseConvTensor(f, idx, [3, 3, 2], 2)
    assert x.indices.dtype == torch.int32
    assert x.spatial_size == 18 and x.sparity == 3 / 18 / 2
    d = x.dense()
    assert d.shape == (2, 2, 3, 3, 2)
    want = torch.zeros(2, 3, 3, 2, 2)
    for r, (b, i, j, k) in enumerate(idx.tolist()):
        want[b, i, j, k] = f[r]
    assert torch.equal(d, want.permute(0, 4, 1, 2, 3))
    assert torch.equal(x.dense(channels_first=False), want)
    assert x.find_indice_pair(None) is None and x.find_indice_pair('k') is None
    x.indice_dict['k'] = 1
    assert x.find_indice_pair('k') == 1
    assert torch.equal(S.scatter_nd(torch.tensor([[1], [3]]), torch.tensor([5., 7.]), [4]),
                       torch.tensor([0., 5., 0., 7.]))


def test_sequential_dispatch_on_cpu():
    """Dense modules act on the features of a SparseConvTensor (not on an
    empty one); sparse modules receive the tensor itself."""
    seen = []

    class Probe(S.SparseModule):
        def forward(self, t):
            seen.append(type(t).__name__)
            return t

    seq = S.SparseSequential(Probe(), nn.ReLU(), Probe())
    x = S.SparseConvTensor(torch.tensor([[-1., 2.]]), torch.zeros(1, 4, dtype=torch.int32), [2, 2, 2], 1)
    y = seq(x)
    assert seen == ['SparseConvTensor', 'SparseConvTensor'] and torch.equal(y.features, torch.tensor([[0., 2.]]))
    assert set(seq.sparity_dict) == {'0', '2'}
    empty = S.SparseConvTensor(torch.tensor([[-1.]])[:0], torch.zeros(0, 4, dtype=torch.int32), [2, 2, 2], 1)
    assert seq(empty).features.shape == (0, 1)
    assert len(seq) == 3 and isinstance(seq[-1], Probe)
    with pytest.raises(IndexError):
        seq[3]
    seq.add(nn.Identity())
    assert len(seq) == 4
    assert torch.equal(S.SparseSequential(nn.ReLU())(torch.tensor([-2., 3.])), torch.tensor([0., 3.]))


def test_fused_folds_batch_norm_with_the_reference_formula():
    torch.manual_seed(1)
    conv = S.SubMConv3d(4, 6, 3, indice_key='a')
    bn = nn.BatchNorm1d(6, eps=1e-3)
    with torch.no_grad():
        bn.running_mean.uniform_(-1, 1)
        bn.running_var.uniform_(0.5, 2)
        bn.weight.uniform_(0.5, 1.5)
        bn.bias.uniform_(-1, 1)
    fused = S.SparseSequential(conv, bn, nn.ReLU()).fused()
    assert len(fused) == 2 and fused[0].fused_bn and fused[0].indice_key == 'a'
    scale = bn.weight / (torch.sqrt(bn.running_var) + bn.eps)
    torch.testing.assert_close(fused[0].weight, conv.weight * scale)
    torch.testing.assert_close(fused[0].bias, -bn.running_mean * scale + bn.bias)


def test_legacy_import_paths():
    """The reference's legacy module names resolve to this library's ops."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool_legacy
    from bevfusion_triton_b200.ops.spconv import ops_legacy
    from bevfusion_triton_b200.ops.voxel import voxel_layer_legacy
    assert ops_legacy.indice_conv is S.indice_conv and ops_legacy.get_indice_pairs is S.get_indice_pairs
    assert voxel_layer_legacy.voxel_layer_ext.dynamic_voxelize is voxel_layer_legacy.dynamic_voxelize
    assert callable(bev_pool_legacy.bev_pool)


REFERENCE_SPCONV_ALL = ['SparseConv2d', 'SparseConv3d', 'SubMConv2d', 'SubMConv3d', 'SparseConvTranspose2d',
                        'SparseConvTranspose3d', 'SparseInverseConv2d', 'SparseInverseConv3d', 'SparseModule',
                        'SparseSequential', 'SparseMaxPool2d', 'SparseMaxPool3d', 'SparseConvTensor', 'scatter_nd']


def test_package_exports_match_the_reference():
    """The export lists the reference's own tests pin
    (tests/test_ops/test_spconv/test_spconv.py:27-42, 221-227), and the
    symbols are the module-level classes."""
    from bevfusion_triton_b200.ops import voxel
    from bevfusion_triton_b200.ops.spconv import conv, modules, pool, structure
    assert S.__all__ == REFERENCE_SPCONV_ALL and all(hasattr(S, n) for n in S.__all__)
    assert voxel.__all__ == ['Voxelization', 'voxelization', 'dynamic_scatter', 'DynamicScatter']
    assert S.SparseConv3d is conv.SparseConv3d and S.SparseSequential is modules.SparseSequential
    assert S.SparseMaxPool2d is pool.SparseMaxPool2d and S.SparseConvTensor is structure.SparseConvTensor
    for m in (S.SparseConv2d(3, 4, 3, stride=1, padding=1), S.SparseConv3d(3, 4, 3, stride=1, padding=1),
              S.SubMConv2d(3, 4, 3), S.SubMConv3d(3, 4, 3), S.SparseConvTranspose2d(3, 4, 3, stride=1, padding=1),
              S.SparseConvTranspose3d(3, 4, 3, stride=1, padding=1), S.SparseInverseConv2d(3, 4, 3, indice_key='k'),
              S.SparseInverseConv3d(3, 4, 3, indice_key='k'), S.SparseMaxPool2d(1), S.SparseMaxPool3d(1),
              S.SparseSequential()):
        assert isinstance(m, S.SparseModule)
    dense = S.scatter_nd(torch.tensor([[0, 0], [1, 1]]), torch.tensor([1.0, 2.0]), [2, 2])
    assert dense.tolist() == [[1.0, 0.0], [0.0, 2.0]]
    st = S.SparseConvTensor(torch.tensor([[1.0, 2.0], [3.0, 4.0]]), torch.tensor([[0, 0, 0], [0, 0, 1]],
                                                                                dtype=torch.int32), [1, 2], 1)
    assert st.dense(channels_first=True).shape == (1, 2, 1, 2) and st.dense(channels_first=False).shape == (1, 1, 2, 2)
