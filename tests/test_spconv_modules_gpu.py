"""The sparse-convolution module layer on the GPU against a composition of
the reference's own installed GPU functions (spconv_triton.get_indice_pairs
/ indice_conv / indice_maxpool, ops/spconv/src/spconv_triton.py) in the
order the reference modules call them (ops/spconv/conv.py:114-224,
pool.py:40-71): rulebooks cached by indice_key, the inverse convolution on
the strided layer's rulebook, bias after the convolution, batch norm and
ReLU on the features.  fp32 forward: equal bit for bit."""
import sys
from pathlib import Path

import pytest
import torch
from torch import nn

from bevfusion_triton_b200.ops import spconv as S
from tests.test_spconv_gpu import SPARSE_SHAPE, lidar_voxel_indices

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / 'baseline'))
import ref_triton  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def ref(cuda):
    why = ref_triton.available()
    if why:
        pytest.skip(why)
    try:
        return ref_triton.load_spconv()
    except RuntimeError as e:
        pytest.skip(str(e))


def encoder():
    torch.manual_seed(5)
    net = S.SparseSequential(
        S.SubMConv3d(5, 16, 3, padding=1, bias=False, indice_key='subm1'), nn.BatchNorm1d(16, eps=1e-3), nn.ReLU(),
        S.SubMConv3d(16, 16, 3, padding=1, bias=False, indice_key='subm1'), nn.BatchNorm1d(16, eps=1e-3), nn.ReLU(),
        S.SparseConv3d(16, 32, 3, stride=2, padding=1, bias=False, indice_key='spconv2'),
        nn.BatchNorm1d(32, eps=1e-3), nn.ReLU(),
        S.SubMConv3d(32, 32, 3, padding=1, indice_key='subm2'),
        S.SparseConv3d(32, 32, (1, 1, 3), stride=(1, 1, 2), padding=0, indice_key='out'),
        S.SparseInverseConv3d(32, 16, (1, 1, 3), indice_key='out'),
        S.SubMConv3d(16, 8, 1),
    ).cuda()
    for m in net.modules():
        if isinstance(m, nn.BatchNorm1d):
            with torch.no_grad():
                m.running_mean.uniform_(-0.2, 0.2)
                m.running_var.uniform_(0.5, 1.5)
    return net.eval()


def reference_forward(ref, net, x):
    """The reference modules' sequence of calls, written out."""
    feats, idx, shape, B = x.features, x.indices, list(x.spatial_shape), x.batch_size
    cache = {}
    for m in net:
        if isinstance(m, S.SparseConvolution):
            if m.conv1x1:
                feats = feats @ m.weight.view(m.in_channels, m.out_channels) + m.bias
                continue
            if m.inverse:
                _, outids, pairs, num, out_shape = cache[m.indice_key]
            elif m.indice_key in cache:
                outids, _, pairs, num, _ = cache[m.indice_key]
                out_shape = shape if m.subm else S.get_conv_output_size(shape, m.kernel_size, m.stride, m.padding,
                                                                        m.dilation)
            else:
                outids, pairs, num = ref.get_indice_pairs(idx, B, shape, m.kernel_size, m.stride, m.padding,
                                                          m.dilation, m.output_padding, m.subm, m.transposed)
                out_shape = shape if m.subm else S.get_conv_output_size(shape, m.kernel_size, m.stride, m.padding,
                                                                        m.dilation)
                cache[m.indice_key] = (outids, idx, pairs, num, shape)
            feats = ref.indice_conv(feats, m.weight, pairs, num, outids.shape[0], m.inverse, m.subm)
            if m.bias is not None:
                feats = feats + m.bias
            idx, shape = outids, out_shape
        else:
            feats = m(feats)
    return feats, idx, shape


def test_encoder_stack_matches_reference_composition(ref):
    idx = lidar_voxel_indices(1)
    g = torch.Generator(device='cuda').manual_seed(3)
    feats = torch.randn(idx.size(0), 5, device='cuda', generator=g)
    net = encoder()
    with torch.no_grad():
        out = net(S.SparseConvTensor(feats, idx, SPARSE_SHAPE, 1))
        want, widx, wshape = reference_forward(ref, net, S.SparseConvTensor(feats, idx, SPARSE_SHAPE, 1))
    assert torch.equal(out.indices, widx) and list(out.spatial_shape) == list(wshape)
    assert torch.equal(out.features, want)
    assert set(out.indice_dict) == {'subm1', 'spconv2', 'subm2', 'out'}
    # the inverse convolution maps back onto the strided layer's inputs
    assert torch.equal(out.indices, out.indice_dict['out'][1])


def test_encoder_stack_backward(ref):
    """Gradients flow through the registered backward of every layer and
    equal those of a second identical stack (deterministic kernels)."""
    idx = lidar_voxel_indices(1)
    feats = torch.randn(idx.size(0), 5, device='cuda')
    grads = []
    for _ in range(2):
        net = encoder().train()
        x = feats.clone().requires_grad_(True)
        out = net(S.SparseConvTensor(x, idx, SPARSE_SHAPE, 1))
        out.features.square().sum().backward()
        grads.append([x.grad] + [p.grad for p in net.parameters()])
    assert all(gr is not None and bool(torch.isfinite(gr).all()) for gr in grads[0])
    assert all(torch.equal(a, b) for a, b in zip(*grads))


def test_maxpool_and_dense(ref):
    idx = lidar_voxel_indices(1)
    feats = torch.randn(idx.size(0), 8, device='cuda')
    x = S.SparseConvTensor(feats, idx, SPARSE_SHAPE, 1)
    y = S.SparseMaxPool3d(3, stride=2, padding=1)(x)
    outids, pairs, num = ref.get_indice_pairs(idx, 1, SPARSE_SHAPE, [3] * 3, [2] * 3, [1] * 3, [1] * 3, 0, False)
    assert torch.equal(y.indices, outids)
    assert torch.equal(y.features, ref.indice_maxpool(feats, pairs, num, outids.shape[0]))
    small = S.SparseConvTensor(feats[:100], idx[:100], SPARSE_SHAPE, 1)
    d = S.ToDense()(S.SparseSequential(S.SubMConv3d(8, 4, 1).cuda())(small))
    assert d.shape == (1, 4, *SPARSE_SHAPE)
    assert int((d.abs().sum(1) > 0).sum()) <= 100


def test_autocast_fp16_features_fp32_filters(ref):
    """Under autocast a layer computes in fp16 whatever its inputs' dtypes
    (the reference's matmul does) and returns the features' dtype; fp32
    parameters get gradients.  Outside autocast mismatched dtypes are
    refused, as a plain matmul refuses them."""
    idx = lidar_voxel_indices(1)
    net = S.SparseSequential(S.SubMConv3d(16, 32, 3, padding=1, indice_key='a'), nn.ReLU(),
                             S.SparseConv3d(32, 32, 3, stride=2, padding=1, indice_key='b')).cuda()
    x16 = torch.randn(idx.size(0), 16, device='cuda', dtype=torch.float16)
    with torch.autocast('cuda', dtype=torch.float16):
        out = net(S.SparseConvTensor(x16, idx, SPARSE_SHAPE, 1))
        out32 = net(S.SparseConvTensor(x16.float(), idx, SPARSE_SHAPE, 1))
    assert out.features.dtype == torch.float16 and out32.features.dtype == torch.float32
    # fp32 features under autocast: the same fp16 computation, returned in fp32
    torch.testing.assert_close(out32.features, out.features.float(), rtol=1e-2, atol=1e-2)
    out.features.float().square().mean().backward()
    assert all(p.grad is not None and p.grad.dtype == torch.float32 and bool(torch.isfinite(p.grad).all())
               for p in net.parameters())
    with pytest.raises(TypeError):
        net(S.SparseConvTensor(x16, idx, SPARSE_SHAPE, 1))


def _sites(ndim, shape, dense, seed):
    """(b, c0, ..) int32 rows: every cell of `shape`, or a seeded third of them."""
    grids = torch.meshgrid(*[torch.arange(s) for s in shape], indexing='ij')
    cells = torch.stack([g.reshape(-1) for g in grids], 1)
    if not dense:
        g = torch.Generator().manual_seed(seed)
        cells = cells[torch.randperm(cells.size(0), generator=g)[:max(2, cells.size(0) // 3)]]
    return torch.cat([torch.zeros(cells.size(0), 1, dtype=torch.long), cells], 1).int().cuda()


MODULE_CASES = [
    ('SparseConv', dict(kernel_size=1, bias=True)), ('SparseConv', dict(kernel_size=1, bias=False)),
    ('SparseConv', dict(kernel_size=3, padding=1, bias=True)), ('SubMConv', dict(kernel_size=1, bias=False)),
    ('SubMConv', dict(kernel_size=3, padding=1, bias=True)), ('SparseMaxPool', dict(kernel_size=2, stride=1, padding=1)),
]


@pytest.mark.parametrize('ndim', [2, 3])
@pytest.mark.parametrize('dense', [True, False], ids=['full', 'sparse'])
@pytest.mark.parametrize('kind,kw', MODULE_CASES, ids=[f'{k}-{i}' for i, (k, _) in enumerate(MODULE_CASES)])
def test_small_modules_vs_reference(ref, ndim, dense, kind, kw):
    """Forward and backward of one module on a small grid, against the
    reference's GPU functions called as its module would (fp32: 1e-5)."""
    shape = [3, 4] if ndim == 2 else [2, 3, 3]
    idx = _sites(ndim, shape, dense, seed=ndim * 10 + len(kind))
    torch.manual_seed(123)
    pool = kind == 'SparseMaxPool'
    ctor = getattr(S, f'{kind}{ndim}d')
    m = (ctor(**kw) if pool else ctor(3, 4, **kw)).cuda()
    x = torch.randn(idx.size(0), 3, device='cuda', requires_grad=True)
    out = m(S.SparseConvTensor(x, idx, shape, 1))
    out.features.sum().backward()
    ks = [kw['kernel_size']] * ndim
    st, pd = [kw.get('stride', 1)] * ndim, [kw.get('padding', 0)] * ndim
    subm = kind == 'SubMConv'
    xr = x.detach()
    if not pool and m.conv1x1:
        want = xr @ m.weight.detach().view(3, 4) + (m.bias.detach() if m.bias is not None else 0)
        wid = idx
    else:
        wid, pairs, num = ref.get_indice_pairs(idx, 1, shape, ks, st, pd, [1] * ndim, [0] * ndim, subm, False)
        if pool:
            want = ref.indice_maxpool(xr, pairs, num, wid.shape[0])
            gx_ref = ref.indice_maxpool_backward(xr, want, torch.ones_like(want), pairs, num)
        else:
            want = ref.indice_conv(xr, m.weight.detach(), pairs, num, wid.shape[0], False, subm)
            if m.bias is not None:
                want = want + m.bias.detach()
            gx_ref, gw_ref = ref.indice_conv_backward(xr, m.weight.detach(), torch.ones_like(want), pairs, num)
            torch.testing.assert_close(m.weight.grad, gw_ref.view_as(m.weight), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(x.grad, gx_ref, rtol=1e-5, atol=1e-5)
    assert torch.equal(out.indices, wid)
    torch.testing.assert_close(out.features, want, rtol=1e-5, atol=1e-5)
    if not pool and m.bias is not None:
        torch.testing.assert_close(m.bias.grad, torch.full_like(m.bias, float(out.features.size(0))))
