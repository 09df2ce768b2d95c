"""Sparse convolution and max-pooling over a rulebook on the GPU, against the
reference's own outputs (golden fixtures) and the numpy oracle at LiDAR
scale.

Tolerances: fp32 (fp32 FMA kernel) within 1e-5 of the reference / oracle;
fp16 and bf16 (tensor-core kernel: fp16/bf16 products, fp32 accumulation,
one rounding) within 1e-2 (fp16) / 2e-2 (bf16) relative to max(|ref|, 1), the
oracle computed in float64 from the same rounded inputs.  Max-pooling is
compared exactly.
"""
import ctypes

import numpy as np
import pytest
import torch

from bevfusion_triton_b200 import load_native
from bevfusion_triton_b200.ops.spconv import (fused_indice_conv, get_indice_pairs, indice_conv, indice_conv_backward,
                                              indice_maxpool, indice_maxpool_backward)
from bevfusion_triton_b200.ops.spconv import functional as F
from oracle import oracle
from tests.test_oracle_golden import spconv_conv_case
from tests.test_spconv_gpu import SPARSE_SHAPE, lidar_voxel_indices

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 2e-2}


def close(got, ref, dtype):
    got = got.float().cpu().numpy().astype(np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1.0)
    assert err.max(initial=0.0) <= TOL[dtype], f'max rel err {err.max()} > {TOL[dtype]}'


@pytest.fixture(scope='module')
def lidar_rulebooks():
    """Rulebooks of 2 synthetic LiDAR samples (about 95 k voxels each) on the
    sparse encoder's grid: submanifold 3x3x3, strided 3x3x3, (1, 1, 3)."""
    idx = lidar_voxel_indices(2)
    out = {}
    out['subm3'] = (idx.size(0),) + tuple(get_indice_pairs(idx, 2, SPARSE_SHAPE, ksize=3, padding=1, subm=True))
    out['down3'] = (idx.size(0),) + tuple(get_indice_pairs(idx, 2, SPARSE_SHAPE, ksize=3, stride=2, padding=1))
    out['out113'] = (idx.size(0),) + tuple(get_indice_pairs(idx, 2, SPARSE_SHAPE, ksize=(1, 1, 3),
                                                            stride=(1, 1, 2), padding=0))
    return out


@pytest.mark.parametrize('j', range(5))
def test_golden_fp32(cuda, golden, j):
    g = golden('spconv_conv_cases')
    rb = golden('spconv_cases')
    c, cin, cout, inverse, n_in, n_out = spconv_conv_case(g, j)
    pairs = torch.from_numpy(rb[f'c{c}_pairs']).cuda()
    num = torch.from_numpy(rb[f'c{c}_num']).cuda()
    t = {k: torch.from_numpy(g[f'v{j}_{k}']).cuda() for k in ('x', 'w', 'bias', 'gy')}
    f32 = torch.float32
    close(indice_conv(t['x'], t['w'], pairs, num, n_out, inverse), g[f'v{j}_y'], f32)
    close(fused_indice_conv(t['x'], t['w'], t['bias'], pairs, num, n_out, inverse, False), g[f'v{j}_yb'], f32)
    gx, gw = indice_conv_backward(t['x'], t['w'], t['gy'], pairs, num, inverse)
    close(gx, g[f'v{j}_gx'], f32)
    close(gw, g[f'v{j}_gw'], f32)
    if not inverse:
        xp, gyp = torch.from_numpy(g[f'v{j}_xp']).cuda(), torch.from_numpy(g[f'v{j}_gyp']).cuda()
        yp = indice_maxpool(xp, pairs, num, n_out)
        np.testing.assert_array_equal(yp.cpu().numpy(), g[f'v{j}_yp'])
        gxp = indice_maxpool_backward(xp, yp, gyp, pairs, num)
        np.testing.assert_array_equal(gxp.cpu().numpy(), g[f'v{j}_gxp'])


def _inputs(n_in, n_out, K, cin, cout, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n_in, cin, generator=g).to(dtype)
    w = (torch.randn(K, cin, cout, generator=g) / (cin * 3) ** 0.5).to(dtype)
    gy = torch.randn(n_out, cout, generator=g).to(dtype)
    return x.cuda(), w.cuda(), gy.cuda()


# (layer, cin, cout, dtype): the tensor-core path (fp16 / bf16, multiples of
# 16), its SIMT fallback (odd widths) and fp32
CASES = [
    ('subm3', 16, 16, torch.float16), ('subm3', 32, 64, torch.float16), ('subm3', 64, 64, torch.bfloat16),
    ('down3', 64, 128, torch.float16), ('subm3', 128, 128, torch.bfloat16), ('out113', 128, 256, torch.float16),
    ('subm3', 5, 16, torch.float16), ('subm3', 24, 40, torch.bfloat16),
    ('subm3', 16, 16, torch.float32), ('down3', 64, 64, torch.float32), ('subm3', 5, 16, torch.float32),
]


@pytest.mark.parametrize('layer,cin,cout,dtype', CASES,
                         ids=[f'{a}-{b}x{c}-{str(d)[6:]}' for a, b, c, d in CASES])
def test_lidar_scale_vs_oracle(cuda, lidar_rulebooks, layer, cin, cout, dtype):
    n_in, _, pairs, num = lidar_rulebooks[layer]
    outids = lidar_rulebooks[layer][1]
    n_out = outids.size(0)
    K = pairs.size(0)
    x, w, gy = _inputs(n_in, n_out, K, cin, cout, dtype, seed=cin * 1000 + cout)
    bias = torch.randn(cout, device='cuda').to(dtype)
    pr, nm = pairs.cpu().numpy(), num.cpu().numpy()
    xr, wr, gr = x.float().cpu().numpy(), w.float().cpu().numpy(), gy.float().cpu().numpy()
    y = indice_conv(x, w, pairs, num, n_out)
    close(y, oracle.indice_conv(xr, wr, pr, nm, n_out), dtype)
    yb = fused_indice_conv(x, w, bias, pairs, num, n_out, False, False)
    ref_b = oracle.indice_conv(xr, wr, pr, nm, n_out) + bias.float().cpu().numpy()
    close(yb, ref_b, dtype)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num)
    rgx, rgw = oracle.indice_conv_backward(xr, wr, gr, pr, nm)
    close(gx, rgx, dtype)
    # the filter gradient sums ~10^5 products per entry: scale by its magnitude
    scale = max(1.0, float(np.abs(rgw).max()))
    close(gw.float() / scale, rgw / scale, dtype)
    # deterministic: a second call gives the same bits
    assert torch.equal(indice_conv(x, w, pairs, num, n_out), y)
    gx2, gw2 = indice_conv_backward(x, w, gy, pairs, num)
    assert torch.equal(gx2, gx) and torch.equal(gw2, gw)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_inverse_conv_vs_oracle(cuda, lidar_rulebooks, dtype):
    """SparseInverseConv3d: the strided rulebook used with its slots swapped."""
    n_idx, outids, pairs, num = lidar_rulebooks['down3']
    n_in, n_out = outids.size(0), n_idx
    x, w, gy = _inputs(n_in, n_out, 27, 64, 32, dtype, seed=5)
    pr, nm = pairs.cpu().numpy(), num.cpu().numpy()
    y = indice_conv(x, w, pairs, num, n_out, inverse=True)
    close(y, oracle.indice_conv(x.float().cpu().numpy(), w.float().cpu().numpy(), pr, nm, n_out, True), dtype)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num, inverse=True)
    rgx, rgw = oracle.indice_conv_backward(x.float().cpu().numpy(), w.float().cpu().numpy(),
                                           gy.float().cpu().numpy(), pr, nm, True)
    close(gx, rgx, dtype)
    scale = max(1.0, float(np.abs(rgw).max()))
    close(gw.float() / scale, rgw / scale, dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_maxpool_lidar_scale_exact(cuda, lidar_rulebooks, dtype):
    n_in, outids, pairs, num = lidar_rulebooks['down3']
    n_out = outids.size(0)
    x, _, _ = _inputs(n_in, n_out, 1, 16, 1, dtype, seed=9)
    gy = torch.randn(n_out, 16, device='cuda').to(dtype)
    pr, nm = pairs.cpu().numpy(), num.cpu().numpy()
    y = indice_maxpool(x, pairs, num, n_out)
    npdt = {torch.float32: np.float32, torch.float16: np.float16, torch.bfloat16: np.float32}[dtype]
    ry = oracle.indice_maxpool(x.float().cpu().numpy().astype(npdt), pr, nm, n_out)
    np.testing.assert_array_equal(y.float().cpu().numpy(), ry.astype(np.float32))
    gx = indice_maxpool_backward(x, y, gy, pairs, num)
    if dtype != torch.bfloat16:  # numpy has no bfloat16 to round the sums in
        rgx = oracle.indice_maxpool_backward(x.cpu().numpy(), y.cpu().numpy(), gy.cpu().numpy(), pr, nm)
        np.testing.assert_array_equal(gx.cpu().numpy(), rgx)


def test_autograd_through_the_op(cuda, lidar_rulebooks):
    """functional.indice_subm_conv / indice_maxpool differentiate through the
    registered backward; the bias gradient is the column sum."""
    n_in, outids, pairs, num = lidar_rulebooks['subm3']
    x, w, gy = _inputs(n_in, n_in, 27, 32, 32, torch.float16, seed=3)
    xa, wa = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    y = F.indice_subm_conv(xa, wa, pairs, num, n_in)
    y.backward(gy)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num)
    assert torch.equal(xa.grad, gx) and torch.equal(wa.grad, gw)
    from bevfusion_triton_b200._lib import ops
    b = torch.randn(32, device='cuda', dtype=torch.float16, requires_grad=True)
    ops().indice_conv(x, w, pairs, num, n_in, False, b).backward(gy)
    torch.testing.assert_close(b.grad, gy.sum(0))
    xp = x.clone().requires_grad_(True)
    yp = F.indice_maxpool(xp, pairs, num, n_in)
    yp.backward(gy[:, :32])
    assert torch.equal(xp.grad, indice_maxpool_backward(x, yp.detach(), gy[:, :32], pairs, num))


def test_empty_rulebook_and_sizes(cuda):
    """No pairs: every output row is 0 (+ bias); no outputs; refused shapes."""
    x = torch.randn(50, 16, device='cuda', dtype=torch.float16)
    w = torch.randn(27, 16, 32, device='cuda', dtype=torch.float16)
    pairs = torch.full((27, 2, 50), -1, dtype=torch.int32, device='cuda')
    num = torch.zeros(27, dtype=torch.int32, device='cuda')
    y = indice_conv(x, w, pairs, num, 300)
    assert y.shape == (300, 32) and int(y.abs().sum()) == 0
    b = torch.randn(32, device='cuda', dtype=torch.float16)
    yb = fused_indice_conv(x, w, b, pairs, num, 300, False, False)
    assert torch.equal(yb, b.expand(300, 32))
    assert indice_conv(x, w, pairs, num, 0).shape == (0, 32)
    gx, gw = indice_conv_backward(x, w, torch.randn(300, 32, device='cuda', dtype=torch.float16), pairs, num)
    assert int(gx.abs().sum()) == 0 and int(gw.abs().sum()) == 0
    with pytest.raises(ValueError):
        indice_conv(x, w[:8], pairs, num, 10)  # 8 filter offsets against 27 rules
    with pytest.raises(TypeError):
        indice_conv(x, w.float(), pairs, num, 10)


def test_no_wait_gave_up(cuda, lidar_rulebooks):
    lib = load_native()
    n = ctypes.c_uint64(0)
    assert lib.bfb_spconv_timeouts(ctypes.byref(n), 0) == 0
    assert n.value == 0


def test_opcheck_spconv_ops(cuda, lidar_rulebooks):
    from bevfusion_triton_b200._lib import ops
    n_in, _, pairs, num = lidar_rulebooks['subm3']
    n = 3000
    p, m = pairs[:, :, :n].contiguous(), num.clamp(max=n)
    keep = (p[:, 0] < n) & (p[:, 1] < n)
    p = torch.where(keep.unsqueeze(1), p, torch.full_like(p, -1))  # pairs naming rows >= n are ignored anyway
    x, w, gy = _inputs(n, n, 27, 16, 16, torch.float16, seed=1)
    O = ops()
    torch.library.opcheck(O.indice_conv.default, (x, w, p, m, n, False, None), test_utils=('test_schema',
                                                                                           'test_faketensor'))
    torch.library.opcheck(O.indice_conv_backward.default, (x, w, gy, p, m, False),
                          test_utils=('test_schema', 'test_faketensor'))
    torch.library.opcheck(O.indice_maxpool.default, (x, p, m, n), test_utils=('test_schema', 'test_faketensor'))


def test_wide_channels_and_large_kernel(cuda):
    """Channel counts past the tensor-core shapes and a 5x5x5 kernel run on
    the FMA path (any width; kernel volume up to 7x7x7)."""
    idx = lidar_voxel_indices(1)[:20000].contiguous()
    outids, pairs, num = get_indice_pairs(idx, 1, SPARSE_SHAPE, ksize=5, padding=2, subm=True)
    n = idx.size(0)
    pr, nm = pairs.cpu().numpy(), num.cpu().numpy()
    for cin, cout, dtype in ((260, 300, torch.float32), (48, 272, torch.float16)):
        x, w, gy = _inputs(n, n, 125, cin, cout, dtype, seed=cin)
        y = indice_conv(x, w, pairs, num, n)
        close(y, oracle.indice_conv(x.float().cpu().numpy(), w.float().cpu().numpy(), pr, nm, n), dtype)
        gx, gw = indice_conv_backward(x, w, gy, pairs, num)
        rgx, rgw = oracle.indice_conv_backward(x.float().cpu().numpy(), w.float().cpu().numpy(),
                                               gy.float().cpu().numpy(), pr, nm)
        close(gx, rgx, dtype)
        scale = max(1.0, float(np.abs(rgw).max()))
        close(gw.float() / scale, rgw / scale, dtype)


@pytest.mark.parametrize('kind', ['transposed3d', 'dilated3d', 'conv2d'])
@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_other_rulebook_kinds_vs_oracle(cuda, kind, dtype):
    """Convolution over a transposed 3-D rulebook, a dilated submanifold one
    and a 2-D one (the bird's-eye plane of the LiDAR sites), forward and
    backward against the oracle."""
    idx = lidar_voxel_indices(1)[:30000].contiguous()
    if kind == 'transposed3d':
        shape = [720, 720, 21]
        idx = torch.cat([idx[:, :1], idx[:, 1:] // 2], 1).unique(dim=0).contiguous()
        outids, pairs, num = get_indice_pairs(idx, 1, shape, ksize=3, stride=2, padding=1, transpose=True)
    elif kind == 'dilated3d':
        outids, pairs, num = get_indice_pairs(idx, 1, SPARSE_SHAPE, ksize=3, padding=2, dilation=2, subm=True)
    else:
        idx = idx[:, :3].unique(dim=0).contiguous()
        outids, pairs, num = get_indice_pairs(idx, 1, SPARSE_SHAPE[:2], ksize=3, stride=2, padding=1)
    n_in, n_out, K = idx.size(0), outids.size(0), pairs.size(0)
    x, w, gy = _inputs(n_in, n_out, K, 32, 48, dtype, seed=K + n_in)
    pr, nm = pairs.cpu().numpy(), num.cpu().numpy()
    xr, wr, gr = x.float().cpu().numpy(), w.float().cpu().numpy(), gy.float().cpu().numpy()
    close(indice_conv(x, w, pairs, num, n_out), oracle.indice_conv(xr, wr, pr, nm, n_out), dtype)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num)
    rgx, rgw = oracle.indice_conv_backward(xr, wr, gr, pr, nm)
    close(gx, rgx, dtype)
    scale = max(1.0, float(np.abs(rgw).max()))
    close(gw.float() / scale, rgw / scale, dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_unaligned_feature_rows(cuda, lidar_rulebooks, dtype):
    """A contiguous feature view starting 1 element into its storage (not
    16-byte aligned) takes the paths without 16-byte loads: fp32 gives the
    same bits; 16-bit features leave the tensor cores for the FMA path (other
    summation order), within the 16-bit tolerance."""
    n_in, _, pairs, num = lidar_rulebooks['subm3']
    x, w, gy = _inputs(n_in, n_in, 27, 16, 32, dtype, seed=77)
    base = torch.empty(n_in * 16 + 1, device='cuda', dtype=dtype)
    xu = base[1:].view(n_in, 16)
    xu.copy_(x)
    assert xu.data_ptr() % 16 != 0 and xu.is_contiguous()
    y, yu = indice_conv(x, w, pairs, num, n_in), indice_conv(xu, w, pairs, num, n_in)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num)
    gxu, gwu = indice_conv_backward(xu, w, gy, pairs, num)
    if dtype == torch.float32:
        assert torch.equal(yu, y) and torch.equal(gxu, gx) and torch.equal(gwu, gw)
    else:
        close(yu, y.float().cpu().numpy(), dtype)
        close(gxu, gx.float().cpu().numpy(), dtype)
        scale = float(gw.float().abs().max())
        assert float((gwu.float() - gw.float()).abs().max()) <= 1e-2 * scale
