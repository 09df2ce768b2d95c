"""Parity against the reference's own Triton GPU path, run on the same B200.

The reference's Triton kernels (installed unmodified under baseline/_ref by
baseline/ref_triton.py) are the GPU-side oracle:

* ``bev_pool`` (ops/bev_pool/src/bev_pool_triton.py:219-227): its forward is
  one ``tl.atomic_add`` per element, so fp32 sums come in a run-dependent
  order; ours must agree within rtol = atol = 1e-5 (in cells of ~1000
  points that order alone exceeds 1e-5, so there both are held to the
  recursive-summation error bound around the fp64 sum).  fp16 features: the
  Triton atomics accumulate in fp16 while ours sums in fp32 and rounds once,
  so both are held to 1e-2 of an fp64 sum and ours must be the closer one.
  The backward is a gather in both, compared exactly.
* Division.  The Triton kernels divide fp32 with Triton's default ``/``,
  which is not correctly rounded, where the reference CPU fallback (the
  authority this library matches bit for bit, tested elsewhere) divides in
  IEEE fp32.  A point whose (p - min) / voxel_size lies within a few ulps of
  an integer can therefore land in the neighbouring voxel on the Triton path,
  and a mean gradient can differ in the last bit.  The voxel comparisons
  below run on clouds without such points (any axis quotient within 1e-4 of
  an integer removed) and check separately that every disagreement on the
  full cloud is such a point.
* ``hard_voxelize`` (ops/voxel/src/voxelization_triton.py:674-710,
  deterministic mode): voxel_num, coords and counts exact.  The Triton path
  fills a voxel's slots with ``tl.atomic_add`` (:295), so the order of the
  points inside a voxel, and which points survive in a voxel that overflows
  ``max_points``, vary run to run: voxels that do not overflow are compared
  as sets of rows, overflowing ones by membership of every stored row.
* ``dynamic_voxelize`` (:428-463): the Triton kernel leaves columns of an
  out-of-range row untouched, so valid rows are compared exactly and invalid
  rows by their first column (-1).
* dynamic scatter (ops/voxel/src/scatter_points_triton.py:253-424): coords,
  map and counts exact; max exact; sum / mean (atomics) within 1e-5; the
  backward exactly (mean: within 1 ulp, the division above).

* sparse convolution (ops/spconv/src/spconv_triton.py:981-1111): the
  reference loops over the rules on the host and scatter-adds each rule's
  matmul into the output, one rule after the other, so an output is the
  rule-ordered sum of per-rule dot products, which ours forms the same way
  for fp32: equal bit for bit.  fp16: the reference rounds every rule's
  partial to fp16 while ours accumulates in fp32 and rounds once, both
  within 1e-2.  Gradients within 1e-5 (fp32; the filter gradient's chunked
  sum order differs).  Max-pooling exact.

The reference Triton ``bev_pool`` has no bounds check (an out-of-grid
coordinate makes it write outside its output), so only in-grid coordinates
are given to it.
"""
import sys
from pathlib import Path

import pytest
import torch

from bevfusion_triton_b200.ops.bev_pool import bev_pool
from bevfusion_triton_b200.ops.voxel.voxel_layer import (dynamic_point_to_voxel_backward,
                                                         dynamic_point_to_voxel_forward, dynamic_voxelize,
                                                         hard_voxelize)
from tests import synth
from tests._util import rand_bev_case

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / 'baseline'))
import ref_triton  # noqa: E402

pytestmark = pytest.mark.gpu

FP32_TOL = dict(rtol=1e-5, atol=1e-5)


@pytest.fixture(scope='module')
def ref(cuda):
    why = ref_triton.available()
    if why:
        pytest.skip(why)
    return ref_triton.load()


def _fwd_bwd(fn, feats, coords, shape, up):
    x = feats.clone().requires_grad_(True)
    out = fn(x, coords, *shape)
    (out * up).sum().backward()
    torch.cuda.synchronize()
    return out.detach(), x.grad


@pytest.mark.parametrize('cdtype', [torch.int32, torch.int64])
def test_bev_pool_random_vs_triton(ref, cdtype):
    bev, _, _ = ref
    feats, coords = rand_bev_case(200_000, 80, 2, 2, 64, 64, seed=21, cdtype=cdtype)
    feats, coords = feats.cuda(), coords.cuda()
    shape = (2, 2, 64, 64)
    up = torch.randn((2, 80, 2, 64, 64), generator=torch.Generator().manual_seed(3)).cuda()
    a, ga = _fwd_bwd(bev_pool, feats, coords, shape, up)
    b, gb = _fwd_bwd(bev.bev_pool, feats, coords, shape, up)
    torch.testing.assert_close(a, b, **FP32_TOL)
    assert torch.equal(ga, gb)


def test_bev_pool_hot_cells_vs_triton(ref):
    """3000 extra points piled into three cells (~1000 N(0,1) values each).
    There the Triton atomics' run-dependent order alone moves a sum by more
    than 1e-5 (partial sums reach ~30, whose fp32 spacing is ~2e-6), so such
    a cell is held, for both implementations, to the worst-case error of a
    recursive fp32 sum of k terms in any order, gamma_(k-1) * sum |x_i|
    (gamma_m = m u / (1 - m u), u = 2^-24), around the fp64 sum.  All other
    cells: rtol = atol = 1e-5 between the two."""
    bev, _, _ = ref
    feats, coords = rand_bev_case(200_000, 80, 2, 2, 64, 64, seed=21, hot=3000)
    feats, coords = feats.cuda(), coords.cuda()
    shape = (2, 2, 64, 64)
    a = bev_pool(feats, coords, *shape)
    b = bev.bev_pool(feats, coords, *shape)
    ranks = ((coords[:, 3] * 2 + coords[:, 2]) * 64 + coords[:, 0]) * 64 + coords[:, 1]
    want = torch.zeros((2 * 2 * 64 * 64, 80), dtype=torch.float64, device='cuda').index_add_(0, ranks, feats.double())
    sabs = torch.zeros_like(want).index_add_(0, ranks, feats.double().abs())
    k = torch.zeros(2 * 2 * 64 * 64, dtype=torch.float64, device='cuda').index_add_(
        0, ranks, torch.ones_like(ranks, dtype=torch.float64))
    to5 = lambda t: t.view(2, 2, 64, 64, 80).permute(0, 4, 1, 2, 3)  # noqa: E731
    u = 2.0 ** -24
    m = (k - 1).clamp(min=0).unsqueeze(1)
    bound = to5(m * u / (1 - m * u) * sabs)
    want = to5(want)
    assert bool(((a.double() - want).abs() <= bound).all())
    assert bool(((b.double() - want).abs() <= bound).all())
    hot = to5(k.unsqueeze(1).expand(-1, 80)) > 100
    assert int(hot.sum()) == 3 * 80
    torch.testing.assert_close(a[~hot], b[~hot], **FP32_TOL)


def test_bev_pool_det_sample_vs_triton(ref):
    """One full det sample (1.77 M frustum points, 360 x 360 grid), fp32."""
    bev, _, _ = ref
    case = synth.det_bev_pool_case(1, device='cuda')
    shape = (case.B, case.D, case.H, case.W)
    up = torch.randn((case.B, case.feats.size(1), case.D, case.H, case.W),
                     generator=torch.Generator().manual_seed(4)).cuda()
    a, ga = _fwd_bwd(bev_pool, case.feats, case.coords, shape, up)
    b, gb = _fwd_bwd(bev.bev_pool, case.feats, case.coords, shape, up)
    torch.testing.assert_close(a, b, **FP32_TOL)
    assert torch.equal(ga, gb)


def test_bev_pool_fp16_vs_triton(ref):
    bev, _, _ = ref
    case = synth.det_bev_pool_case(1, device='cuda', dtype=torch.float16)
    shape = (case.B, case.D, case.H, case.W)
    ranks = ((case.coords[:, 3] * case.D + case.coords[:, 2]) * case.H + case.coords[:, 0]) * case.W + case.coords[:, 1]
    want = torch.zeros((case.B * case.D * case.H * case.W, case.feats.size(1)), dtype=torch.float64, device='cuda')
    want.index_add_(0, ranks, case.feats.double())
    want = want.view(case.B, case.D, case.H, case.W, -1).permute(0, 4, 1, 2, 3)
    a = bev_pool(case.feats, case.coords, *shape)
    b = bev.bev_pool(case.feats, case.coords, *shape)
    torch.cuda.synchronize()
    err_a = (a.double() - want).abs().max().item()
    err_b = (b.double() - want).abs().max().item()
    torch.testing.assert_close(a.double(), want, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(b.double(), want, rtol=1e-2, atol=1e-2)
    assert err_a <= err_b


def _hard_outputs(fn, pts, vs, cr, mp, mv):
    voxels = torch.zeros((mv, mp, pts.size(1)), dtype=pts.dtype, device='cuda')
    coors = torch.zeros((mv, 3), dtype=torch.int32, device='cuda')
    num = torch.zeros((mv,), dtype=torch.int32, device='cuda')
    vn = fn(pts, voxels, coors, num, vs, cr, mp, mv, 3, True)
    torch.cuda.synchronize()
    return voxels, coors, num, int(vn)


def _edge_dist(pts, vs, cr):
    """Per point, the smallest distance over x, y, z of the fp64 quotient
    (p - min) / voxel_size to an integer."""
    q = (pts[:, :3].double() - torch.tensor(cr[:3], dtype=torch.float64, device=pts.device)) / \
        torch.tensor(vs, dtype=torch.float64, device=pts.device)
    return (q - q.round()).abs().min(1).values


EDGE = 1e-4


@pytest.mark.parametrize('sample', [0, 1])
def test_hard_voxelize_lidar_vs_triton(ref, sample):
    _, vox, _ = ref
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    pts = synth.lidar_sweeps(sample).cuda()
    pts = pts[_edge_dist(pts, vs, cr) > EDGE].contiguous()
    mp, mv = synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS
    v, c, n, vn = _hard_outputs(hard_voxelize, pts, vs, cr, mp, mv)
    rv, rc, rn, rvn = _hard_outputs(vox.hard_voxelize, pts, vs, cr, mp, mv)
    assert vn == rvn and vn > 0
    assert torch.equal(c, rc) and torch.equal(n, rn)
    # rows past voxel_num are zero in both
    assert not v[vn:].any() and not rv[vn:].any()
    # per-voxel contents: sets of rows for voxels that kept every point
    cnt = torch.zeros(vn, dtype=torch.int64, device='cuda')
    cells = torch.floor((pts[:, :3] - torch.tensor(cr[:3], device='cuda')) /
                        torch.tensor(vs, device='cuda')).long()
    grid = [round((cr[3 + i] - cr[i]) / vs[i]) for i in range(3)]
    inr = ((cells >= 0) & (cells < torch.tensor(grid, device='cuda'))).all(1)
    key = (cells[:, 0] * grid[1] + cells[:, 1]) * grid[2] + cells[:, 2]
    vkey = (c[:vn, 0].long() * grid[1] + c[:vn, 1].long()) * grid[2] + c[:vn, 2].long()
    order = torch.argsort(vkey)
    pos = torch.searchsorted(vkey[order], key[inr])
    pos = pos.clamp(max=vn - 1)
    hit = vkey[order][pos] == key[inr]
    cnt.index_add_(0, order[pos[hit]], torch.ones_like(pos[hit]))
    full = cnt <= mp  # the voxel stored all of its points
    assert torch.equal(cnt.clamp(max=mp).to(torch.int32), n[:vn])

    def row_sets(vx, sel):
        rows = vx[:vn][sel]  # [m, P, F]
        # sort each voxel's rows lexicographically (zero padding rows sort first)
        m, P, F = rows.shape
        keyed = rows.double()
        for f in reversed(range(F)):
            idx = torch.argsort(keyed[:, :, f], dim=1, stable=True)
            keyed = torch.gather(keyed, 1, idx.unsqueeze(-1).expand(-1, -1, F))
        return keyed

    assert torch.equal(row_sets(v, full), row_sets(rv, full))
    # overflowing voxels: every stored Triton row lies in its voxel
    over = torch.nonzero(~full).squeeze(1)
    if over.numel():
        rows = rv[over]  # [m, P, F], all P slots filled
        rc3 = torch.floor((rows[..., :3] - torch.tensor(cr[:3], device='cuda')) /
                          torch.tensor(vs, device='cuda')).to(torch.int32)
        assert torch.equal(rc3, c[over].unsqueeze(1).expand_as(rc3))


def test_hard_voxelize_full_cloud_differs_only_at_voxel_edges(ref):
    _, vox, _ = ref
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    pts = synth.lidar_sweeps(0).cuda()
    mp, mv = synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS
    _, _, _, vn = _hard_outputs(hard_voxelize, pts, vs, cr, mp, mv)
    _, _, _, rvn = _hard_outputs(vox.hard_voxelize, pts, vs, cr, mp, mv)
    near = int((_edge_dist(pts, vs, cr) <= EDGE).sum())
    assert abs(vn - rvn) <= near


def test_dynamic_voxelize_vs_triton(ref):
    _, vox, _ = ref
    pts = synth.lidar_sweeps(0).cuda()
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    a = torch.zeros((pts.size(0), 3), dtype=torch.int32, device='cuda')
    b = torch.zeros_like(a)
    dynamic_voxelize(pts, a, vs, cr, 3)
    vox.dynamic_voxelize(pts, b, vs, cr, 3)
    torch.cuda.synchronize()
    # ours is the IEEE fp32 floor((p - min) / size) of the reference CPU path
    ieee = torch.floor((pts[:, :3] - torch.tensor(cr[:3], device='cuda')) / torch.tensor(vs, device='cuda'))
    grid = torch.tensor([round((cr[3 + i] - cr[i]) / vs[i]) for i in range(3)], device='cuda')
    inr = ((ieee >= 0) & (ieee < grid)).all(1)
    assert torch.equal(a[inr], ieee[inr].to(torch.int32))
    assert bool((a[~inr] == -1).all())
    # Triton: equal on every point away from a voxel edge
    far = _edge_dist(pts, vs, cr) > EDGE
    valid = b[:, 0] != -1
    assert torch.equal((a[:, 0] != -1)[far], valid[far])
    assert torch.equal(a[far & valid], b[far & valid])
    differ = (a != b).any(1) & valid
    assert int(differ.sum()) <= int((~far).sum()) and not bool((differ & far).any())


@pytest.mark.parametrize('red', ['sum', 'mean', 'max'])
def test_dynamic_scatter_vs_triton(ref, red):
    _, _, sc = ref
    g = torch.Generator().manual_seed(12)
    n, C = 60_000, 16
    f = torch.randn((n, C), generator=g).cuda()
    c = torch.randint(-1, 30, (n, 3), generator=g).to(torch.int32).cuda()
    a = dynamic_point_to_voxel_forward(f, c, red)
    b = sc.dynamic_point_to_voxel_forward(f, c, red)
    torch.cuda.synchronize()
    m = b[1].size(0)
    assert torch.equal(a[1][:m], b[1]) and a[1].size(0) == m
    assert torch.equal(a[2], b[2]) and torch.equal(a[3], b[3])
    if red == 'max':
        assert torch.equal(a[0], b[0])
    else:
        torch.testing.assert_close(a[0], b[0], **FP32_TOL)
    up = torch.randn((m, C), generator=g).cuda()
    ga = torch.empty_like(f)
    gb = torch.empty_like(f)
    dynamic_point_to_voxel_backward(ga, up, f, b[0], b[2], b[3], red)
    sc.dynamic_point_to_voxel_backward(gb, up, f, b[0], b[2], b[3], red)
    torch.cuda.synchronize()
    if red == 'mean':  # Triton's fp32 division is not correctly rounded
        torch.testing.assert_close(ga, gb, rtol=2.5e-7, atol=0)
        want = up[b[2].clamp(min=0).long()] / b[3][b[2].clamp(min=0).long()].unsqueeze(1).float()
        want[b[2] < 0] = 0
        assert torch.equal(ga, want)  # IEEE division, as the reference CPU path
    else:
        assert torch.equal(ga, gb)


@pytest.fixture(scope='module')
def ref_spconv(cuda):
    why = ref_triton.available()
    if why:
        pytest.skip(why)
    try:
        return ref_triton.load_spconv()
    except RuntimeError as e:
        pytest.skip(str(e))


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('layer', ['subm', 'down'])
def test_sparse_conv_vs_reference_gpu(ref_spconv, dtype, layer):
    from bevfusion_triton_b200.ops.spconv import (get_indice_pairs, indice_conv, indice_conv_backward, indice_maxpool,
                                                  indice_maxpool_backward)
    from tests.test_spconv_gpu import SPARSE_SHAPE, lidar_voxel_indices
    idx = lidar_voxel_indices(1)
    kw = dict(ksize=3, padding=1, subm=True) if layer == 'subm' else dict(ksize=3, stride=2, padding=1)
    outids, pairs, num = get_indice_pairs(idx, 1, SPARSE_SHAPE, **kw)
    n_in, n_out = idx.size(0), outids.size(0)
    g = torch.Generator(device='cuda').manual_seed(13)
    x = torch.randn(n_in, 32, device='cuda', generator=g).to(dtype)
    w = (torch.randn(27, 32, 64, device='cuda', generator=g) / 30).to(dtype)
    gy = torch.randn(n_out, 64, device='cuda', generator=g).to(dtype)
    y, yr = indice_conv(x, w, pairs, num, n_out), ref_spconv.indice_conv(x, w, pairs, num, n_out)
    gx, gw = indice_conv_backward(x, w, gy, pairs, num)
    gxr, gwr = ref_spconv.indice_conv_backward(x, w, gy, pairs, num)
    if dtype == torch.float32:
        assert torch.equal(y, yr)
        torch.testing.assert_close(gx, gxr, **FP32_TOL)
        scale = float(gwr.abs().max())
        torch.testing.assert_close(gw / scale, gwr / scale, **FP32_TOL)
    else:
        for a, b in ((y, yr), (gx, gxr)):
            assert float(((a.float() - b.float()).abs() / b.float().abs().clamp(min=1.0)).max()) <= 1e-2
        scale = float(gwr.float().abs().max())
        assert float((gw.float() - gwr.float()).abs().max()) <= 1e-2 * scale
    p, pr = indice_maxpool(x, pairs, num, n_out), ref_spconv.indice_maxpool(x, pairs, num, n_out)
    assert torch.equal(p, pr)
    gp = indice_maxpool_backward(x, p, gy[:, :32].contiguous(), pairs, num)
    gpr = ref_spconv.indice_maxpool_backward(x, pr, gy[:, :32].contiguous(), pairs, num)
    if dtype == torch.float32:
        torch.testing.assert_close(gp, gpr, **FP32_TOL)
    else:
        torch.testing.assert_close(gp, gpr, rtol=1e-2, atol=1e-2)
