"""Voxelisation and dynamic scatter on the GPU against the reference's golden
outputs and the CPU oracle.  Voxel coordinates, counts, per-voxel point order
and stored features are compared bit for bit."""
import numpy as np
import pytest
import torch

from tests import synth
from bevfusion_triton_b200.ops.voxel import DynamicScatter, Voxelization, dynamic_scatter, voxelization, voxelize_batch
from bevfusion_triton_b200.ops.voxel.voxel_layer import (dynamic_point_to_voxel_backward,
                                                         dynamic_point_to_voxel_forward, dynamic_voxelize,
                                                         hard_voxelize, hard_voxelize_batch)
from oracle import oracle
from tests._util import sha

pytestmark = pytest.mark.gpu

VS8, CR8 = [1.0, 1.0, 1.0], [0.0, 0.0, 0.0, 4.0, 4.0, 4.0]


def run_hard(points, vsize, crange, mp, mv, fill=None, deterministic=True):
    dev = 'cuda'
    pts = points.to(dev)
    n = pts.size(0)
    P = n if mp == -1 else mp
    MV = n if mv == -1 else mv
    mk = (lambda shape, dt: torch.full(shape, fill, dtype=dt, device=dev)) if fill is not None else \
        (lambda shape, dt: torch.zeros(shape, dtype=dt, device=dev))
    voxels = mk((MV, P, pts.size(1)), pts.dtype)
    coors = mk((MV, 3), torch.int32)
    num = mk((MV,), torch.int32)
    vn = hard_voxelize(pts, voxels, coors, num, vsize, crange, mp, mv, 3, deterministic)
    return voxels.cpu(), coors.cpu(), num.cpu(), vn


def assert_hard_equal(got, ref):
    v, c, n, vn = got
    rv, rc, rn, rvn = ref
    assert vn == rvn
    np.testing.assert_array_equal(c.numpy(), np.asarray(rc))
    np.testing.assert_array_equal(n.numpy(), np.asarray(rn))
    np.testing.assert_array_equal(v.float().numpy(), np.asarray(rv, dtype=np.float32))


def test_dynamic_voxelize_golden(cuda, golden):
    g = golden('voxel_points8')
    c = torch.zeros((8, 3), dtype=torch.int32, device='cuda')
    dynamic_voxelize(torch.from_numpy(g['points']).cuda(), c, VS8, CR8, 3)
    np.testing.assert_array_equal(c.cpu().numpy(), g['dyn_coors'])
    g = golden('voxel_rand_noncubic')
    c = torch.zeros((g['points'].shape[0], 3), dtype=torch.int32, device='cuda')
    dynamic_voxelize(torch.from_numpy(g['points']).cuda(), c, g['vsize'].tolist(), g['crange'].tolist(), 3)
    np.testing.assert_array_equal(c.cpu().numpy(), g['dyn_coors'])


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16])
def test_dynamic_voxelize_low_precision(cuda, golden, dtype):
    g = golden('voxel_rand_noncubic')
    pts = torch.from_numpy(g['points']).to(dtype)
    c = torch.zeros((pts.size(0), 3), dtype=torch.int32, device='cuda')
    dynamic_voxelize(pts.cuda(), c, g['vsize'].tolist(), g['crange'].tolist(), 3)
    ref = oracle.dynamic_voxelize(pts.float().numpy(), g['vsize'], g['crange'])
    np.testing.assert_array_equal(c.cpu().numpy(), ref)


@pytest.mark.parametrize('mp,mv', [(2, 8), (3, 8), (1, 2)])
@pytest.mark.parametrize('deterministic', [True, False])
def test_hard_voxelize_points8(cuda, golden, mp, mv, deterministic):
    g = golden('voxel_points8')
    k = f'mp{mp}_mv{mv}'
    got = run_hard(torch.from_numpy(g['points']), VS8, CR8, mp, mv, deterministic=deterministic)
    assert_hard_equal(got, (g[f'{k}_voxels'], g[f'{k}_coors'], g[f'{k}_num'], int(g[f'{k}_vn'])))


@pytest.mark.parametrize('mp,mv', [(5, 300), (5, 100000), (32, 50)])
def test_hard_voxelize_noncubic(cuda, golden, mp, mv):
    g = golden('voxel_rand_noncubic')
    k = f'mp{mp}_mv{mv}'
    got = run_hard(torch.from_numpy(g['points']), g['vsize'].tolist(), g['crange'].tolist(), mp, mv, fill=7)
    assert_hard_equal(got, (g[f'{k}_voxels'], g[f'{k}_coors'], g[f'{k}_num'], int(g[f'{k}_vn'])))


def test_hard_voxelize_lidar_full_size_digest(cuda, digests):
    """Config 3 (346,880 points, 1440 x 1440 x 40 grid): equal to the
    reference CPU path's output bit for bit."""
    d = digests['lidar_s0']
    pts = synth.lidar_sweeps(0)
    assert sha(pts) == d['points_sha']
    for _ in range(2):  # second call checks that the hash table was left clean
        v, c, n, vn = run_hard(pts, list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE), synth.LIDAR_MAX_POINTS,
                               synth.LIDAR_MAX_VOXELS, fill=3)
        assert vn == d['voxel_num']
        assert sha(c[:vn]) == d['coors_sha'] and sha(n[:vn]) == d['num_sha'] and sha(v[:vn]) == d['voxels_sha']
        assert not v[vn:].any() and not c[vn:].any() and not n[vn:].any()


@pytest.mark.parametrize('mp,mv', [(-1, 64), (4, -1), (3, 5)])
@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_hard_voxelize_random_vs_oracle(cuda, mp, mv, dtype):
    g = torch.Generator().manual_seed(mp * 7 + mv)
    n = 1500
    pts = torch.rand((n, 4), generator=g) * torch.tensor([6.0, 5.0, 3.0, 1.0]) - torch.tensor([3.0, 2.5, 1.5, 0.0])
    pts[::5, :3] = pts[0, :3]  # one crowded voxel
    pts = pts.to(dtype)
    vs, cr = [0.5, 0.5, 0.75], [-2.5, -2.0, -1.5, 2.5, 2.0, 1.5]
    got = run_hard(pts, vs, cr, mp, mv)
    ref = oracle.hard_voxelize(pts.float().numpy(), vs, cr, mp if mp != -1 else n, mv)
    rv, rc, rn, rvn = ref
    v, c, nn, vn = got
    assert vn == rvn
    np.testing.assert_array_equal(c[:vn].numpy(), rc[:vn])
    np.testing.assert_array_equal(nn[:vn].numpy(), rn[:vn])
    np.testing.assert_array_equal(v[:vn].float().numpy(), rv[:vn])


def test_hard_voxelize_empty_and_all_outside(cuda):
    for pts in (torch.zeros((0, 4)), torch.full((50, 4), 100.0)):
        v, c, n, vn = run_hard(pts, VS8, CR8, 3, 8, fill=9)
        assert vn == 0
        assert not v.any() and not c.any() and not n.any()


def test_voxelization_module_matches_function(cuda, golden):
    g = golden('voxel_points8')
    pts = torch.from_numpy(g['points']).cuda()
    m = Voxelization(voxel_size=VS8, point_cloud_range=CR8, max_num_points=3, max_voxels=8, deterministic=True)
    m.eval()
    a = m(pts)
    b = voxelization(pts, VS8, CR8, 3, 8, True)
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    k = 'mp3_mv8'
    vn = int(g[f'{k}_vn'])
    np.testing.assert_array_equal(a[0].cpu().numpy(), g[f'{k}_voxels'][:vn])
    np.testing.assert_array_equal(a[1].cpu().numpy(), g[f'{k}_coors'][:vn])
    dyn = voxelization(pts, VS8, CR8, -1, -1, True)
    np.testing.assert_array_equal(dyn.cpu().numpy(), g['dyn_coors'])


def test_hard_voxelize_batch_matches_single(cuda):
    clouds = [synth.lidar_sweeps(s)[: 50000 + 7000 * s] for s in range(3)] + [torch.zeros((0, 5))]
    clouds = [clouds[0], clouds[3], clouds[1], clouds[2]]  # an empty sample in the middle
    offs = [0]
    for c in clouds:
        offs.append(offs[-1] + c.size(0))
    pts = torch.cat(clouds).cuda()
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    V, C, N, VN = hard_voxelize_batch(pts, offs, vs, cr, 10, 20000)
    for s, cl in enumerate(clouds):
        v, c, n, vn = run_hard(cl, vs, cr, 10, 20000)
        assert int(VN[s]) == vn
        assert torch.equal(V[s, :vn].cpu(), v[:vn]) and torch.equal(C[s, :vn].cpu(), c[:vn])
        assert torch.equal(N[s, :vn].cpu(), n[:vn])


def test_hard_voxelize_batch_many_samples(cuda):
    """70 samples: the per-call offset and tile tables (2 x 71 words) go to
    the device in more than one parameter upload; every sample still matches
    its single-sample result."""
    clouds = [synth.lidar_sweeps(s % 5)[: 300 + 97 * s] for s in range(70)]
    offs = [0]
    for c in clouds:
        offs.append(offs[-1] + c.size(0))
    pts = torch.cat(clouds).cuda()
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    V, C, N, VN = hard_voxelize_batch(pts, offs, vs, cr, 10, 2000)
    for s in (0, 1, 63, 64, 69):
        v, c, n, vn = run_hard(clouds[s], vs, cr, 10, 2000)
        assert int(VN[s]) == vn
        assert torch.equal(V[s, :vn].cpu(), v[:vn]) and torch.equal(C[s, :vn].cpu(), c[:vn])
        assert torch.equal(N[s, :vn].cpu(), n[:vn])


def test_hard_voxelize_batch_graph_capture(cuda):
    """The batched call issues no host copy or synchronisation, so it can be
    captured into a CUDA graph; replays over new points in the same buffers
    give the eager results."""
    from bevfusion_triton_b200._lib import ops
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    sizes = [40000, 0, 35000]
    offs = [0, 40000, 40000, 75000]
    pts = torch.empty((75000, 5), device='cuda')
    outs = (torch.empty((3, 8000, 10, 5), device='cuda'), torch.empty((3, 8000, 3), dtype=torch.int32, device='cuda'),
            torch.empty((3, 8000), dtype=torch.int32, device='cuda'), torch.empty((3,), dtype=torch.int32, device='cuda'))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):  # warm-up on the capture stream: its hash table is made here
            ops().hard_voxelize_batch(pts.zero_(), offs, *outs, vs, cr, 10, 8000, True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        ops().hard_voxelize_batch(pts, offs, *outs, vs, cr, 10, 8000, True)
    for seed in (3, 4):
        pts.copy_(torch.cat([synth.lidar_sweeps(seed)[:40000], synth.lidar_sweeps(seed + 1)[:35000]]).cuda())
        g.replay()
        torch.cuda.synchronize()
        V, C, N, VN = hard_voxelize_batch(pts, offs, vs, cr, 10, 8000, True)
        assert torch.equal(VN, outs[3]) and torch.equal(C, outs[1]) and torch.equal(N, outs[2])
        assert torch.equal(V, outs[0])
    assert int(outs[3][1]) == 0 and sizes[1] == 0


def test_voxelize_batch_mean_features(cuda):
    """The one-launch epilogue against the reference composition
    (models/fusion_models/bevfusion.py:269-296: per-sample voxelisation, batch
    index padded on, concatenated, feats.sum(1) / num_points): coords and
    sizes bit-exact; the mean equals a sequential fp32 sum over the point slots
    divided once by the count bit for bit, and the torch composition within
    1e-6 (its reduction may associate the slot sum differently)."""
    clouds = [synth.lidar_sweeps(s)[:30000].cuda() for s in range(3)]
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    feats, coords, sizes = voxelize_batch(clouds, vs, cr, 10, 12000)
    rf, rc, rs = [], [], []
    for b, c in enumerate(clouds):
        v, cc, nn = voxelization(c, vs, cr, 10, 12000, True)
        rf.append(v)
        rc.append(torch.nn.functional.pad(cc, (1, 0), mode='constant', value=b))
        rs.append(nn)
    rs = torch.cat(rs)
    rv = torch.cat(rf)
    assert torch.equal(coords, torch.cat(rc)) and torch.equal(sizes, rs)
    seq = np.zeros((rv.size(0), rv.size(2)), dtype=np.float32)
    rvn = rv.cpu().numpy()
    for j in range(rv.size(1)):
        seq = (seq + rvn[:, j]).astype(np.float32)
    seq = seq / rs.cpu().numpy().astype(np.float32)[:, None]
    np.testing.assert_array_equal(feats.cpu().numpy(), seq)
    ref = rv.sum(1) / rs.to(torch.float32).unsqueeze(1)
    torch.testing.assert_close(feats, ref, rtol=1e-6, atol=1e-6)
    # unreduced rows
    f2, c2, s2 = voxelize_batch(clouds, vs, cr, 10, 12000, reduce_mean=False)
    assert torch.equal(f2, rv) and torch.equal(c2, coords) and torch.equal(s2, sizes)


def test_voxelize_batch_empty_sample_and_cap(cuda):
    """A sample without points, and max_voxels reached: packing stays right."""
    clouds = [synth.lidar_sweeps(0)[:20000].cuda(), torch.empty((0, 5), device='cuda'),
              synth.lidar_sweeps(1)[:20000].cuda()]
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    feats, coords, sizes = voxelize_batch(clouds, vs, cr, 5, 3000)
    rc = []
    for b, c in enumerate(clouds):
        if c.size(0) == 0:
            continue
        _, cc, _ = voxelization(c, vs, cr, 5, 3000, True)
        rc.append(torch.nn.functional.pad(cc, (1, 0), mode='constant', value=b))
    assert torch.equal(coords, torch.cat(rc))
    assert coords.size(0) == 6000 and int(sizes.max()) <= 5


# ----------------------------------------------------------------- scatter
@pytest.mark.parametrize('case', ['fix', 'rand'])
@pytest.mark.parametrize('red', ['sum', 'mean', 'max'])
def test_dynamic_scatter_golden(cuda, golden, case, red):
    g = golden('scatter_cases')
    f = torch.from_numpy(g[f'{case}_feats']).cuda()
    c = torch.from_numpy(g[f'{case}_coors']).cuda()
    vf, vc, mp, cnt = dynamic_point_to_voxel_forward(f, c, red)
    np.testing.assert_array_equal(vc.cpu().numpy(), g[f'{case}_{red}_vc'])
    np.testing.assert_array_equal(mp.cpu().numpy(), g[f'{case}_{red}_map'])
    np.testing.assert_array_equal(cnt.cpu().numpy(), g[f'{case}_{red}_cnt'])
    np.testing.assert_array_equal(vf.cpu().numpy(), g[f'{case}_{red}_vf'])
    gf = torch.zeros_like(f)
    dynamic_point_to_voxel_backward(gf, torch.from_numpy(g[f'{case}_{red}_up']).cuda(), f, vf, mp, cnt, red)
    np.testing.assert_array_equal(gf.cpu().numpy(), g[f'{case}_{red}_grad'])


@pytest.mark.parametrize('red', ['sum', 'mean', 'max'])
@pytest.mark.parametrize('dtype', [torch.float32, torch.float16, torch.bfloat16])
def test_dynamic_scatter_random_vs_oracle(cuda, red, dtype):
    g = torch.Generator().manual_seed(11)
    n, C = 5000, 37
    f = torch.randn((n, C), generator=g).to(dtype)
    c = torch.randint(-1, 40, (n, 3), generator=g).to(torch.int32)
    x = f.cuda().requires_grad_(True)
    vf, vc = dynamic_scatter(x, c.cuda(), red)
    rf, rc, rm, rcnt = oracle.dynamic_scatter(f.float().numpy(), c.numpy(), red)
    np.testing.assert_array_equal(vc.cpu().numpy(), rc)
    tol = dict(rtol=0, atol=0) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    np.testing.assert_allclose(vf.detach().float().cpu().numpy(), rf, **tol)
    up = torch.linspace(0.1, 1.0, vf.numel(), device='cuda', dtype=vf.dtype).view_as(vf)
    (vf * up).sum().backward()
    rg = oracle.dynamic_scatter_backward(up.float().cpu().numpy(), f.float().numpy(),
                                         vf.detach().float().cpu().numpy(), rm, rcnt, red)
    np.testing.assert_allclose(x.grad.float().cpu().numpy(), rg, **tol)


def test_dynamic_scatter_module(cuda, golden):
    g = golden('scatter_cases')
    f = torch.from_numpy(g['fix_feats']).cuda()
    c = torch.from_numpy(g['fix_coors']).cuda()
    m = DynamicScatter(VS8, CR8, average_points=True)
    a = m(f, c)
    b = dynamic_scatter(f, c, 'mean')
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    # batched form: (b, x, y, z) rows
    cb = torch.cat([torch.zeros((c.size(0), 1), dtype=torch.int32, device='cuda'), c], 1)
    cb = torch.cat([cb, cb.clone().index_fill_(1, torch.tensor([0], device='cuda'), 1)])
    fb = torch.cat([f, f * 2])
    ob, ocb = m(fb, cb)
    assert ob.shape[0] == 2 * b[0].shape[0] and torch.equal(ocb[:, 1:], torch.cat([b[1], b[1]]))


def _lidar_rows(samples):
    """(b, x, y, z) int32 rows and 5 features of `samples` LiDAR clouds on
    the config-3 grid (out-of-range points keep their -1 rows)."""
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    feats, rows = [], []
    for b in range(samples):
        p = synth.lidar_sweeps(b).cuda()
        c = torch.empty((p.size(0), 3), dtype=torch.int32, device='cuda')
        dynamic_voxelize(p, c, vs, cr, 3)
        rows.append(torch.cat((torch.full((p.size(0), 1), b, dtype=torch.int32, device='cuda'), c), 1))
        feats.append(p)
    return torch.cat(feats), torch.cat(rows)


@pytest.mark.parametrize('red', ['sum', 'mean', 'max'])
def test_dynamic_scatter_batch16_wide_keys(cuda, red):
    """16 samples of (b, x, y, z) rows on the 1440 x 1440 x 40 grid need a
    32-bit row key (4 + 11 + 11 + 6 bits), past the one-word sort: the wide
    path must equal sample-by-sample calls (one-word keys) bit for bit,
    forward and backward, and so must the single module call."""
    feats, rows = _lidar_rows(16)
    x = feats.clone().requires_grad_(True)
    vf, vc = dynamic_scatter(x, rows, red)
    up = torch.randn(vf.shape, generator=torch.Generator().manual_seed(2)).cuda()
    (vf * up).sum().backward()
    wf, wc, wg, off = [], [], torch.zeros_like(feats), 0
    for b in range(16):
        sel = torch.nonzero(rows[:, 0] == b).squeeze(1)
        xb = feats[sel].clone().requires_grad_(True)
        f, c = dynamic_scatter(xb, rows[sel, 1:], red)
        (f * up[off:off + f.size(0)]).sum().backward()
        off += f.size(0)
        wf.append(f.detach())
        wc.append(torch.cat((torch.full((c.size(0), 1), b, dtype=torch.int32, device='cuda'), c), 1))
        wg[sel] = xb.grad
    assert off == vf.size(0)
    assert torch.equal(vc, torch.cat(wc)) and torch.equal(vf.detach(), torch.cat(wf))
    assert torch.equal(x.grad, wg)
    m = DynamicScatter(list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE), average_points=(red == 'mean'))
    if red in ('mean', 'max'):
        mf, mc = m(feats, rows)
        assert torch.equal(mf, vf.detach()) and torch.equal(mc, vc)


def test_dynamic_scatter_extents(cuda):
    """Known extents pack the keys without the coordinate pass: same result;
    a valid row beyond an extent is refused."""
    feats, rows = _lidar_rows(3)
    a = dynamic_point_to_voxel_forward(feats, rows, 'mean')
    b = dynamic_point_to_voxel_forward(feats, rows, 'mean', extents=[3, 1440, 1440, 40])
    for u, v in zip(a, b):
        assert torch.equal(u, v)
    with pytest.raises(ValueError, match='beyond the given extents'):
        dynamic_point_to_voxel_forward(feats, rows, 'mean', extents=[2, 1440, 1440, 40])


def test_opcheck_voxel_ops(cuda):
    """torch.library.opcheck on the voxel ops: the schemas declare exactly
    the buffers the kernels write, and the fake kernels match."""
    O = torch.ops.bfb_b200
    pts = synth.lidar_sweeps(0)[:5000].cuda()
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
    coors = torch.empty((5000, 3), dtype=torch.int32, device='cuda')
    torch.library.opcheck(O.dynamic_voxelize, (pts, coors, vs, cr), test_utils=('test_schema', 'test_faketensor'))
    vox = torch.zeros((4000, 10, 5), device='cuda')
    co = torch.zeros((4000, 3), dtype=torch.int32, device='cuda')
    num = torch.zeros((4000,), dtype=torch.int32, device='cuda')
    torch.library.opcheck(O.hard_voxelize, (pts, vox, co, num, vs, cr, 10, 4000, True), test_utils=('test_schema',))
    f = torch.randn((5000, 8), device='cuda', requires_grad=True)
    c = torch.randint(0, 20, (5000, 3), dtype=torch.int32, device='cuda')
    torch.library.opcheck(O.dynamic_scatter_forward, (f, c, 'max', None),
                          test_utils=('test_schema', 'test_autograd_registration'))


def test_legacy_import_path(cuda, golden):
    """ops.voxel.voxel_layer_legacy (the compiled extension's import name and
    positional signatures) runs the same ops."""
    from bevfusion_triton_b200.ops.voxel import voxel_layer_legacy as legacy
    g = golden('voxel_points8')
    pts = torch.from_numpy(g['points']).cuda()
    a = [torch.zeros((64, 5, pts.size(1)), device='cuda'), torch.zeros((64, 3), dtype=torch.int32, device='cuda'),
         torch.zeros((64,), dtype=torch.int32, device='cuda')]
    b = [t.clone() for t in a]
    n1 = legacy.hard_voxelize(pts, *a, VS8, CR8, 5, 64, 3)
    n2 = legacy.voxel_layer_ext.hard_voxelize(pts, *b, VS8, CR8, 5, 64)
    n3 = hard_voxelize(pts, *[t.clone() for t in b], VS8, CR8, 5, 64)
    assert n1 == n2 == n3 and all(torch.equal(x, y) for x, y in zip(a, b))
    c1 = torch.empty((pts.size(0), 3), dtype=torch.int32, device='cuda')
    c2 = torch.empty_like(c1)
    legacy.dynamic_voxelize(pts, c1, VS8, CR8, 3)
    dynamic_voxelize(pts, c2, VS8, CR8)
    assert torch.equal(c1, c2)
