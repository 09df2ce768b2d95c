"""The CPU oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the reference checkout).  CPU only."""
import numpy as np
import pytest
import torch

from tests import synth
from oracle import oracle
from tests._util import sha


def test_bev_known_case(golden):
    g = golden('bev_known')
    out, bad = oracle.bev_pool(g['feats'], g['coords'], *g['shape'])
    assert bad == 0
    np.testing.assert_array_equal(out, g['out'])


@pytest.mark.parametrize('name', ['bev_rand_small_f32', 'bev_rand_medium_i64', 'bev_rand_odd_c'])
def test_bev_rand_fp32_bit_exact(golden, name):
    """fp32 sums in ascending point order reproduce index_add_ bit for bit."""
    g = golden(name)
    out, bad = oracle.bev_pool(g['feats'], g['coords'], *g['shape'])
    assert bad == 0
    np.testing.assert_array_equal(out, g['out'])
    grad = oracle.bev_pool_backward(g['upstream'], g['coords'], *g['shape'])
    np.testing.assert_array_equal(grad, g['grad'])


def test_bev_rand_fp16_within_tolerance(golden):
    """The reference CPU path accumulates fp16 in fp16; the oracle in fp32."""
    g = golden('bev_rand_small_f16')
    out, _ = oracle.bev_pool(g['feats'], g['coords'], *g['shape'])
    np.testing.assert_allclose(out, g['out'], rtol=1e-2, atol=1e-2)
    grad = oracle.bev_pool_backward(g['upstream'], g['coords'], *g['shape'])
    np.testing.assert_array_equal(grad, g['grad'])


def test_det_full_size_digest(digests):
    d = digests['det_b1_dyadic']
    case = synth.det_bev_pool_case(1, dyadic=True)
    assert sha(case.coords) == d['coords_sha'] and sha(case.feats) == d['feats_sha'], 'generator drifted'
    out, bad = oracle.bev_pool(case.feats.numpy(), case.coords.numpy(), case.B, case.D, case.H, case.W)
    assert bad == 0
    assert sha(out) == d['out_sha']


def test_dynamic_voxelize_points8(golden):
    g = golden('voxel_points8')
    c = oracle.dynamic_voxelize(g['points'], [1, 1, 1], [0, 0, 0, 4, 4, 4])
    np.testing.assert_array_equal(c, g['dyn_coors'])


@pytest.mark.parametrize('mp,mv', [(2, 8), (3, 8), (1, 2)])
def test_hard_voxelize_points8(golden, mp, mv):
    g = golden('voxel_points8')
    v, c, n, vn = oracle.hard_voxelize(g['points'], [1, 1, 1], [0, 0, 0, 4, 4, 4], mp, mv)
    k = f'mp{mp}_mv{mv}'
    assert vn == int(g[f'{k}_vn'])
    np.testing.assert_array_equal(c, g[f'{k}_coors'])
    np.testing.assert_array_equal(n, g[f'{k}_num'])
    np.testing.assert_array_equal(v, g[f'{k}_voxels'])


def test_dynamic_voxelize_noncubic_edges(golden):
    g = golden('voxel_rand_noncubic')
    c = oracle.dynamic_voxelize(g['points'], g['vsize'], g['crange'])
    np.testing.assert_array_equal(c, g['dyn_coors'])


@pytest.mark.parametrize('mp,mv', [(5, 300), (5, 100000), (32, 50)])
def test_hard_voxelize_noncubic(golden, mp, mv):
    g = golden('voxel_rand_noncubic')
    v, c, n, vn = oracle.hard_voxelize(g['points'], g['vsize'], g['crange'], mp, mv)
    k = f'mp{mp}_mv{mv}'
    assert vn == int(g[f'{k}_vn'])
    np.testing.assert_array_equal(c, g[f'{k}_coors'])
    np.testing.assert_array_equal(n, g[f'{k}_num'])
    np.testing.assert_array_equal(v, g[f'{k}_voxels'])


def test_lidar_full_size_digest(digests):
    d = digests['lidar_s0']
    pts = synth.lidar_sweeps(0)
    assert sha(pts) == d['points_sha'], 'generator drifted'
    v, c, n, vn = oracle.hard_voxelize(pts.numpy(), synth.LIDAR_VOXEL_SIZE, synth.LIDAR_RANGE,
                                       synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS)
    assert vn == d['voxel_num']
    assert sha(c[:vn]) == d['coors_sha']
    assert sha(n[:vn]) == d['num_sha']
    assert sha(v[:vn]) == d['voxels_sha']


@pytest.mark.parametrize('case', ['fix', 'rand'])
@pytest.mark.parametrize('red', ['sum', 'mean', 'max'])
def test_dynamic_scatter(golden, case, red):
    g = golden('scatter_cases')
    f, c = g[f'{case}_feats'], g[f'{case}_coors']
    vf, vc, mp, cnt = oracle.dynamic_scatter(f, c, red)
    np.testing.assert_array_equal(vc, g[f'{case}_{red}_vc'])
    np.testing.assert_array_equal(mp, g[f'{case}_{red}_map'])
    np.testing.assert_array_equal(cnt, g[f'{case}_{red}_cnt'])
    np.testing.assert_allclose(vf, g[f'{case}_{red}_vf'], rtol=1e-6, atol=1e-6)
    grad = oracle.dynamic_scatter_backward(g[f'{case}_{red}_up'], f, vf, mp, cnt, red)
    np.testing.assert_allclose(grad, g[f'{case}_{red}_grad'], rtol=1e-6, atol=1e-6)


def spconv_case(g, i):
    """Decode one rulebook fixture: (indices, out_shape, params, expected)."""
    cfg = [int(v) for v in g[f'c{i}_cfg']]
    nd = (len(cfg) - 3) // 5
    shape, k, s, p, d = (cfg[j * nd:(j + 1) * nd] for j in range(5))
    subm, tr, B = cfg[5 * nd:]
    return (g[f'c{i}_indices'], [int(v) for v in g[f'c{i}_outshape']], shape, k, s, p, d, bool(subm), bool(tr), B,
            (g[f'c{i}_outids'], g[f'c{i}_pairs'], g[f'c{i}_num']))


@pytest.mark.parametrize('i', range(9))
def test_indice_pairs_match_reference(golden, i):
    """The C restatement of the rulebook against the reference's own
    _get_indice_pairs_impl (GPU ordering): outputs, pairs and counts equal."""
    g = golden('spconv_cases')
    idx, outs, _, k, s, p, d, subm, tr, _, (w_out, w_pairs, w_num) = spconv_case(g, i)
    o, pr, nm = oracle.indice_pairs(idx, outs, k, s, p, d, subm, tr)
    np.testing.assert_array_equal(o, w_out)
    np.testing.assert_array_equal(pr, w_pairs)
    np.testing.assert_array_equal(nm, w_num)


def spconv_conv_case(g, j):
    c, cin, cout, inverse, n_in, n_out = (int(v) for v in g[f'v{j}_case'])
    return c, cin, cout, bool(inverse), n_in, n_out


@pytest.mark.parametrize('j', range(5))
def test_spconv_conv_oracle_vs_reference(golden, j):
    """The numpy restatement of indice_conv / fused / backward (float64)
    against the reference's own fp32 CPU results, and of max-pooling (exact)."""
    g = golden('spconv_conv_cases')
    rb = golden('spconv_cases')
    c, cin, cout, inverse, n_in, n_out = spconv_conv_case(g, j)
    pairs, num = rb[f'c{c}_pairs'], rb[f'c{c}_num']
    x, w, bias, gy = g[f'v{j}_x'], g[f'v{j}_w'], g[f'v{j}_bias'], g[f'v{j}_gy']
    tol = dict(rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(oracle.indice_conv(x, w, pairs, num, n_out, inverse), g[f'v{j}_y'], **tol)
    np.testing.assert_allclose(oracle.indice_conv(x, w, pairs, num, n_out, inverse, bias), g[f'v{j}_yb'], **tol)
    gx, gw = oracle.indice_conv_backward(x, w, gy, pairs, num, inverse)
    np.testing.assert_allclose(gx, g[f'v{j}_gx'], **tol)
    np.testing.assert_allclose(gw, g[f'v{j}_gw'], **tol)
    if not inverse:
        xp = g[f'v{j}_xp']
        yp = oracle.indice_maxpool(xp, pairs, num, n_out)
        np.testing.assert_array_equal(yp, g[f'v{j}_yp'])
        np.testing.assert_array_equal(oracle.indice_maxpool_backward(xp, yp, g[f'v{j}_gyp'], pairs, num),
                                      g[f'v{j}_gxp'])
