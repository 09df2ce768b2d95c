"""Sparse-convolution rulebook (get_indice_pairs) on the GPU against the
reference's own outputs (golden fixtures) and the C oracle at LiDAR scale.
Integer work: compared exactly."""
import numpy as np
import pytest
import torch

from tests import synth
from bevfusion_triton_b200.ops.spconv import get_conv_output_size, get_indice_pairs
from bevfusion_triton_b200.ops.voxel.voxel_layer import hard_voxelize_batch
from oracle import oracle
from tests.test_oracle_golden import spconv_case

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('i', range(9))
def test_golden_rulebooks(cuda, golden, i):
    g = golden('spconv_cases')
    idx, outs, shape, k, s, p, d, subm, tr, B, (w_out, w_pairs, w_num) = spconv_case(g, i)
    o, pr, nm = get_indice_pairs(torch.from_numpy(idx).cuda(), B, shape, ksize=k, stride=s, padding=p, dilation=d,
                                 subm=subm, transpose=tr)
    np.testing.assert_array_equal(o.cpu().numpy(), w_out)
    np.testing.assert_array_equal(pr.cpu().numpy(), w_pairs)
    np.testing.assert_array_equal(nm.cpu().numpy(), w_num)


def lidar_voxel_indices(batch):
    """(b, x, y, z) int32 sites of `batch` synthetic LiDAR samples after hard
    voxelisation (config 3 grid 1440 x 1440 x 40): the sparse encoder's input."""
    pts = [synth.lidar_sweeps(i).cuda() for i in range(batch)]
    offs = [0]
    for q in pts:
        offs.append(offs[-1] + q.size(0))
    V, C, N, VN = hard_voxelize_batch(torch.cat(pts), offs, list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE),
                                      synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS)
    rows = []
    for b in range(batch):
        c = C[b, :int(VN[b])].int()
        rows.append(torch.cat((torch.full((c.size(0), 1), b, dtype=torch.int32, device=c.device), c), 1))
    return torch.cat(rows).contiguous()


SPARSE_SHAPE = [1440, 1440, 41]  # the sparse encoder's (x, y, z) shape (swint_v0p075)
LAYERS = [
    dict(ksize=3, stride=1, padding=1, subm=True),                                # conv_input / SubMConv3d
    dict(ksize=3, stride=2, padding=1, subm=False),                               # SparseConv3d down
    dict(ksize=(1, 1, 3), stride=(1, 1, 2), padding=0, subm=False),               # conv_out
    dict(ksize=3, stride=2, padding=(1, 1, 0), subm=False),                       # asymmetric padding
]


@pytest.mark.parametrize('layer', LAYERS, ids=['subm3', 'down3', 'out113', 'down3_pad110'])
def test_lidar_scale_vs_oracle(cuda, layer):
    idx = lidar_voxel_indices(2)
    o, pr, nm = get_indice_pairs(idx, 2, SPARSE_SHAPE, **layer)
    k = layer['ksize']
    nd = 3
    norm = (lambda v: list(v) if isinstance(v, tuple) else [v] * nd)
    ks, st, pd = norm(k), norm(layer['stride']), norm(layer['padding'])
    outs = SPARSE_SHAPE if layer['subm'] else get_conv_output_size(SPARSE_SHAPE, ks, st, pd, [1, 1, 1])
    w_out, w_pairs, w_num = oracle.indice_pairs(idx.cpu().numpy(), outs, ks, st, pd, [1, 1, 1], layer['subm'], False)
    np.testing.assert_array_equal(nm.cpu().numpy(), w_num)
    np.testing.assert_array_equal(o.cpu().numpy(), w_out)
    np.testing.assert_array_equal(pr.cpu().numpy(), w_pairs)


def test_edge_cases(cuda):
    empty = torch.empty((0, 4), dtype=torch.int32, device='cuda')
    o, pr, nm = get_indice_pairs(empty, 1, [8, 8, 8], ksize=3, stride=2, padding=1)
    assert o.shape == (0, 4) and pr.shape == (27, 2, 0) and int(nm.sum()) == 0
    idx = torch.tensor([[0, 1, 1, 1], [1, 7, 7, 7]], dtype=torch.int32, device='cuda')
    with pytest.raises(ValueError):
        get_indice_pairs(idx, 1, [8, 8, 8])  # batch column exceeds batch_size
    with pytest.raises(AssertionError):
        get_indice_pairs(idx, 2, [8, 8, 8], stride=2, dilation=2)
    grid = torch.zeros(2 * 8 * 8 * 8, dtype=torch.int32, device='cuda')
    o, pr, nm = get_indice_pairs(idx, 2, [8, 8, 8], ksize=3, padding=1, subm=True, grid=grid)
    assert bool((grid == -1).all())
    assert torch.equal(o, idx)
    assert int(nm.sum()) == 2 and int(nm[13]) == 2  # only the centre offset pairs each site with itself
    # a site whose every neighbour is outside the grid: corner, 1x1x1 output
    o, pr, nm = get_indice_pairs(idx[:1], 1, [2, 2, 2], ksize=2, stride=2)
    assert o.tolist() == [[0, 0, 0, 0]] and int(nm.sum()) == 1


@pytest.mark.parametrize('subm', [False, True])
def test_out_of_range_batch_rows_are_ignored_by_the_c_abi(cuda, subm):
    """The C entry point is memory-safe on its own: rows whose batch column is
    outside [0, batch) (which the Python wrapper refuses) reach no output cell
    and pair with nothing, instead of addressing past the output bitmap."""
    from bevfusion_triton_b200._lib import ops
    good = lidar_voxel_indices(2)[:20000].contiguous()
    bad = good[:4].clone()
    bad[:, 0] = torch.tensor([2, 7, -1, 1 << 30], dtype=torch.int32)
    mixed = torch.cat([good, bad]).contiguous()
    shape, ks, st, pd = SPARSE_SHAPE, [3, 3, 3], [1, 1, 1] if subm else [2, 2, 2], [1, 1, 1]
    outs = SPARSE_SHAPE if subm else get_conv_output_size(SPARSE_SHAPE, ks, st, pd, [1, 1, 1])
    a = ops().get_indice_pairs(good, 2, outs, ks, st, pd, [1, 1, 1], subm, False)
    b = ops().get_indice_pairs(mixed, 2, outs, ks, st, pd, [1, 1, 1], subm, False)
    assert torch.equal(a[2], b[2])
    if not subm:
        assert torch.equal(a[0], b[0])
    n = good.size(0)
    for k in range(27):
        m = int(a[2][k])
        assert torch.equal(a[1][k, :, :m], b[1][k, :, :m])
        assert bool((b[1][k, :, m:] == -1).all())
    assert int(b[2].sum()) == int(a[2].sum()) and int((b[1][:, 0] >= n).sum()) == 0
