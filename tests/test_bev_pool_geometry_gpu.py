"""Camera-parameters -> plan producer (the LSS geometry, quantise and filter
fused into the plan's keys kernel) against a plain PyTorch fp32 restatement
of the reference caller, and the pooling paths that consume such a plan.

Tolerance: the producer is floating-point geometry followed by truncation,
so a point that lies within rounding of a cell edge can land in the
neighbouring cell when the 3x3 products are summed in another order (the
reference uses a batched matmul).  The bar: at most 1e-5 of the frustum
points differ from the reference's cells, and every one of them is within
1e-3 of a cell edge in the reference's own fp32 coordinates.  Everything
downstream of the cells is compared bit for bit.
"""
import numpy as np
import pytest
import torch

from tests import synth
from tests._util import sha
from bevfusion_triton_b200.ops.bev_pool import (bev_grid, bev_pool, bev_pool_depth_context, bev_pool_geometry_plan,
                                                bev_pool_planned)
from bevfusion_triton_b200.ops.bev_pool.bev_pool import invalid_count, plan_cells

pytestmark = pytest.mark.gpu

MAX_MISMATCH_FRACTION = 1e-5
EDGE_TOL = 1e-3


ref_geometry = synth.lss_geometry  # base.py:82-126 in torch fp32


def ref_cells(geom, grid):
    """Quantise + in-grid filter of base.py:131-158 -> cell rank per frustum
    point (-1 when filtered out) and the fp32 grid coordinates before
    truncation."""
    lower, dx, nx = bev_grid(**grid)
    lower_t = torch.tensor(lower, dtype=torch.float32, device=geom.device)
    dx_t = torch.tensor(dx, dtype=torch.float32, device=geom.device)
    B = geom.size(0)
    v = (geom - lower_t) / dx_t
    g = v.long().reshape(-1, 3)
    b = torch.arange(B, device=geom.device).repeat_interleave(geom[0].numel() // 3)
    kept = (g[:, 0] >= 0) & (g[:, 0] < nx[0]) & (g[:, 1] >= 0) & (g[:, 1] < nx[1]) & (g[:, 2] >= 0) & (
        g[:, 2] < nx[2])
    cell = ((b * nx[2] + g[:, 2]) * nx[0] + g[:, 0]) * nx[1] + g[:, 1]
    return torch.where(kept, cell, torch.full_like(cell, -1)), v.reshape(-1, 3), (B, nx[2], nx[0], nx[1])


def check_cells(ours, ref, v):
    bad = torch.nonzero(ours != ref).squeeze(1)
    assert bad.numel() <= max(1, int(MAX_MISMATCH_FRACTION * ref.numel())), f'{bad.numel()} cells differ'
    if bad.numel():
        frac = v[bad] - v[bad].round()
        assert bool((frac.abs().min(1).values < EDGE_TOL).all()), 'a differing point is not at a cell edge'
    return bad.numel()


@pytest.mark.parametrize('augment', [False, True], ids=['rig', 'augmented'])
@pytest.mark.parametrize('grid', ['det', 'seg'])
def test_geometry_plan_cells_match_reference(cuda, augment, grid):
    grid_d = synth.DET_GRID if grid == 'det' else synth.SEG_GRID
    rig = synth.camera_rig(2, augment=augment, seed=3, device='cuda')
    plan, shape = bev_pool_geometry_plan(xbound=grid_d['xbound'], ybound=grid_d['ybound'], zbound=grid_d['zbound'],
                                         **rig)
    want, v, rshape = ref_cells(ref_geometry(**rig), grid_d)
    assert shape == rshape
    n = want.numel()
    got = plan_cells(plan, n, *shape)
    check_cells(got, want, v)
    assert invalid_count(plan) == int((got < 0).sum())


FIXTURE_CASES = {'det_plain': ('det', 1, False), 'det_aug': ('det', 2, True), 'seg_plain': ('seg', 1, False),
                 'seg_aug': ('seg', 1, True)}


@pytest.mark.parametrize('name', sorted(FIXTURE_CASES))
def test_geometry_plan_cells_match_reference_fixture(cuda, golden, digests, name):
    """Pinned to the reference itself: tests/golden/make_golden.py ran the
    reference's BaseTransform.get_geometry and the quantise + filter of its
    bev_pool (models/vtransforms/base.py:82-158) on this rig on the CPU.  Every
    point whose quantiser input is more than 1e-4 cells from a cell edge has
    exactly the reference's cell (digest of the whole cell array with the
    near-edge points masked); a near-edge point is in the reference's cell or
    a neighbour of it (one axis, one step, or across the grid border)."""
    grid, batch, augment = FIXTURE_CASES[name]
    grid_d = synth.DET_GRID if grid == 'det' else synth.SEG_GRID
    rig = synth.camera_rig(batch, augment=augment, seed=5, device='cuda')
    plan, shape = bev_pool_geometry_plan(xbound=grid_d['xbound'], ybound=grid_d['ybound'], zbound=grid_d['zbound'],
                                         **rig)
    g = golden('geometry_cells')
    assert list(shape) == g[f'{name}_grid'].tolist()
    n = batch * 6 * rig['frustum'][..., 0].numel()
    got = plan_cells(plan, n, *shape).cpu()
    near = torch.from_numpy(g[f'{name}_near_idx'].astype(np.int64))
    masked = got.clone()
    masked[near] = -2
    assert sha(masked) == digests[f'geometry_{name}_masked_cells']
    B, D, H, W = shape
    want = torch.from_numpy(g[f'{name}_near_cells'])
    ours = got[near]

    def split(c):
        return torch.stack((c // (D * H * W), (c // (H * W)) % D, (c // W) % H, c % W), 1)

    both = (want >= 0) & (ours >= 0)
    step = (split(ours[both]) - split(want[both])).abs().sum(1)
    assert bool((step <= 1).all())
    # a point dropped on one side only sits on the grid border
    one = (want >= 0) ^ (ours >= 0)
    kept = want[one].clamp_min(0) * (want[one] >= 0) + ours[one].clamp_min(0) * (ours[one] >= 0)
    k = split(kept)
    border = (k[:, 1] == 0) | (k[:, 1] == D - 1) | (k[:, 2] == 0) | (k[:, 2] == H - 1) | (k[:, 3] == 0) | (
        k[:, 3] == W - 1)
    assert bool(border.all())
    assert int((ours != want).sum()) <= max(1, near.numel() // 10)


def test_geometry_plan_pools_unfiltered_features(cuda):
    """bev_pool_planned over the UNFILTERED frustum features equals bev_pool
    over the filtered ones with the same cells, bit for bit, forward and
    backward."""
    grid_d = synth.DET_GRID
    rig = synth.camera_rig(2, augment=True, seed=5, device='cuda')
    plan, shape = bev_pool_geometry_plan(xbound=grid_d['xbound'], ybound=grid_d['ybound'], zbound=grid_d['zbound'],
                                         **rig)
    B, D, H, W = shape
    n = B * 6 * rig['frustum'][..., 0].numel()
    cells = plan_cells(plan, n, *shape)
    kept = cells >= 0
    c = cells[kept]
    coords = torch.stack(((c // W) % H, c % W, (c // (H * W)) % D, c // (D * H * W)), 1)
    g = torch.Generator(device='cuda').manual_seed(1)
    x = torch.randn((n, 16), generator=g, device='cuda')
    a = x.clone().requires_grad_(True)
    out_a = bev_pool_planned(a, plan, *shape)
    b = x[kept].clone().requires_grad_(True)
    out_b = bev_pool(b, coords, *shape)
    assert torch.equal(out_a, out_b)
    up = torch.randn(out_a.shape, generator=g, device='cuda')
    out_a.backward(up)
    out_b.backward(up)
    assert torch.equal(a.grad[kept], b.grad)
    assert bool((a.grad[~kept] == 0).all())


def test_geometry_plan_depth_context(cuda):
    """The camera branch with no coordinate tensor at all: geometry plan ->
    fused depth x context pooling, against the coords-driven fused op fed the
    plan's own cells (forward and gradients bit for bit)."""
    grid_d = synth.DET_GRID
    B = 2
    rig = synth.camera_rig(B, augment=True, seed=7, device='cuda')
    plan, shape = bev_pool_geometry_plan(xbound=grid_d['xbound'], ybound=grid_d['ybound'], zbound=grid_d['zbound'],
                                         **rig)
    Bs, D, H, W = shape
    nd, fh, fw = rig['frustum'].shape[:3]
    g = torch.Generator(device='cuda').manual_seed(2)
    depth = torch.randn((B, 6, nd, fh, fw), generator=g, device='cuda').softmax(2)
    ctx = torch.randn((B, 6, 32, fh, fw), generator=g, device='cuda')
    n = depth.numel()
    cells = plan_cells(plan, n, *shape)
    # unfiltered coords: dropped points get an out-of-grid x
    c = cells.clamp_min(0)
    coords = torch.stack(((c // W) % H, c % W, (c // (H * W)) % D, c // (D * H * W)), 1)
    coords[cells < 0, 0] = H
    d1, c1 = depth.clone().requires_grad_(True), ctx.clone().requires_grad_(True)
    d2, c2 = depth.clone().requires_grad_(True), ctx.clone().requires_grad_(True)
    o1 = bev_pool_depth_context(d1, c1, None, *shape, plan=plan)
    o2 = bev_pool_depth_context(d2, c2, coords, *shape)
    assert torch.equal(o1, o2)
    up = torch.randn(o1.shape, generator=g, device='cuda')
    o1.backward(up)
    o2.backward(up)
    assert torch.equal(d1.grad, d2.grad)
    assert torch.equal(c1.grad, c2.grad)
