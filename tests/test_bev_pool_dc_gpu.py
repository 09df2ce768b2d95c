"""Fused depth x context pooling against the unfused reference composition
(models/vtransforms/depth_lss.py:91-94 product, base.py:136-160 flatten /
filter, then bev_pool).  The forward must match bit for bit (same fp32
product, same summation order); gradients w.r.t. depth and context are
reductions whose order differs from torch's, so they are compared at
rtol = atol = 1e-5 (the fp32 bar)."""
import numpy as np
import pytest
import torch

from tests import synth
from bevfusion_triton_b200.ops.bev_pool import bev_pool, bev_pool_depth_context
from oracle import oracle

pytestmark = pytest.mark.gpu


def unfused(depth, ctx, coords, kept, shape):
    B, N = depth.shape[:2]
    x = depth.unsqueeze(2) * ctx.unsqueeze(3)                     # [B, N, C, D, fH, fW]
    x = x.permute(0, 1, 3, 4, 5, 2).reshape(-1, ctx.size(2))      # (b n d h w) c
    return bev_pool(x[kept], coords[kept], *shape)


@pytest.mark.parametrize('grid', ['det', 'seg'])
def test_fused_forward_backward(cuda, grid):
    case = synth.depth_context_case(2, synth.DET_GRID if grid == 'det' else synth.SEG_GRID, device='cuda')
    shape = (case.B, case.D, case.H, case.W)
    d1 = case.depth.clone().requires_grad_(True)
    c1 = case.context.clone().requires_grad_(True)
    out = bev_pool_depth_context(d1, c1, case.coords, *shape)
    d2 = case.depth.clone().requires_grad_(True)
    c2 = case.context.clone().requires_grad_(True)
    ref = unfused(d2, c2, case.coords, case.kept, shape)
    assert torch.equal(out, ref)
    up = torch.randn(out.shape, device='cuda', generator=torch.Generator(device='cuda').manual_seed(1))
    out.backward(up)
    ref.backward(up)
    torch.testing.assert_close(d1.grad, d2.grad, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(c1.grad, c2.grad, rtol=1e-5, atol=1e-5)


def test_fused_forward_vs_oracle_small(cuda):
    g = torch.Generator().manual_seed(5)
    cams, nd, fh, fw, C = 3, 7, 5, 9, 12
    B, D, H, W = 2, 2, 6, 7
    depth = torch.rand((cams, nd, fh, fw), generator=g)
    ctx = torch.randn((cams, C, fh, fw), generator=g)
    n = cams * nd * fh * fw
    coords = torch.stack([torch.randint(-1, H + 1, (n,), generator=g), torch.randint(0, W, (n,), generator=g),
                          torch.randint(0, D, (n,), generator=g), torch.randint(0, B, (n,), generator=g)], 1)
    out = bev_pool_depth_context(depth.cuda(), ctx.cuda(), coords.cuda(), B, D, H, W)
    feats = (depth.unsqueeze(1) * ctx.unsqueeze(2)).permute(0, 2, 3, 4, 1).reshape(-1, C)
    ref, bad = oracle.bev_pool(feats.numpy(), coords.numpy(), B, D, H, W)
    assert bad > 0
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_fused_forward_vs_oracle_det_sample(cuda):
    """One full det sample (6 cameras x 118 bins x 32 x 88, C = 80, the
    config-1 grid) through the fused op against the C oracle's sequential sum
    of the materialised product (unfiltered: the oracle drops the out-of-grid
    points as the caller's filter does), bit for bit; and the gradients
    against the oracle's backward gather contracted on the CPU in fp64."""
    case = synth.depth_context_case(1, synth.DET_GRID, device='cuda')
    shape = (case.B, case.D, case.H, case.W)
    d = case.depth.clone().requires_grad_(True)
    c = case.context.clone().requires_grad_(True)
    out = bev_pool_depth_context(d, c, case.coords, *shape)
    C = case.context.size(2)
    feats = (case.depth.unsqueeze(2) * case.context.unsqueeze(3)).permute(0, 1, 3, 4, 5, 2).reshape(-1, C)
    ref, bad = oracle.bev_pool(feats.cpu().numpy(), case.coords.cpu().numpy(), *shape)
    assert bad == int((~case.kept).sum())
    np.testing.assert_array_equal(out.detach().cpu().numpy(), ref)
    up = torch.randn(out.shape, device='cuda', generator=torch.Generator(device='cuda').manual_seed(3))
    out.backward(up)
    # d feats[n] = up[cell(n)] (oracle gather), then the product rule in fp64
    gf = torch.from_numpy(oracle.bev_pool_backward(up.cpu().numpy(), case.coords.cpu().numpy(), *shape))
    gf = gf.double().view(1, 6, -1, 32, 88, C)                     # (b n d h w) c
    dep = case.depth.double().cpu()
    ctx = case.context.double().cpu()                              # [1, 6, C, fH, fW]
    want_d = (gf * ctx.permute(0, 1, 3, 4, 2).unsqueeze(2)).sum(-1)
    want_c = (gf * dep.unsqueeze(-1)).sum(2).permute(0, 1, 4, 2, 3)
    torch.testing.assert_close(d.grad.double().cpu(), want_d, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(c.grad.double().cpu(), want_c, rtol=1e-5, atol=1e-5)
