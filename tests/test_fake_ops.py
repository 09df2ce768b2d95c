"""Fake (meta) kernels and registered autograd of the torch.ops.bfb_b200
custom ops, on CPU: every op traces under FakeTensorMode with the shapes the
CUDA kernels produce (workspace tensors sized by the library's host-only
queries), and the differentiable ops carry an autograd formula on the op
itself (no Python autograd.Function)."""
import ctypes

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.symbolic_shapes import ShapeEnv

from bevfusion_triton_b200 import load_native
from bevfusion_triton_b200._lib import bev_pool_plan_bytes, ops


@pytest.fixture(scope='module')
def O():
    load_native()
    return ops()


def fake_mode():
    return FakeTensorMode(shape_env=ShapeEnv())


def test_bev_pool_ops_trace(O):
    n, C, B, D, H, W = 5000, 80, 2, 1, 40, 30
    with fake_mode():
        feats = torch.empty(n, C, device='cuda')
        coords = torch.empty(n, 4, dtype=torch.int64, device='cuda')
        out, plan = O.bev_pool_forward(feats, coords, B, D, H, W)
        assert out.shape == (B, C, D, H, W) and out.dtype == feats.dtype
        assert plan.shape == (bev_pool_plan_bytes(n, B, D, H, W),) and plan.dtype == torch.uint8
        assert O.bev_pool_plan(coords, B, D, H, W).shape == plan.shape
        assert O.bev_pool_forward_planned(feats.half(), plan, B, D, H, W).dtype == torch.float16
        assert O.bev_pool_backward(out, plan, n, B, D, H, W).shape == (n, C)
        assert O.bev_pool_plan_cells(plan, n, B, D, H, W).shape == (n,)


def test_dc_and_geometry_ops_trace(O):
    cams, nd, fh, fw, C, B, D, H, W = 6, 118, 4, 8, 80, 1, 1, 50, 50
    lib = load_native()
    sz = [ctypes.c_size_t() for _ in range(4)]
    assert lib.bfb_bev_pool_dc_workspace_sizes(*[ctypes.c_int64(v) for v in (cams, nd, fh, fw, C, B, D, H, W)],
                                               *[ctypes.byref(s) for s in sz]) == 0
    with fake_mode():
        depth = torch.empty(cams, nd, fh, fw, device='cuda')
        ctx = torch.empty(cams, C, fh, fw, device='cuda')
        coords = torch.empty(cams * nd * fh * fw, 4, dtype=torch.int64, device='cuda')
        out, aux = O.bev_pool_dc_forward(depth, ctx, coords, B, D, H, W)
        assert out.shape == (B, C, D, H, W) and aux.shape == (sz[2].value,)
        gd, gc = O.bev_pool_dc_backward(out, depth, coords[:0], aux, C, B, D, H, W)
        assert gd.shape == depth.shape and gc.shape == ctx.shape
        frustum = torch.empty(nd, fh, fw, 3, device='cuda')
        r = torch.empty(B, cams, 3, 3, device='cuda')
        t = torch.empty(B, cams, 3, device='cuda')
        plan = O.bev_pool_geometry_plan(frustum, r, t, r, t, None, None, [0., 0., 0.], [1., 1., 1.], D, H, W)
        assert plan.shape == (sz[0].value,)


def test_voxel_and_scatter_ops_trace(O):
    with fake_mode():
        pts = torch.empty(1000, 5, device='cuda')
        vox = torch.empty(100, 10, 5, device='cuda')
        co = torch.empty(100, 3, dtype=torch.int32, device='cuda')
        num = torch.empty(100, dtype=torch.int32, device='cuda')
        O.dynamic_voxelize(pts, co, [0.1] * 3, [0.] * 3 + [1.] * 3)
        del vox, num
        feats = torch.empty(1000, 16, device='cuda')
        c4 = torch.empty(1000, 4, dtype=torch.int32, device='cuda')
        vf, vc, mp, cnt = O.dynamic_scatter_forward(feats, c4, 'mean', None)
        assert vf.shape[1] == 16 and vc.shape[1] == 4 and mp.shape == (1000,) and cnt.shape[0] == vf.shape[0]
        idx = torch.empty(300, 4, dtype=torch.int32, device='cuda')
        o, pr, nm = O.get_indice_pairs(idx, 2, [8, 8, 8], [3, 3, 3], [1] * 3, [1] * 3, [1] * 3, True, False)
        assert o.shape == (300, 4) and pr.shape == (27, 2, 300) and nm.shape == (27,)
        o, pr, nm = O.get_indice_pairs(idx, 2, [4, 4, 4], [3, 3, 3], [2] * 3, [1] * 3, [1] * 3, False, False)
        assert o.shape[1] == 4 and isinstance(o.shape[0], torch.SymInt)


def test_every_op_has_a_fake_kernel(O):
    from torch._library.simple_registry import singleton
    names = sorted({s.name.split('::')[1] for s in torch._C._jit_get_all_schemas() if s.name.startswith('bfb_b200::')})
    assert len(names) >= 17
    missing = [n for n in names if singleton.find(f'bfb_b200::{n}').fake_impl.kernel is None]
    assert not missing, missing


@pytest.mark.parametrize('name', ['bev_pool_forward', 'bev_pool_forward_planned', 'bev_pool_dc_forward',
                                  'bev_pool_dc_forward_planned', 'dynamic_scatter_forward'])
def test_autograd_registered_on_the_op(O, name):
    op = getattr(O, name).default
    assert torch._C._dispatch_has_kernel_for_dispatch_key(op.name(), 'Autograd')


def test_bev_pool_graph_traces_forward_and_backward(O):
    """make_fx over the bev_pool op and its registered backward on meta
    tensors (no device): the graph holds the forward op and the backward op."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def step(feats, coords, up):
        x = feats.detach().requires_grad_(True)
        out = O.bev_pool_forward(x, coords, 2, 1, 16, 16)[0]
        (g,) = torch.autograd.grad((out * up).sum(), x)
        return out, g

    feats = torch.empty(700, 8, device='meta')
    coords = torch.zeros(700, 4, dtype=torch.int64, device='meta')
    up = torch.empty(2, 8, 1, 16, 16, device='meta')
    gm = make_fx(step, tracing_mode='fake')(feats, coords, up)
    targets = {str(n.target) for n in gm.graph.nodes if n.op == 'call_function'}
    assert 'bfb_b200.bev_pool_forward.default' in targets
    assert 'bfb_b200.bev_pool_backward.default' in targets
