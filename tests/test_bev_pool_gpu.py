"""bev_pool parity on the GPU: the sm_100a kernels against the reference's
golden outputs and the CPU oracle.

Tolerance: the stated bar is fp32 rtol = atol = 1e-5 and fp16 within 1e-2 of
an fp32 sum of the same inputs.  The kernels sum each cell in ascending point
order in fp32, exactly as torch.index_add_ does, so the tests hold them to
more than that: fp32 outputs must be bit-identical to the reference / oracle,
and fp16 / bf16 outputs must equal the oracle's fp32 sum rounded once to the
storage type.  The backward is a gather and is compared exactly.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests import synth
from bevfusion_triton_b200.ops.bev_pool import bev_pool, bev_pool_plan, bev_pool_planned
from bevfusion_triton_b200.ops.bev_pool.bev_pool import invalid_count
from oracle import oracle
from tests._util import rand_bev_case, sha

pytestmark = pytest.mark.gpu

FP32_TOL = dict(rtol=1e-5, atol=1e-5)
LOW_TOL = {torch.float16: dict(rtol=1e-2, atol=1e-2), torch.bfloat16: dict(rtol=2e-2, atol=2e-2)}


def run_fwd_bwd(feats, coords, shape, upstream=None, dev='cuda'):
    x = feats.to(dev).clone().requires_grad_(True)
    out = bev_pool(x, coords.to(dev), *shape)
    grad = None
    if upstream is not None:
        (out * upstream.to(dev).to(out.dtype)).sum().backward()
        grad = x.grad
    return out, grad


def test_known_case(cuda, golden):
    g = golden('bev_known')
    out, _ = run_fwd_bwd(torch.from_numpy(g['feats']), torch.from_numpy(g['coords']), list(g['shape']))
    assert torch.equal(out.cpu(), torch.from_numpy(g['out']))


@pytest.mark.parametrize('name', ['bev_rand_small_f32', 'bev_rand_medium_i64', 'bev_rand_odd_c'])
def test_reference_golden_fp32(cuda, golden, name):
    g = golden(name)
    out, grad = run_fwd_bwd(torch.from_numpy(g['feats']), torch.from_numpy(g['coords']), list(g['shape']),
                            torch.from_numpy(g['upstream']))
    np.testing.assert_array_equal(out.detach().cpu().numpy(), g['out'])
    np.testing.assert_array_equal(grad.cpu().numpy(), g['grad'])


def test_reference_golden_fp16(cuda, golden):
    g = golden('bev_rand_small_f16')
    feats = torch.from_numpy(g['feats']).half()
    out, grad = run_fwd_bwd(feats, torch.from_numpy(g['coords']), list(g['shape']), torch.from_numpy(g['upstream']))
    ref, _ = oracle.bev_pool(feats.float().numpy(), g['coords'], *g['shape'])
    np.testing.assert_allclose(out.detach().float().cpu().numpy(), ref, **LOW_TOL[torch.float16])
    assert torch.equal(out.detach().cpu(), torch.from_numpy(ref).half())
    # the reference itself (fp16 accumulation) is within the fp16 bar of the fp32 sum
    np.testing.assert_allclose(g['out'], ref, **LOW_TOL[torch.float16])
    np.testing.assert_array_equal(grad.float().cpu().numpy(), g['grad'])


CASES = [
    # n, c, B, D, H, W, cdtype, hot, invalid
    (0, 8, 1, 1, 4, 4, torch.int64, None, 0),          # empty input
    (1, 1, 1, 1, 1, 1, torch.int32, None, 0),          # single point, single cell
    (777, 3, 2, 2, 5, 7, torch.int32, None, 0),        # odd C: scalar path
    (5000, 80, 2, 1, 36, 50, torch.int64, None, 0),    # det channels, W not a multiple of 32
    (20000, 80, 1, 1, 64, 64, torch.int64, 9000, 0),   # cells beyond one work piece
    (4000, 130, 1, 2, 9, 33, torch.int64, None, 0),    # C > 128: two channel slices
    (3000, 16, 2, 1, 10, 10, torch.int64, None, 400),  # out-of-range points dropped
    (300, 8, 1, 1, 3, 3, torch.int32, None, 300),      # every point dropped
]


@pytest.mark.parametrize('case', CASES, ids=lambda c: f'n{c[0]}_c{c[1]}_B{c[2]}')
@pytest.mark.parametrize('fdtype', [torch.float32, torch.float16, torch.bfloat16])
def test_random_vs_oracle(cuda, case, fdtype):
    n, c, B, D, H, W, cdtype, hot, invalid = case
    feats, coords = rand_bev_case(n, c, B, D, H, W, seed=n + c, cdtype=cdtype, fdtype=fdtype, hot=hot,
                                  invalid=invalid)
    g = torch.Generator().manual_seed(7)
    up = torch.randn((B, c, D, H, W), generator=g).to(fdtype)
    out, grad = run_fwd_bwd(feats, coords, (B, D, H, W), up)
    ref, bad = oracle.bev_pool(feats.float().numpy(), coords.numpy(), B, D, H, W)
    assert bad == invalid
    tol = FP32_TOL if fdtype == torch.float32 else LOW_TOL[fdtype]
    np.testing.assert_allclose(out.detach().float().cpu().numpy(), ref, **tol)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(ref).to(fdtype))  # one rounding of the fp32 sum
    rgrad = oracle.bev_pool_backward(up.float().numpy(), coords.numpy(), B, D, H, W)
    np.testing.assert_array_equal(grad.float().cpu().numpy(), rgrad)  # a gather: exact


def test_invalid_count_reported(cuda):
    feats, coords = rand_bev_case(1000, 4, 1, 1, 8, 8, seed=3, invalid=77)
    plan = bev_pool_plan(coords.cuda(), 1, 1, 8, 8)
    assert invalid_count(plan) == 77


def test_det_full_size_bit_exact_digest(cuda, digests):
    """Full det sample (1,770,765 points, 360x360) with exactly-summable
    features: the output must equal the reference's bit for bit."""
    d = digests['det_b1_dyadic']
    case = synth.det_bev_pool_case(1, dyadic=True)
    assert sha(case.coords) == d['coords_sha'] and sha(case.feats) == d['feats_sha']
    out, _ = run_fwd_bwd(case.feats, case.coords, (case.B, case.D, case.H, case.W))
    assert sha(out.detach().cpu()) == d['out_sha']


def test_det_batch8_vs_oracle_and_deterministic(cuda):
    """Config 1 shape (det, batch 8, fp32 softmax x context features)."""
    case = synth.det_bev_pool_case(8, device='cuda')
    shape = (case.B, case.D, case.H, case.W)
    out1 = bev_pool(case.feats, case.coords, *shape)
    out2 = bev_pool(case.feats, case.coords, *shape)
    assert torch.equal(out1, out2), 'forward must be bitwise deterministic'
    ref, bad = oracle.bev_pool(case.feats.cpu().numpy(), case.coords.cpu().numpy(), *shape)
    assert bad == 0
    np.testing.assert_array_equal(out1.cpu().numpy(), ref)
    # backward: exact gather
    g = torch.Generator(device='cuda').manual_seed(11)
    up = torch.randn(out1.shape, generator=g, device='cuda')
    x = case.feats.clone().requires_grad_(True)
    (bev_pool(x, case.coords, *shape) * up).sum().backward()
    idx = case.coords.cpu()
    s = ((idx[:, 2] * case.H + idx[:, 0]) * case.W + idx[:, 1]).cuda()
    want = up.reshape(case.B, up.size(1), -1).permute(0, 2, 1)[idx[:, 3].cuda(), s]
    assert torch.equal(x.grad, want)


def test_planned_matches_unplanned(cuda):
    feats, coords = rand_bev_case(10000, 80, 2, 1, 40, 40, seed=5)
    feats, coords = feats.cuda(), coords.cuda()
    plan = bev_pool_plan(coords, 2, 1, 40, 40)
    a = bev_pool(feats, coords, 2, 1, 40, 40)
    x = feats.clone().requires_grad_(True)
    b = bev_pool_planned(x, plan, 2, 1, 40, 40)
    assert torch.equal(a, b)
    b.sum().backward()
    assert torch.equal(x.grad, torch.ones_like(x))


def test_cabi_direct_call(cuda):
    """Drive the C ABI with raw device pointers (no torch op in between)."""
    from bevfusion_triton_b200 import load_native
    L = load_native()
    feats, coords = rand_bev_case(3000, 8, 1, 1, 16, 16, seed=9)
    feats, coords = feats.cuda(), coords.cuda()
    plan_b, scr_b = ctypes.c_size_t(), ctypes.c_size_t()
    i64 = ctypes.c_int64
    assert L.bfb_bev_pool_workspace_sizes(i64(3000), i64(8), i64(1), i64(1), i64(16), i64(16),
                                          ctypes.byref(plan_b), ctypes.byref(scr_b)) == 0
    plan = torch.empty(plan_b.value, dtype=torch.uint8, device='cuda')
    scr = torch.empty(scr_b.value, dtype=torch.uint8, device='cuda')
    out = torch.empty((1, 8, 1, 16, 16), device='cuda')
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.bfb_bev_pool_forward(ctypes.c_void_p(feats.data_ptr()), 0, ctypes.c_void_p(coords.data_ptr()), 1,
                                i64(3000), i64(8), i64(1), i64(1), i64(16), i64(16), ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(plan.data_ptr()), plan_b, ctypes.c_void_p(scr.data_ptr()), scr_b,
                                stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref, _ = oracle.bev_pool(feats.cpu().numpy(), coords.cpu().numpy(), 1, 1, 16, 16)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    # a workspace one byte short is refused
    rc = L.bfb_bev_pool_forward(ctypes.c_void_p(feats.data_ptr()), 0, ctypes.c_void_p(coords.data_ptr()), 1,
                                i64(3000), i64(8), i64(1), i64(1), i64(16), i64(16), ctypes.c_void_p(out.data_ptr()),
                                ctypes.c_void_p(plan.data_ptr()), ctypes.c_size_t(plan_b.value - 1),
                                ctypes.c_void_p(scr.data_ptr()), scr_b, stream)
    assert rc == -3


def test_plan_of_another_geometry_writes_nothing(cuda):
    """A plan built for 10000 points / B=2, handed (through the C ABI, with a
    buffer size that passes the size check) to a forward of 5000 points /
    B=1: the kernels compare the stamped geometry, write no output, and the
    plan check reports the mismatch.  The torch layer refuses it outright."""
    from bevfusion_triton_b200 import load_native
    from bevfusion_triton_b200.ops.bev_pool import plan_matches
    L = load_native()
    i64 = ctypes.c_int64
    feats, coords = rand_bev_case(10000, 8, 2, 1, 16, 16, seed=11)
    feats, coords = feats.cuda(), coords.cuda()
    plan = bev_pool_plan(coords, 2, 1, 16, 16)
    assert plan_matches(plan, 10000, 2, 1, 16, 16)
    short = feats[:5000].contiguous()
    out = torch.full((1, 8, 1, 16, 16), 7.0, device='cuda')
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.bfb_bev_pool_forward_planned(ctypes.c_void_p(short.data_ptr()), 0, i64(5000), i64(8), i64(1), i64(1),
                                        i64(16), i64(16), ctypes.c_void_p(plan.data_ptr()),
                                        ctypes.c_size_t(plan.numel()), ctypes.c_void_p(out.data_ptr()), stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)
    rc = L.bfb_bev_pool_plan_check(ctypes.c_void_p(plan.data_ptr()), i64(5000), i64(1), i64(1), i64(16), i64(16),
                                   stream)
    assert rc == -7
    assert not plan_matches(plan, 10000, 2, 1, 16, 16)  # the flag stays raised
    with pytest.raises(ValueError, match='another geometry'):
        bev_pool_planned(short, bev_pool_plan(coords, 2, 1, 16, 16), 1, 1, 16, 16)


def test_seg_batch4_fwd_bwd_vs_oracle(cuda):
    """Config 4: segmentation grid 256 x 256, batch 4, fp32, forward + backward."""
    case = synth.seg_bev_pool_case(4, device='cuda')
    shape = (case.B, case.D, case.H, case.W)
    assert shape == (4, 1, 256, 256)
    x = case.feats.clone().requires_grad_(True)
    out = bev_pool(x, case.coords, *shape)
    g = torch.Generator(device='cuda').manual_seed(3)
    up = torch.randn(out.shape, generator=g, device='cuda')
    out.backward(up)
    ref, bad = oracle.bev_pool(case.feats.cpu().numpy(), case.coords.cpu().numpy(), *shape)
    assert bad == 0
    np.testing.assert_array_equal(out.detach().cpu().numpy(), ref)
    rg = oracle.bev_pool_backward(up.cpu().numpy(), case.coords.cpu().numpy(), *shape)
    np.testing.assert_array_equal(x.grad.cpu().numpy(), rg)


def test_det_batch8_fp16_features(cuda):
    """Config 2's fp16-feature variant: the fp16 output equals the fp32 sum of
    the same fp16 inputs rounded once (the stated bar is 1e-2)."""
    case = synth.det_bev_pool_case(8, device='cuda', dtype=torch.float16)
    shape = (case.B, case.D, case.H, case.W)
    x = case.feats.clone().requires_grad_(True)
    out = bev_pool(x, case.coords, *shape)
    assert out.dtype == torch.float16
    ref, _ = oracle.bev_pool(case.feats.float().cpu().numpy(), case.coords.cpu().numpy(), *shape)
    np.testing.assert_allclose(out.detach().float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(ref).half())
    up = torch.randn(out.shape, device='cuda').half()
    out.backward(up)
    idx = case.coords.cpu()
    s = ((idx[:, 2] * case.H + idx[:, 0]) * case.W + idx[:, 1]).cuda()
    want = up.reshape(case.B, up.size(1), -1).permute(0, 2, 1)[idx[:, 3].cuda(), s]
    assert torch.equal(x.grad, want)


@pytest.mark.parametrize('case', CASES[1:], ids=lambda c: f'n{c[0]}_c{c[1]}_B{c[2]}')
@pytest.mark.parametrize('fdtype', [torch.float32, torch.float16, torch.bfloat16])
def test_backward_gather_equals_scatter(cuda, case, fdtype):
    """Both backward forms of the C ABI (scatter: no workspace; gather: one
    row per grid cell) give the oracle's gradient exactly."""
    from bevfusion_triton_b200 import load_native
    L = load_native()
    n, c, B, D, H, W, cdtype, hot, invalid = case
    feats, coords = rand_bev_case(n, c, B, D, H, W, seed=n + c, cdtype=cdtype, fdtype=fdtype, hot=hot,
                                  invalid=invalid)
    plan = bev_pool_plan(coords.cuda(), B, D, H, W)
    up = torch.randn((B, c, D, H, W), generator=torch.Generator().manual_seed(5)).to(fdtype).cuda()
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[fdtype]
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    stream = vp(torch.cuda.current_stream().cuda_stream)
    dims = [i64(v) for v in (n, c, B, D, H, W)]
    g_scatter = torch.full((n, c), 7, dtype=fdtype, device='cuda')
    assert L.bfb_bev_pool_backward(vp(up.data_ptr()), code, *dims, vp(plan.data_ptr()), ctypes.c_size_t(plan.numel()),
                                   vp(g_scatter.data_ptr()), stream) == 0
    ws_b = ctypes.c_size_t()
    assert L.bfb_bev_pool_backward_workspace_size(*dims, code, ctypes.byref(ws_b)) == 0
    assert ws_b.value == B * D * H * W * c * up.element_size()
    ws = torch.empty(ws_b.value, dtype=torch.uint8, device='cuda')
    g_gather = torch.full((n, c), 7, dtype=fdtype, device='cuda')
    args = [vp(up.data_ptr()), code, *dims, vp(plan.data_ptr()), ctypes.c_size_t(plan.numel()),
            vp(g_gather.data_ptr()), vp(ws.data_ptr())]
    assert L.bfb_bev_pool_backward_gather(*args, ctypes.c_size_t(ws_b.value - 1), stream) == -3
    assert L.bfb_bev_pool_backward_gather(*args, ws_b, stream) == 0
    torch.cuda.synchronize()
    rgrad = oracle.bev_pool_backward(up.float().cpu().numpy(), coords.numpy(), B, D, H, W)
    np.testing.assert_array_equal(g_gather.float().cpu().numpy(), rgrad)
    assert torch.equal(g_gather, g_scatter)


def test_torch_compile_fullgraph_matches_eager(cuda):
    """bev_pool forward + backward under torch.compile(fullgraph=True): the
    custom ops trace through their fake kernels and registered backward, and
    the compiled step returns what eager returns, bit for bit."""
    feats, coords = rand_bev_case(20000, 80, 2, 1, 40, 40, seed=31)
    feats, coords = feats.cuda(), coords.cuda()
    up = torch.randn((2, 80, 1, 40, 40), generator=torch.Generator().manual_seed(1)).cuda()

    def pool(x, c):
        return bev_pool(x, c, 2, 1, 40, 40)

    torch._dynamo.reset()
    compiled = torch.compile(pool, fullgraph=True)
    results = []
    for fn in (pool, compiled):  # AOTAutograd compiles the backward graph as well
        x = feats.clone().requires_grad_(True)
        out = fn(x, coords)
        (out * up).sum().backward()
        results.append((out.detach(), x.grad))
    (a, ga), (b, gb) = results
    assert torch.equal(a, b) and torch.equal(ga, gb)


def test_opcheck_bev_pool_ops(cuda):
    """torch.library.opcheck: schema (mutation / aliasing), fake kernel
    against the real one, autograd registration."""
    feats, coords = rand_bev_case(3000, 16, 1, 1, 20, 20, seed=32)
    feats, coords = feats.cuda().requires_grad_(True), coords.cuda()
    utils = ('test_schema', 'test_faketensor', 'test_autograd_registration')
    O = torch.ops.bfb_b200
    torch.library.opcheck(O.bev_pool_forward, (feats, coords, 1, 1, 20, 20), test_utils=utils)
    plan = O.bev_pool_plan(coords, 1, 1, 20, 20)
    torch.library.opcheck(O.bev_pool_forward_planned, (feats, plan, 1, 1, 20, 20), test_utils=utils)
    g = torch.randn((1, 16, 1, 20, 20), device='cuda')
    torch.library.opcheck(O.bev_pool_backward, (g, plan, 3000, 1, 1, 20, 20), test_utils=utils)


def test_legacy_import_path(cuda):
    """ops.bev_pool.bev_pool_legacy.bev_pool (the sort + interval path's
    import name) is the same op: equal outputs; mismatched lengths assert."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool as current
    from bevfusion_triton_b200.ops.bev_pool.bev_pool_legacy import bev_pool as legacy
    g = torch.Generator().manual_seed(4)
    n, C, B, D, H, W = 5000, 16, 2, 2, 12, 10
    feats = torch.randn(n, C, generator=g).cuda()
    coords = torch.stack([torch.randint(0, H, (n,), generator=g), torch.randint(0, W, (n,), generator=g),
                          torch.randint(0, D, (n,), generator=g), torch.randint(0, B, (n,), generator=g)], 1).cuda()
    assert torch.equal(legacy(feats, coords, B, D, H, W), current(feats, coords, B, D, H, W))
    with pytest.raises(AssertionError):
        legacy(feats[:-1], coords, B, D, H, W)
