"""Diagnostics on the GPU: statuses injected on the host surface as the
reference's exception types through the torch ops and leave the library
usable; the debug build (device index checks counted into an error word)
runs the hot path with no violation and counts synthetic ones."""
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

from bevfusion_triton_b200._lib import load_native
from bevfusion_triton_b200.ops.bev_pool import bev_pool
from bevfusion_triton_b200.ops.voxel.voxel_layer import hard_voxelize
from tests import synth
from tests._util import rand_bev_case

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
DEBUG_LIB = ROOT / 'bevfusion_triton_b200' / 'debug' / 'libbfb_b200.so'


def test_injected_status_raises_and_recovers(cuda):
    L = load_native()
    feats, coords = rand_bev_case(5000, 16, 1, 1, 20, 20, seed=41)
    feats, coords = feats.cuda(), coords.cuda()
    want = bev_pool(feats, coords, 1, 1, 20, 20)
    L.bfb_debug_inject_status(-5, 1)
    with pytest.raises(RuntimeError, match='CUDA error'):
        bev_pool(feats, coords, 1, 1, 20, 20)
    L.bfb_debug_inject_status(-1, 1)
    with pytest.raises(ValueError):
        bev_pool(feats, coords, 1, 1, 20, 20)
    assert torch.equal(bev_pool(feats, coords, 1, 1, 20, 20), want)
    # a failed voxelisation drops the cached hash table; the next call rebuilds it
    pts = synth.lidar_sweeps(0).cuda()
    vs, cr = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)

    def run():
        v = torch.zeros((120000, 10, 5), device='cuda')
        c = torch.zeros((120000, 3), dtype=torch.int32, device='cuda')
        n = torch.zeros((120000,), dtype=torch.int32, device='cuda')
        return hard_voxelize(pts, v, c, n, vs, cr, 10, 120000), v, c, n

    a = run()
    L.bfb_debug_inject_status(-5, 1)
    with pytest.raises(RuntimeError):
        run()
    b = run()
    assert a[0] == b[0] and all(torch.equal(x, y) for x, y in zip(a[1:], b[1:]))


DEBUG_SCRIPT = textwrap.dedent('''
    import ctypes, sys, torch
    L = ctypes.CDLL(sys.argv[1])
    i64, vp = ctypes.c_int64, ctypes.c_void_p
    assert L.bfb_debug_checks_enabled() == 1
    cnt = ctypes.c_uint64()
    st = vp(torch.cuda.current_stream().cuda_stream)
    assert L.bfb_debug_violations(ctypes.byref(cnt), 1) == 0
    g = torch.Generator().manual_seed(3)
    n, c, B, D, H, W = 40000, 32, 2, 1, 64, 48
    feats = torch.randn((n, c), generator=g).cuda()
    coords = torch.stack([torch.randint(0, H, (n,), generator=g), torch.randint(0, W, (n,), generator=g),
                          torch.zeros(n, dtype=torch.long), torch.randint(0, B, (n,), generator=g)], 1).cuda()
    pb, sb = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.bfb_bev_pool_workspace_sizes(i64(n), i64(c), i64(B), i64(D), i64(H), i64(W), ctypes.byref(pb),
                                          ctypes.byref(sb)) == 0
    plan = torch.empty(pb.value, dtype=torch.uint8, device='cuda')
    scr = torch.empty(sb.value, dtype=torch.uint8, device='cuda')
    out = torch.empty((B, c, D, H, W), device='cuda')
    assert L.bfb_bev_pool_forward(vp(feats.data_ptr()), 0, vp(coords.data_ptr()), 1, i64(n), i64(c), i64(B),
                                  i64(D), i64(H), i64(W), vp(out.data_ptr()), vp(plan.data_ptr()), pb,
                                  vp(scr.data_ptr()), sb, st) == 0
    up = torch.randn(out.shape, generator=g).cuda()
    gf = torch.empty_like(feats)
    rb = ctypes.c_size_t()
    assert L.bfb_bev_pool_backward_workspace_size(i64(n), i64(c), i64(B), i64(D), i64(H), i64(W), 0,
                                                  ctypes.byref(rb)) == 0
    rows = torch.empty(rb.value, dtype=torch.uint8, device='cuda')
    assert L.bfb_bev_pool_backward_gather(vp(up.data_ptr()), 0, i64(n), i64(c), i64(B), i64(D), i64(H), i64(W),
                                          vp(plan.data_ptr()), pb, vp(gf.data_ptr()), vp(rows.data_ptr()), rb,
                                          st) == 0
    torch.cuda.synchronize()
    ref = torch.zeros((B * D * H * W, c), device='cuda').index_add_(
        0, (coords[:, 3] * H + coords[:, 0]) * W + coords[:, 1], feats)
    assert torch.allclose(out, ref.view(B, H, W, c).permute(0, 3, 1, 2).unsqueeze(2), atol=1e-4)
    assert L.bfb_debug_violations(ctypes.byref(cnt), 0) == 0 and cnt.value == 0, cnt.value
    assert L.bfb_debug_selftest(7, st) == 0
    torch.cuda.synchronize()
    assert L.bfb_debug_violations(ctypes.byref(cnt), 1) == 0 and cnt.value == 7, cnt.value
    assert L.bfb_debug_violations(ctypes.byref(cnt), 0) == 0 and cnt.value == 0
    print('ok')
''')


def test_debug_build_counts_violations(cuda):
    if not DEBUG_LIB.exists():
        pytest.skip('debug build missing (python -m bevfusion_triton_b200._build --debug-checks)')
    r = subprocess.run([sys.executable, '-c', DEBUG_SCRIPT, str(DEBUG_LIB)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith('ok'), r.stdout + r.stderr
