"""The allocation-free bev_pool forward, called through the C ABI.

Some callers cannot allocate GPU memory while they run (a real-time loop in
which cudaMalloc would stall, or code that does not own an allocator).  For
them bfb_bev_pool_forward_noalloc works out of a fixed device array inside
the library.  This test checks, on two calls in a row, that it returns the
same output as the regular entry point (bit-identical: the kernels are
deterministic and the fp32 tests of this suite compare exactly), and that a
size beyond the array is refused.  It lives in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests._util import rand_bev_case

pytestmark = pytest.mark.gpu

i64 = ctypes.c_int64
vp = ctypes.c_void_p


def _lib():
    from bevfusion_triton_b200 import load_native
    L = load_native()
    L.bfb_bev_pool_noalloc_capacity.restype = ctypes.c_size_t
    return L


def _regular(L, feats, coords, shape, stream):
    n, c = feats.shape
    plan_b, scr_b = ctypes.c_size_t(), ctypes.c_size_t()
    assert L.bfb_bev_pool_workspace_sizes(i64(n), i64(c), *[i64(x) for x in shape], ctypes.byref(plan_b),
                                          ctypes.byref(scr_b)) == 0
    plan = torch.empty(plan_b.value, dtype=torch.uint8, device='cuda')
    scr = torch.empty(scr_b.value, dtype=torch.uint8, device='cuda')
    out = torch.empty((shape[0], c, *shape[1:]), device='cuda')
    rc = L.bfb_bev_pool_forward(vp(feats.data_ptr()), 0, vp(coords.data_ptr()), 1, i64(n), i64(c),
                                *[i64(x) for x in shape], vp(out.data_ptr()), vp(plan.data_ptr()), plan_b,
                                vp(scr.data_ptr()), scr_b, stream)
    assert rc == 0
    return out


def _noalloc(L, feats, coords, shape, stream):
    n, c = feats.shape
    out = torch.full((shape[0], c, *shape[1:]), float('nan'), device='cuda')
    rc = L.bfb_bev_pool_forward_noalloc(vp(feats.data_ptr()), 0, vp(coords.data_ptr()), 1, i64(n), i64(c),
                                        *[i64(x) for x in shape], vp(out.data_ptr()), stream)
    assert rc == 0
    return out


def test_noalloc_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip('CUDA device required')
    L = _lib()
    stream = vp(torch.cuda.current_stream().cuda_stream)
    cases = [(rand_bev_case(200000, 80, 2, 1, 120, 130, seed=21, hot=30000), (2, 1, 120, 130)),
             (rand_bev_case(50000, 80, 1, 2, 64, 40, seed=22, invalid=333), (1, 2, 64, 40))]
    for (feats, coords), shape in cases:  # two calls in a row, different inputs
        feats, coords = feats.cuda(), coords.cuda()
        got = _noalloc(L, feats, coords, shape, stream)
        want = _regular(L, feats, coords, shape, stream)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())


def test_noalloc_refuses_sizes_beyond_its_array():
    """A grid whose plan exceeds the fixed array is refused.  Every buffer
    handed over is a real device allocation sized for the call (16 in-grid
    points, 4 channels, a 4096 x 4096 grid whose per-cell plan table alone
    needs 128 MiB), so the call is valid apart from the size limit."""
    if not torch.cuda.is_available():
        pytest.skip('CUDA device required')
    L = _lib()
    cap = L.bfb_bev_pool_noalloc_capacity()
    shape = (1, 1, 4096, 4096)
    assert (shape[2] * shape[3] + 1) * 8 > cap
    feats, coords = rand_bev_case(16, 4, *shape, seed=23, cdtype=torch.int64)
    feats, coords = feats.cuda(), coords.cuda()
    out = torch.full((1, 4, 1, 4096, 4096), 5.0, device='cuda')
    rc = L.bfb_bev_pool_forward_noalloc(vp(feats.data_ptr()), 0, vp(coords.data_ptr()), 1, i64(16), i64(4),
                                        *[i64(x) for x in shape], vp(out.data_ptr()),
                                        vp(torch.cuda.current_stream().cuda_stream))
    assert rc == -4  # BFB_ERR_TOO_LARGE, before any device work
    torch.cuda.synchronize()
    assert bool((out == 5.0).all())
