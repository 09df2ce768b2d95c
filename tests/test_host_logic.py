"""Host-side logic that needs no GPU: the C-ABI library loads and exports
every declared symbol, argument validation, workspace queries, error types
of the Python drop-ins (tests/test_ops/test_bev_pool.py:122-131 style)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / 'include').glob('*.h'):
        names |= set(re.findall(r'^\s*(?:int|const char\*|size_t|void|uint64_t)\s+(bfb_\w+)\s*\(', h.read_text(), re.M))
    return sorted(names)


@pytest.fixture(scope='module')
def cabi():
    from bevfusion_triton_b200 import load_native
    return load_native()


def test_header_declares_symbols():
    assert len(declared_symbols()) >= 10


def test_cabi_exports_every_declared_symbol(cabi):
    missing = [n for n in declared_symbols() if not hasattr(cabi, n)]
    assert not missing, missing


def test_version_and_status_strings(cabi):
    assert cabi.bfb_abi_version() == 2
    cabi.bfb_status_string.restype = ctypes.c_char_p
    assert cabi.bfb_status_string(0) == b'ok'
    assert cabi.bfb_status_string(-3).startswith(b'workspace')
    assert cabi.bfb_status_string(12345) == b'unknown status'


def _i64(*v):
    return [ctypes.c_int64(x) for x in v]


def test_bev_pool_workspace_query(cabi):
    plan, scratch = ctypes.c_size_t(), ctypes.c_size_t()
    rc = cabi.bfb_bev_pool_workspace_sizes(*_i64(1770765, 80, 8, 1, 360, 360), ctypes.byref(plan), ctypes.byref(scratch))
    assert rc == 0
    assert plan.value >= 2 * 4 * 1770765 and scratch.value >= 2 * 4 * 1770765
    # monotone in n
    plan2 = ctypes.c_size_t()
    assert cabi.bfb_bev_pool_workspace_sizes(*_i64(10, 80, 8, 1, 360, 360), ctypes.byref(plan2), None) == 0
    assert plan2.value < plan.value


@pytest.mark.parametrize('args,code', [
    ((10, 80, 0, 1, 2, 2), -1),       # B = 0
    ((-1, 80, 1, 1, 2, 2), -1),       # negative n
    ((10, 80, 1 << 20, 1 << 12, 1, 1), -4),  # > 2^31 cells
])
def test_bev_pool_bad_sizes(cabi, args, code):
    a = ctypes.c_size_t()
    assert cabi.bfb_bev_pool_workspace_sizes(*_i64(*args), ctypes.byref(a), ctypes.byref(a)) == code


def test_bev_pool_rejects_missing_workspace(cabi):
    rc = cabi.bfb_bev_pool_plan(ctypes.c_void_p(16), 1, *_i64(10, 1, 1, 2, 2), None, ctypes.c_size_t(0),
                                None, ctypes.c_size_t(0), None)
    assert rc == -3


def test_bev_pool_rejects_bad_itype(cabi):
    rc = cabi.bfb_bev_pool_plan(ctypes.c_void_p(16), 7, *_i64(10, 1, 1, 2, 2), ctypes.c_void_p(16),
                                ctypes.c_size_t(1 << 30), ctypes.c_void_p(16), ctypes.c_size_t(1 << 30), None)
    assert rc == -2


def test_bev_pool_rejects_invalid_inputs():
    """Same exception types as the reference (test_bev_pool.py:122-131)."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool
    feats = torch.randint(0, 4, (4, 3), dtype=torch.int32)
    coords = torch.zeros((4, 4), dtype=torch.int32)
    with pytest.raises(TypeError):
        bev_pool(feats, coords, 1, 1, 1, 1)
    feats = torch.randn((4, 3), dtype=torch.float32)
    with pytest.raises(TypeError):
        bev_pool(feats, torch.zeros((4, 4), dtype=torch.float32), 1, 1, 1, 1)
    with pytest.raises(ValueError):
        bev_pool(torch.randn(4), coords, 1, 1, 1, 1)
    with pytest.raises(ValueError):
        bev_pool(feats, torch.zeros((4, 3), dtype=torch.int32), 1, 1, 1, 1)
    with pytest.raises(ValueError):
        bev_pool(feats, torch.zeros((5, 4), dtype=torch.int32), 1, 1, 1, 1)
    with pytest.raises(ValueError):
        bev_pool(feats, coords, 0, 1, 1, 1)


def test_bev_pool_has_no_cpu_path():
    from bevfusion_triton_b200.ops.bev_pool import bev_pool
    with pytest.raises(RuntimeError, match='CUDA'):
        bev_pool(torch.randn(4, 3), torch.zeros((4, 4), dtype=torch.int32), 1, 1, 1, 1)


def test_rulebook_output_shapes_and_checks(cabi):
    """ops/spconv/ops.py:25-50 output-size helpers, the rulebook's argument
    errors (before any device work) and the C-ABI workspace query."""
    from bevfusion_triton_b200.ops.spconv import get_conv_output_size, get_deconv_output_size, get_indice_pairs
    assert get_conv_output_size([1440, 1440, 41], [3, 3, 3], [2, 2, 2], [1, 1, 1], [1, 1, 1]) == [720, 720, 21]
    assert get_conv_output_size([8, 8], [-1, 3], [1, 1], [0, 0], [1, 1]) == [1, 6]
    assert get_deconv_output_size([5, 6], [3, 3], [2, 2], [1, 1], [1, 1], [0, 0]) == [9, 11]
    with pytest.raises(ValueError):
        get_deconv_output_size([5], [-1], [1], [0], [1], [0])
    idx = torch.zeros((3, 4), dtype=torch.int32)
    with pytest.raises(ValueError):
        get_indice_pairs(idx, 0, [8, 8, 8])
    with pytest.raises(RuntimeError, match='CUDA'):
        get_indice_pairs(idx, 1, [8, 8, 8])
    ws = ctypes.c_size_t()
    shape = (ctypes.c_int64 * 3)(720, 720, 21)
    ks = (ctypes.c_int64 * 3)(3, 3, 3)
    assert cabi.bfb_indice_pairs_workspace_size(ctypes.c_int64(1000), 3, ctypes.c_int64(8), shape, ks, 0,
                                                ctypes.byref(ws)) == 0
    assert ws.value >= 8 * 720 * 720 * 21 // 8  # one bit per output cell
    big = (ctypes.c_int64 * 3)(1 << 20, 1 << 20, 8)
    assert cabi.bfb_indice_pairs_workspace_size(ctypes.c_int64(10), 3, ctypes.c_int64(1), big, ks, 0,
                                                ctypes.byref(ws)) == -4  # cells must fit 32 bits


def test_bev_grid_matches_reference_formula():
    """gen_dx_bx + the lower edge of models/vtransforms/base.py:19-23,138."""
    from bevfusion_triton_b200.ops.bev_pool import bev_grid
    lower, dx, nx = bev_grid((-54.0, 54.0, 0.3), (-54.0, 54.0, 0.3), (-10.0, 10.0, 20.0))
    assert nx == [360, 360, 1]
    d = torch.tensor([0.3, 0.3, 20.0])
    b = torch.tensor([-54.0 + 0.15, -54.0 + 0.15, 0.0])
    assert lower == (b - d / 2.0).tolist() and dx == d.tolist()


def test_plan_of_another_geometry_is_refused():
    """A plan kept for a fixed rig and handed a short last batch (fewer points,
    smaller B) must be refused before any device work."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool_planned, check_plan
    from bevfusion_triton_b200._lib import bev_pool_plan_bytes
    full = bev_pool_plan_bytes(200_000, 8, 1, 64, 64)
    plan = torch.zeros(full, dtype=torch.uint8)
    check_plan(plan, 200_000, 8, 1, 64, 64)  # its own geometry passes
    with pytest.raises(ValueError, match='another geometry'):
        check_plan(plan, 100_000, 4, 1, 64, 64)
    feats = torch.zeros(100_000, 8)
    with pytest.raises(ValueError, match='another geometry'):
        bev_pool_planned(feats, plan, 4, 1, 64, 64)
    with pytest.raises(ValueError, match='uint8'):
        check_plan(plan.view(torch.int32), 200_000, 8, 1, 64, 64)


def test_plan_mismatch_status_string(cabi):
    cabi.bfb_status_string.restype = ctypes.c_char_p
    assert b'another geometry' in cabi.bfb_status_string(-7)


def test_status_injection_returns_before_touching_arguments(cabi):
    """Host-side fault injection: an armed status is returned by the next
    entry-point calls without reading their (here invalid) pointers; then the
    entry point validates its arguments as usual."""
    i64 = ctypes.c_int64
    assert cabi.bfb_debug_inject_status(-5, 2) == 0
    args = (None, 1, i64(10), i64(1), i64(1), i64(2), i64(2), None, ctypes.c_size_t(0), None, ctypes.c_size_t(0),
            None)
    assert cabi.bfb_bev_pool_plan(*args) == -5
    assert cabi.bfb_bev_pool_plan(*args) == -5
    assert cabi.bfb_bev_pool_plan(*args) == -3  # disarmed: the missing workspace is reported
    assert cabi.bfb_debug_inject_status(-1, 5) == 0
    assert cabi.bfb_debug_inject_status(0, 0) == 0  # disarm
    assert cabi.bfb_bev_pool_plan(*args) == -3
    assert cabi.bfb_debug_inject_status(3, 1) == -1  # a positive status is not a status


def test_release_build_has_no_debug_checks(cabi):
    cabi.bfb_debug_checks_enabled.restype = ctypes.c_int
    assert cabi.bfb_debug_checks_enabled() == 0


def test_sparse_conv_argument_checks(cabi):
    """Size queries and argument checks of the sparse-convolution entry
    points, host side only (no launch)."""
    sz = ctypes.c_size_t()
    q = cabi.bfb_indice_conv_workspace_size
    q.argtypes = [ctypes.c_int64] * 6 + [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t)]
    assert q(1000, 900, 27, 64, 64, 1000, 1, 0, ctypes.byref(sz)) == 0 and sz.value > 0
    fwd = sz.value
    assert q(1000, 900, 27, 64, 64, 1000, 1, 1, ctypes.byref(sz)) == 0 and sz.value > fwd  # + backward parts
    assert q(1000, 900, 343, 300, 260, 1000, 0, 1, ctypes.byref(sz)) == 0  # any width, up to 7x7x7
    assert q(1000, 900, 344, 64, 64, 1000, 0, 0, ctypes.byref(sz)) == -1  # kernel volume past 7x7x7
    assert q(1000, 900, 0, 64, 64, 1000, 0, 0, ctypes.byref(sz)) == -1
    assert q(-1, 900, 27, 64, 64, 1000, 0, 0, ctypes.byref(sz)) == -1
    assert q(1000, 900, 27, 64, 64, 1000, 9, 0, ctypes.byref(sz)) == -2  # dtype code
    assert q(1 << 30, 900, 27, 64, 64, 1000, 0, 0, ctypes.byref(sz)) == -4  # n * K past 32 bits
    m = cabi.bfb_indice_maxpool_workspace_size
    m.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t)]
    assert m(1000, 300, 27, 0, ctypes.byref(sz)) == 0 and sz.value >= 300 * 27 * 4
    assert m(1000, 300, 27, 1, ctypes.byref(sz)) == 0 and sz.value >= 1000 * 27 * 4
