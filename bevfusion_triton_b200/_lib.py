"""Loads the in-tree native libraries; fails loudly when they are missing.

The libraries are built by ``bevfusion_triton_b200._build`` (or
``__graft_entry__.build()``).  There is deliberately no fallback: an op
called without them raises instead of running some other implementation.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

PKG = Path(__file__).resolve().parent
LIB = PKG / 'libbfb_b200.so'
TORCH_LIB = PKG / '_bfb_torch.so'

_loaded = False
_cdll = None


def native_paths() -> tuple[Path, Path]:
    return LIB, TORCH_LIB


def load_native():
    """Load libbfb_b200.so (ctypes handle, returned) and register the
    ``torch.ops.bfb_b200`` custom ops."""
    global _loaded, _cdll
    if _loaded:
        return _cdll
    for p in (LIB, TORCH_LIB):
        if not p.exists():
            raise RuntimeError(
                f'native library {p.name} is missing; build it with '
                '`python -m bevfusion_triton_b200._build` (no CPU fallback exists)')
    _cdll = ctypes.CDLL(str(LIB), mode=ctypes.RTLD_GLOBAL)
    torch.ops.load_library(str(TORCH_LIB))
    _loaded = True
    from .ops import _registry  # fake kernels + autograd of the ops just loaded
    _registry.register()
    return _cdll


def ops():
    load_native()
    return torch.ops.bfb_b200


def bev_pool_plan_bytes(n: int, B: int, D: int, H: int, W: int) -> int:
    """Size in bytes of a bev_pool plan for (n, B, D, H, W): a host-only query
    of the C ABI (no GPU needed).  Raises ValueError for sizes it refuses."""
    lib = load_native()
    plan = ctypes.c_size_t(0)
    st = lib.bfb_bev_pool_workspace_sizes(ctypes.c_int64(n), ctypes.c_int64(1), ctypes.c_int64(B),
                                          ctypes.c_int64(D), ctypes.c_int64(H), ctypes.c_int64(W),
                                          ctypes.byref(plan), None)
    if st != 0:
        raise ValueError(f'bev_pool geometry (n={n}, B={B}, D={D}, H={H}, W={W}) is refused (status {st})')
    return plan.value
