"""Shared helpers for the tests (hashing, seeded case builders)."""
from __future__ import annotations

import hashlib

import numpy as np
import torch


def sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu().numpy()
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.tobytes()).hexdigest()


def rand_bev_case(n, c, B, D, H, W, seed, cdtype=torch.int64, fdtype=torch.float32, hot=None, invalid=0):
    """Seeded random bev_pool inputs (CPU tensors).  ``hot`` piles that many
    points into three cells; ``invalid`` puts that many points off the grid."""
    g = torch.Generator().manual_seed(seed)
    feats = torch.randn((n, c), generator=g).to(fdtype)
    coords = torch.stack([
        torch.randint(0, H, (n,), generator=g), torch.randint(0, W, (n,), generator=g),
        torch.randint(0, D, (n,), generator=g), torch.randint(0, B, (n,), generator=g)], 1)
    if hot:
        idx = torch.randperm(n, generator=g)[:hot]
        cells = torch.tensor([[0, 0, 0, 0], [H // 2, W // 2, D - 1, B - 1], [H - 1, W - 1, D - 1, B - 1]])
        coords[idx] = cells[torch.randint(0, 3, (hot,), generator=g)]
    if invalid:
        idx = torch.randperm(n, generator=g)[:invalid]
        bad = torch.tensor([[-1, 0, 0, 0], [H, 0, 0, 0], [0, W, 0, 0], [0, 0, D, 0], [0, 0, 0, B], [0, -5, 0, 0]])
        coords[idx] = bad[torch.randint(0, bad.size(0), (invalid,), generator=g)]
    return feats.contiguous(), coords.to(cdtype).contiguous()
