"""Batch-sample sharding over ranks (one process per GPU).

The hot path shards by sample: bev_pool cells never mix across samples and
voxelisation is per sample, so each rank runs the same kernels on its own
contiguous block of samples and no collective is needed on the path.  The
helpers here are host logic: the shard of a rank, reductions used for
timing (max over ranks), and a ragged all-gather that assembles per-rank
outputs of different lengths (voxel counts differ) on every rank, used only
to check a sharded run against a single-GPU run.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_samples(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first sample, number of samples) of `rank`: contiguous, sizes differ by
    at most one, lower ranks take the remainder."""
    if world < 1 or not 0 <= rank < world or global_batch < 0:
        raise ValueError('bad world / rank / batch')
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    first = rank * base + min(rank, extra)
    return first, count


def _reduce(x: float, op, device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(x: float, device='cpu') -> float:
    return _reduce(x, dist.ReduceOp.MAX, device)


def sum_over_ranks(x: float, device='cpu') -> float:
    return _reduce(x, dist.ReduceOp.SUM, device)


def gather_ragged(t: torch.Tensor) -> list[torch.Tensor]:
    """All-gather tensors whose first dimension differs per rank (same
    trailing shape and dtype): sizes first, then a padded all_gather."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [t]
    world = dist.get_world_size()
    n = torch.tensor([t.size(0)], dtype=torch.int64, device=t.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    sizes = [int(s.item()) for s in sizes]
    m = max(sizes)
    pad = t.new_zeros((m,) + tuple(t.shape[1:]))
    pad[: t.size(0)] = t
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad)
    return [b[:s] for b, s in zip(bufs, sizes)]
