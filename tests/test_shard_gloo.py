"""Host logic of the multi-rank path on CPU: world_size 2 over gloo
(127.0.0.1), including a rank that never joins a collective."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bevfusion_triton_b200.shard import gather_ragged, max_over_ranks, shard_samples, sum_over_ranks


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


@pytest.mark.parametrize('batch,world', [(64, 8), (64, 3), (5, 4), (0, 2), (8, 1)])
def test_shard_samples_partition(batch, world):
    seen = []
    for r in range(world):
        first, count = shard_samples(batch, world, r)
        seen.extend(range(first, first + count))
    assert seen == list(range(batch))
    counts = [shard_samples(batch, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_shard_samples_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_samples(8, 2, 2)


def _worker_collectives(rank, world, port, q):
    try:
        _init(rank, world, port)
        first, count = shard_samples(7, world, rank)
        # a ragged per-rank output: one row per sample, rows hold the sample id
        local = torch.arange(first, first + count, dtype=torch.float32).unsqueeze(1).repeat(1, 3)
        parts = gather_ragged(local)
        full = torch.cat(parts)
        ok = torch.equal(full[:, 0], torch.arange(7, dtype=torch.float32))
        mx = max_over_ranks(float(rank + 1))
        sm = sum_over_ranks(float(rank + 1))
        q.put((rank, ok, mx, sm))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), None, None))


def test_gather_and_reductions_world2():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_collectives, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, ok, mx, sm in res:
        assert ok is True, ok
        assert mx == 2.0 and sm == 3.0


def _worker_dropout(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, 'left'))  # leaves between steps, joins no collective
        return
    try:
        max_over_ranks(1.0)
        q.put((rank, 'no error'))
    except Exception as e:
        q.put((rank, 'error:' + type(e).__name__))


def test_rank_that_leaves_is_detected_by_timeout():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dropout, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == 'left'
    assert res[0].startswith('error:')
