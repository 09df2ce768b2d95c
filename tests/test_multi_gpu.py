"""Sharded run on two GPUs (one process per GPU, NCCL) against the same batch
on one GPU: each rank pools and voxelises its own contiguous block of
samples with no collective on the path; the ragged all-gather then assembles
the per-rank outputs, which must equal the single-GPU batch bit for bit.
Skipped when fewer than two GPUs are visible."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

BATCH = 4  # det camera samples and LiDAR samples, split 2 + 2


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _shard_outputs(first, count, device):
    """bev_pool fwd + bwd of det samples [first, first + count) and hard
    voxelisation of LiDAR samples of the same ids, on `device`."""
    from tests import synth
    from bevfusion_triton_b200.ops.bev_pool import bev_pool
    from bevfusion_triton_b200.ops.voxel.voxel_layer import hard_voxelize_batch
    case = synth.det_bev_pool_case(count, device=device, sample_offset=first)
    x = case.feats.clone().requires_grad_(True)
    out = bev_pool(x, case.coords, case.B, case.D, case.H, case.W)
    up = []
    for s in range(first, first + count):  # per-sample upstream gradient
        g = torch.Generator(device=device).manual_seed(1000 + s)
        up.append(torch.randn((1,) + tuple(out.shape[1:]), generator=g, device=device))
    out.backward(torch.cat(up))
    pts = [synth.lidar_sweeps(first + i).to(device) for i in range(count)]
    offs = [0]
    for p in pts:
        offs.append(offs[-1] + p.size(0))
    V, C, N, VN = hard_voxelize_batch(torch.cat(pts), offs, list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE),
                                      synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS)
    vox = torch.cat([V[i, :int(VN[i])].reshape(-1) for i in range(count)])
    coors = torch.cat([C[i, :int(VN[i])].reshape(-1) for i in range(count)])
    return out.detach().reshape(count, -1), x.grad.reshape(count, -1), vox, coors, VN


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        from bevfusion_triton_b200.shard import gather_ragged, shard_samples
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        torch.cuda.set_device(rank)
        dist.init_process_group('nccl', rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device('cuda', rank))
        first, count = shard_samples(BATCH, world, rank)
        outs = _shard_outputs(first, count, torch.device('cuda', rank))
        gathered = [torch.cat(gather_ragged(t)) for t in outs]
        if rank == 0:
            full = _shard_outputs(0, BATCH, torch.device('cuda', 0))
            names = ['bev_out', 'bev_grad', 'voxels', 'coors', 'voxel_num']
            q.put({n: bool(torch.equal(a, b)) for n, a, b in zip(names, gathered, full)})
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put({'error': f'rank {rank}: {e!r}'})


def test_two_gpu_shards_match_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs two GPUs')
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=180)
            if p.is_alive():  # only our own child processes
                p.terminate()
    assert 'error' not in res, res['error']
    assert all(res.values()), res
