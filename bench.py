#!/usr/bin/env python
"""Benchmark of the BEVFusion grid scatter-reduce hot path on B200.

One step on every GPU = config 1 of BASELINE.json (det bev_pool forward +
backward over a batch of 8 camera samples, fp32, 1,770,765 points x 80
channels per sample, 360 x 360 grid) plus hard voxelisation of a batch of 8
synthetic LiDAR sweeps (config 3 shape, 346,880 points each).  Sample i of
rank r is sample r * 8 + i of one global batch, so 8 GPUs run exactly the
batch-64 scaling sweep (config 5); per-GPU work is fixed ("weak" scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` is milliseconds per sample over the
whole job (step time, max over ranks, divided by all samples of all ranks),
with inputs resident in HBM; `e2e` is the same metric through the public
Python API with the step's inputs copied from pinned host memory and its
outputs copied back inside the timed region.  `--impl reference` times the
reference's own CPU algorithms (oracle/ref_cpu.py) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from bevfusion_triton_b200 import shard  # noqa: E402
from tests import synth  # noqa: E402

METRIC = 'bev_pool fwd+bwd & voxelize ms/sample and GB/s (% of B200 HBM peak), 1/2/4/8 GPU'
UNIT = 'ms/sample'
SAMPLES_PER_GPU = 8
C = synth.CHANNELS
FALLBACK_HBM_GBS = 6650.0

# DRAM traffic (read + write bytes) of the dominant kernels per point, from an
# ncu capture of a one-sample launch; traffic grows in proportion to the
# points, so a launch's traffic is this times its points.
NCU_TRAFFIC_PER_POINT = {
    'bev_fwd_kernel': 340.6,
    # backward: bev_rows_kernel (37.3 MB) + bev_gather_kernel (533.7 MB) of one sample
    'bev_rows_kernel+bev_gather_kernel': 322.4,
}


def measured_peak():
    p = ROOT / 'MEASURED_PEAKS.json'
    try:
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    except Exception:
        return FALLBACK_HBM_GBS, 'fallback'


# ------------------------------------------------------------------ dist
def dist_setup(args):
    ws = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if ws > 1:
        import torch.distributed as dist
        backend = 'nccl' if torch.cuda.is_available() else 'gloo'
        if backend == 'nccl':
            torch.cuda.set_device(local)
            dist.init_process_group(backend, timeout=timedelta(seconds=600),
                                    device_id=torch.device('cuda', local))
        else:
            dist.init_process_group(backend, timeout=timedelta(seconds=600))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    return shard.max_over_ranks(x, 'cuda' if torch.cuda.is_available() else 'cpu')


def sum_over_ranks(x: float, ws: int) -> float:
    return shard.sum_over_ranks(x, 'cuda' if torch.cuda.is_available() else 'cpu')


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []

    def _gpu_id(self):
        try:
            p = torch.cuda.get_device_properties(self.dev)
            return f'{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0'
        except Exception:
            return None

    def start(self):
        cmd = ['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits', '-lms', '100']
        gid = self._gpu_id()
        if gid:
            cmd += ['-i', gid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith('active'):
                    reasons.add(nm)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons), 'samples': len(sm)}


# ------------------------------------------------------------------ inputs
def upstream_grad(sample: int, case, device):
    """N(0, 1) upstream gradient of one det sample, seeded by the sample's
    index in the global batch (any shard reproduces it)."""
    g = torch.Generator(device=device)
    g.manual_seed(1000 + sample)
    return torch.randn((1, C, case.D, case.H, case.W), generator=g, device=device)


def checksum(*ts) -> int:
    """Order-sensitive integer checksum of tensors' bytes (bit-exact results
    give equal checksums on any GPU)."""
    acc = 0
    for t in ts:
        w = t.detach().contiguous().view(-1).view(torch.int32).to(torch.int64)
        k = torch.arange(1, w.numel() + 1, device=w.device, dtype=torch.int64) % 65521
        acc = (acc * 1000003 + int((w * k).sum().item())) % (1 << 61)
    return acc


class Workload:
    """The rank's shard: det bev_pool batch + LiDAR batch, resident on the GPU."""

    def __init__(self, rank: int, samples: int, device, world: int = 1, sample_offset=None):
        self.S = samples
        if sample_offset is None:
            first, count = shard.shard_samples(samples * world, world, rank)
            assert count == samples
        else:
            first = sample_offset
        case = synth.det_bev_pool_case(samples, device=device, sample_offset=first)
        self.feats, self.coords = case.feats, case.coords
        self.shape = (case.B, case.D, case.H, case.W)
        self.n = self.feats.size(0)
        self.first = first
        self.up = torch.cat([upstream_grad(first + i, case, device) for i in range(samples)])
        dhw = case.D * case.H * case.W
        r = (self.coords[:, 3] * dhw + (self.coords[:, 2] * case.H + self.coords[:, 0]) * case.W + self.coords[:, 1])
        self.nonempty = int(torch.unique(r).numel())
        clouds = [synth.lidar_sweeps(first + i) for i in range(samples)]
        self.offs = [0]
        for c in clouds:
            self.offs.append(self.offs[-1] + c.size(0))
        self.points_cpu = torch.cat(clouds)
        self.points = self.points_cpu.to(device)
        self.vsize, self.crange = list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE)
        self.mp, self.mv = synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS
        F = self.points.size(1)
        self.voxels = torch.empty((samples, self.mv, self.mp, F), device=device)
        self.vcoors = torch.empty((samples, self.mv, 3), dtype=torch.int32, device=device)
        self.vnum = torch.empty((samples, self.mv), dtype=torch.int32, device=device)
        self.vn = torch.empty((samples,), dtype=torch.int32, device=device)

    # algorithmic bytes per rank: fwd = N*C*4 + N*4*8 + B*C*D*H*W*4, bwd = N*C*4 + N*4*8 + U*C*4
    # (U non-empty cells), voxelize = N*F*4 + M*(P*F*4 + 3*4 + 4) (M voxels)
    def bytes_fwd(self):
        B, D, H, W = self.shape
        return self.n * C * 4 + self.n * 4 * 8 + B * C * D * H * W * 4

    def bytes_bwd(self):
        return self.n * C * 4 + self.n * 4 * 8 + self.nonempty * C * 4

    def bytes_vox(self, vn_total: int):
        F = self.points.size(1)
        return self.points.numel() * 4 + vn_total * (self.mp * F * 4 + 3 * 4 + 4)


def run_ours(args, ws, rank, local):
    from bevfusion_triton_b200 import load_native
    from bevfusion_triton_b200._lib import ops
    cdll = load_native()
    cdll.bfb_kernel_launches.restype = ctypes.c_uint64
    O = ops()
    dev = torch.device('cuda', local)
    wl = Workload(rank, args.samples_per_gpu, dev, ws)
    B, D, H, W = wl.shape
    stream = torch.cuda.current_stream()
    # the LiDAR branch, concurrent with the camera branch
    s_lid = torch.cuda.Stream(priority=-1 if args.lidar_priority else 0)

    def lidar(ev):
        if ev:
            ev[4].record(torch.cuda.current_stream())
        O.hard_voxelize_batch(wl.points, wl.offs, wl.voxels, wl.vcoors, wl.vnum, wl.vn, wl.vsize, wl.crange,
                              wl.mp, wl.mv, False)
        if ev:
            ev[5].record(torch.cuda.current_stream())

    def step(ev=None):
        """det bev_pool plan + forward + backward and the LiDAR voxelisation.
        The two branches are independent: by default the voxelisation (a
        latency-bound chain) runs on its own stream beside the plan (also
        latency-bound), and the step ends when both have finished; --serial
        runs them one after the other on one stream, --lidar-beside gather
        starts it after the plan."""
        if not args.serial and args.lidar_beside == 'plan':
            s_lid.wait_stream(stream)
            with torch.cuda.stream(s_lid):
                lidar(ev)
        if ev:
            ev[0].record(stream)
        plan = O.bev_pool_plan(wl.coords, B, D, H, W)
        if ev:
            ev[1].record(stream)
        if not args.serial and args.lidar_beside == 'gather':
            s_lid.wait_stream(stream)
            with torch.cuda.stream(s_lid):
                lidar(ev)
        out = O.bev_pool_forward_planned(wl.feats, plan, B, D, H, W)
        if ev:
            ev[2].record(stream)
        g = O.bev_pool_backward(wl.up, plan, wl.n, B, D, H, W)
        if ev:
            ev[3].record(stream)
        if args.serial:
            lidar(ev)
        else:
            stream.wait_stream(s_lid)
        return out, g

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(ws)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)
    launches0 = cdll.bfb_kernel_launches()
    torch.cuda.synchronize()
    barrier(ws)
    t0.record(stream)
    for k in range(args.steps):
        out_last, g_last = step(evs[k])
    t1.record(stream)
    torch.cuda.synchronize()
    barrier(ws)
    launches = int(cdll.bfb_kernel_launches() - launches0)
    clocks = clk.stop()
    total_ms = max_over_ranks(t0.elapsed_time(t1), ws)
    ms_step = total_ms / args.steps
    phase = [statistics.median(e[i].elapsed_time(e[i + 1]) for e in evs) for i in (0, 1, 2, 4)]
    vn_total = int(wl.vn.sum().item())

    samples_total = args.samples_per_gpu * ws
    per_rank_bytes = wl.bytes_fwd() + wl.bytes_bwd() + wl.bytes_vox(vn_total)
    job_bytes = sum_over_ranks(per_rank_bytes, ws)
    peak, peak_kind = measured_peak()
    gbs = job_bytes / (ms_step * 1e-3) / 1e9

    # roofline of the dominant kernel (one launch per step each)
    B_, D_, H_, W_ = wl.shape
    fwd_alg = wl.n * C * 4 + B_ * C * D_ * H_ * W_ * 4
    bwd_alg = wl.n * C * 4 + wl.nonempty * C * 4
    cand = {'bev_fwd_kernel': (phase[1], fwd_alg), 'bev_rows_kernel+bev_gather_kernel': (phase[2], bwd_alg)}
    kname = max(cand, key=lambda k: cand[k][0])
    kms, kbytes = cand[kname]
    achieved = kbytes / (kms * 1e-3) / 1e9
    tpp = NCU_TRAFFIC_PER_POINT.get(kname)
    roofline = {'kernel': kname, 'bound': 'hbm', 'achieved': round(achieved, 1), 'peak': peak,
                'peak_kind': peak_kind, 'unit': 'GB/s', 'frac': round(achieved / peak, 4),
                'traffic': (round(tpp * wl.n) if tpp else None), 'algorithmic_bytes': kbytes,
                'ms_per_launch': round(kms, 4)}

    line = {
        'metric': METRIC, 'value': round(ms_step / samples_total, 5), 'unit': UNIT, 'n_gpus': ws,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms_step, 4),
        'higher_is_better': False, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32',
        'data': 'synthetic (seeded stand-ins for nuScenes: 6-camera det frustum, 32-beam 10-sweep LiDAR)',
        'config': {
            'workload': (f'per GPU: det bev_pool fwd+bwd batch {args.samples_per_gpu} (config 1, 360x360, C=80, fp32, '
                         f'int64 coords) + LiDAR hard_voxelize batch {args.samples_per_gpu} (config 3 shape, '
                         f'1440x1440x40, max_points 10, max_voxels 120000)'),
            'samples_per_gpu': args.samples_per_gpu, 'global_batch': samples_total,
            'points_per_det_sample': wl.n // args.samples_per_gpu,
            'l2': 'inputs larger than L2 (det feats %.1f GB per GPU)' % (wl.feats.numel() * 4 / 1e9),
            'parallelism': f'batch-sample sharding over {ws} GPU(s), no collective on the hot path',
            'branches': ('serial: voxelisation after bev_pool on one stream' if args.serial else
                         'concurrent: voxelisation on a second stream beside bev_pool; phase times '
                         'are per stream and overlap'),
        },
        'gbs': round(gbs, 1), 'hbm_frac': round(gbs / (peak * ws), 4),
        'breakdown_ms_per_step': {'plan': round(phase[0], 4), 'bev_fwd': round(phase[1], 4),
                                  'bev_bwd': round(phase[2], 4), 'voxelize': round(phase[3], 4)},
        'roofline': roofline, 'gpu_launches': launches, 'clocks': clocks,
    }
    try:
        line['shard_check'] = shard_check(O, wl, out_last, g_last, ws, rank)
    except Exception as e:  # the parity check must not cost the benchmark line
        line['shard_check'] = {'error': repr(e)[:300]}
    if not args.no_e2e:
        line['e2e'] = run_e2e(args, wl, ws, samples_total)
    if not args.no_rulebook:
        line['sparse_rulebook'] = run_rulebook(args, wl, ws)
    if not args.no_spconv:
        try:
            line['sparse_conv'] = run_spconv(args, wl, ws)
        except Exception as e:  # an extra leg must not cost the benchmark line
            line['sparse_conv'] = {'error': repr(e)[:300]}
    if not args.no_spconv:
        try:
            line['sparse_encoder'] = run_sparse_encoder(args, wl, ws)
        except Exception as e:  # an extra leg must not cost the benchmark line
            line['sparse_encoder'] = {'error': repr(e)[:300]}
    if not args.no_triton:
        try:
            line['triton_reference'] = run_triton_reference(args, wl, ws)
        except Exception as e:  # an extra leg must not cost the benchmark line
            line['triton_reference'] = {'error': repr(e)[:300]}
    if not args.no_fused:
        del wl
        torch.cuda.empty_cache()
        line['fused_camera_branch'] = run_fused(args, rank, ws)
    if not args.no_extra:
        torch.cuda.empty_cache()
        line['other_configs'] = run_extra_configs(args, rank, ws)
    if not args.no_cpu_baseline and ws == 1 and rank == 0:
        line['cpu_baseline'] = cpu_baseline(args)
    if rank == 0:
        print(json.dumps(line), flush=True)


def sample_checksums(O, feats_out, grad, wl_vox, n1):
    """Checksum of every sample's outputs: bev_pool forward plane, the
    sample's gradient rows, and its voxel rows / coords / counts."""
    voxels, vcoors, vnum, vn = wl_vox
    res = []
    for i in range(feats_out.size(0)):
        m = int(vn[i])
        res.append(checksum(feats_out[i], grad[i * n1:(i + 1) * n1], voxels[i, :m], vcoors[i, :m], vnum[i, :m]))
    return res


def shard_check(O, wl, out, g, ws, rank):
    """Multi-GPU parity of the sharded step: every rank checksums each of its
    samples' outputs; rank 0 gathers them and recomputes the first sample of
    every other rank's shard on its own GPU from the same seeds (outside the
    timed region).  At N = 1 the checksums are reported for comparison with
    the N > 1 lines (sample i gives the same checksum on any rank)."""
    n1 = wl.n // wl.S
    mine = sample_checksums(O, out, g, (wl.voxels, wl.vcoors, wl.vnum, wl.vn.tolist()), n1)
    if ws == 1:
        return {'sample_checksums': mine, 'recomputed': 0, 'match': True}
    import torch.distributed as dist
    allc = [None] * ws
    dist.all_gather_object(allc, mine)
    res = None
    if rank == 0:
        try:
            ok = True
            for r in range(1, ws):
                one = Workload(r, 1, wl.feats.device, ws, sample_offset=r * wl.S)
                B, D, H, W = one.shape
                plan = O.bev_pool_plan(one.coords, B, D, H, W)
                o1 = O.bev_pool_forward_planned(one.feats, plan, B, D, H, W)
                g1 = O.bev_pool_backward(one.up, plan, one.n, B, D, H, W)
                O.hard_voxelize_batch(one.points, one.offs, one.voxels, one.vcoors, one.vnum, one.vn, one.vsize,
                                      one.crange, one.mp, one.mv, False)
                c1 = sample_checksums(O, o1, g1, (one.voxels, one.vcoors, one.vnum, one.vn.tolist()), one.n)[0]
                ok = ok and c1 == allc[r][0]
                del one
            res = {'sample_checksums': [c for cs in allc for c in cs], 'recomputed': ws - 1, 'match': ok}
        except Exception as e:  # report, and still meet the other ranks at the barrier
            res = {'sample_checksums': [c for cs in allc for c in cs], 'error': repr(e)[:300]}
    dist.barrier()
    return res


def run_e2e(args, wl, ws, samples_total):
    """Public API, host buffers: pinned H2D of the step's inputs, bev_pool
    forward + backward through autograd per det sample, the batched LiDAR
    voxelisation with its mean epilogue (what BEVFusion.voxelize returns:
    packed mean features, (b, x, y, z) coords and counts; one host read of
    the voxel total, at the end of the step), and D2H of every output, all
    inside the timed region.  Det samples are pipelined over three streams
    (copy in, compute, copy out), so both PCIe directions and the kernels
    overlap, also across consecutive steps; device inputs are double-buffered.

    The same copies with no kernels (same bytes, streams and ordering) give
    the host-link ceiling the end-to-end number is held against."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool
    from bevfusion_triton_b200.ops.voxel.voxel_layer import hard_voxelize_batch
    O = torch.ops.bfb_b200
    S = wl.S
    n1 = wl.n // S  # every det sample has the rig's kept points
    B, D, H, W = wl.shape
    feats_h = wl.feats.cpu().pin_memory()
    coords_h = wl.coords.cpu()
    coords_h[:, 3] = 0  # per-sample coordinates (batch column 0)
    coords_h = coords_h.pin_memory()
    up_h = wl.up.cpu().pin_memory()
    pts_h = wl.points_cpu.pin_memory()
    out_h = torch.empty(wl.up.shape, dtype=torch.float32).pin_memory()
    grad_h = torch.empty(wl.feats.shape, dtype=torch.float32).pin_memory()
    dev = torch.device('cuda', torch.cuda.current_device())
    clouds_d = torch.empty(pts_h.shape, device=dev)
    M = int(wl.vn.sum())  # voxels of the step (deterministic)
    F = pts_h.size(1)
    vf_h = torch.empty((M, F), dtype=torch.float32).pin_memory()
    vc_h = torch.empty((M, 4), dtype=torch.int32).pin_memory()
    vs_h = torch.empty((M,), dtype=torch.int32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (feats_h, coords_h, up_h, pts_h))
    d2h = sum(t.numel() * t.element_size() for t in (out_h, grad_h, vf_h, vc_h, vs_h))
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    slots = [dict(feats=torch.empty((n1, C), device=dev), coords=torch.empty((n1, 4), dtype=torch.int64, device=dev),
                  up=torch.empty((1, C, D, H, W), device=dev)) for _ in range(2)]
    free = [torch.cuda.Event(), torch.cuda.Event()]  # compute finished reading slot
    outs = dict(out=torch.empty((1, C, D, H, W), device=dev), grad=torch.empty((n1, C), device=dev),
                vf=torch.empty((M, F), device=dev), vc=torch.empty((M, 4), dtype=torch.int32, device=dev),
                vs=torch.empty((M,), dtype=torch.int32, device=dev))
    got = {}
    lid = {}

    def lidar_start(compute: bool):
        """H2D of the step's clouds and the batched voxelisation + mean
        epilogue (BEVFusion.voxelize), all asynchronous."""
        with torch.cuda.stream(s_in):
            clouds_d.copy_(pts_h, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ready)
            if compute:
                v, c, n, vn = hard_voxelize_batch(clouds_d, wl.offs, wl.vsize, wl.crange, wl.mp, wl.mv)
                lid['res'] = O.voxelize_mean_epilogue(v, c, n, vn)
            lid['done'] = torch.cuda.Event()
            lid['done'].record(s_cmp)

    def lidar_finish(compute: bool):
        """The one host read (the voxel total), then D2H of the packed rows."""
        if compute:
            vf, vc, vs, total = lid['res']
            got['M'] = m = int(total.item())
            vf, vc, vs = vf[:m], vc[:m], vs[:m]
            for t in (vf, vc, vs):
                t.record_stream(s_out)
        else:
            vf, vc, vs = outs['vf'], outs['vc'], outs['vs']
        with torch.cuda.stream(s_out):
            s_out.wait_event(lid['done'])
            vf_h.copy_(vf, non_blocking=True)
            vc_h.copy_(vc, non_blocking=True)
            vs_h.copy_(vs, non_blocking=True)

    def step(compute=True):
        # no wait on the previous step here: its D2H drains while this step's
        # H2D starts (slot reuse is ordered by the `free` events)
        main = torch.cuda.current_stream()
        lidar_start(compute)
        for s in range(S):
            k = s % 2
            sl = slots[k]
            with torch.cuda.stream(s_in):
                s_in.wait_event(free[k])
                sl['feats'].copy_(feats_h[s * n1:(s + 1) * n1], non_blocking=True)
                sl['coords'].copy_(coords_h[s * n1:(s + 1) * n1], non_blocking=True)
                sl['up'].copy_(up_h[s:s + 1], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(s_in)
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ready)
                if compute:
                    x = sl['feats'].detach().requires_grad_(True)
                    out = bev_pool(x, sl['coords'], 1, D, H, W)
                    out.backward(sl['up'])
                    out, grad = out.detach(), x.grad
                else:
                    out, grad = outs['out'], outs['grad']
                free[k].record(s_cmp)
                done = torch.cuda.Event()
                done.record(s_cmp)
                for t in (out, grad):
                    t.record_stream(s_out)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                out_h[s:s + 1].copy_(out, non_blocking=True)
                grad_h[s * n1:(s + 1) * n1].copy_(grad, non_blocking=True)
        lidar_finish(compute)
        main.wait_stream(s_out)
        main.wait_stream(s_cmp)

    def timed(compute):
        steps = max(2, min(args.steps, args.e2e_steps))
        for _ in range(2):
            step(compute)
        torch.cuda.synchronize()
        barrier(ws)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step(compute)
        e.record()
        torch.cuda.synchronize()
        barrier(ws)
        return max_over_ranks(s.elapsed_time(e), ws) / steps, steps

    ms, steps = timed(True)
    ok = got.get('M') == M  # the pipelined step returns what the batched device step computed
    copy_ms, _ = timed(False)
    agg = lambda b, t: round(sum_over_ranks(b, ws) / (t * 1e-3) / 1e9, 1)  # noqa: E731
    return {'value': round(ms / samples_total, 4), 'unit': UNIT, 'h2d_bytes_per_step': h2d,
            'd2h_bytes_per_step': d2h, 'steps': steps, 'ms_per_step': round(ms, 3),
            'pipeline': 'per det sample over 3 streams (H2D / compute / D2H), consecutive steps overlap; '
                        'LiDAR batch voxelised at once with the mean epilogue, packed rows copied back',
            'voxel_count_matches_device_step': ok,
            'copy_ceiling': {'ms_per_step': round(copy_ms, 3), 'value': round(copy_ms / samples_total, 4),
                             'unit': UNIT, 'h2d_gbs_all_ranks': agg(h2d, copy_ms),
                             'd2h_gbs_all_ranks': agg(d2h, copy_ms),
                             'note': 'same pinned copies, streams and ordering, no kernels'},
            'frac_of_copy_ceiling': round(copy_ms / ms, 4)}


def run_triton_reference(args, wl, ws):
    """The reference's own Triton GPU path (installed unmodified under
    baseline/_ref) on the rank's device-resident workload, beside this
    library through the same public calls: bev_pool forward + backward
    through autograd over the det batch, and hard_voxelize sample by sample
    (the reference API takes one cloud per call).  CUDA events, same warm-up
    rule; ms per sample."""
    sys.path.insert(0, str(ROOT / 'baseline'))
    import ref_triton
    why = ref_triton.available()
    if why:
        return {'unavailable': why}
    rbev, rvox, _ = ref_triton.load()
    from bevfusion_triton_b200.ops.bev_pool import bev_pool
    from bevfusion_triton_b200.ops.voxel.voxel_layer import hard_voxelize
    B, D, H, W = wl.shape
    S = wl.S
    F = wl.points.size(1)
    clouds = [wl.points[a:b] for a, b in zip(wl.offs, wl.offs[1:])]
    vox = torch.empty((wl.mv, wl.mp, F), device=wl.points.device)
    vco = torch.empty((wl.mv, 3), dtype=torch.int32, device=wl.points.device)
    vnm = torch.empty((wl.mv,), dtype=torch.int32, device=wl.points.device)

    def bev(fn):
        def run():
            x = wl.feats.detach().requires_grad_(True)
            fn(x, wl.coords, B, D, H, W).backward(wl.up)
        return run

    def voxelize(fn):
        def run():
            for c in clouds:
                fn(c, vox, vco, vnm, wl.vsize, wl.crange, wl.mp, wl.mv, 3, True)
        return run

    def timed(fn, k):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(ws)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(k):
            fn()
        s1.record()
        torch.cuda.synchronize()
        barrier(ws)
        return max_over_ranks(s0.elapsed_time(s1), ws) / k / S

    k = max(3, min(args.steps, 10))
    res = {}
    for name, pair in (('bev_pool_fwd_bwd', (bev(bev_pool), bev(rbev.bev_pool))),
                       ('hard_voxelize', (voxelize(hard_voxelize), voxelize(rvox.hard_voxelize)))):
        ours, ref = timed(pair[0], k), timed(pair[1], k)
        res[name] = {'ours_ms_per_sample': round(ours, 4), 'triton_ms_per_sample': round(ref, 4),
                     'speedup': round(ref / ours, 2)}
    res['note'] = ('reference Triton kernels (bev_pool_triton.py, voxelization_triton.py, unmodified) vs this '
                   'library, both through their public Python calls on the same device-resident inputs; '
                   'bev_pool over the det batch with autograd, hard_voxelize one cloud per call (deterministic)')
    return res


def run_extra_configs(args, rank, ws):
    """The other bev_pool configurations of BASELINE.json, device-resident,
    plan + forward + backward per step (CUDA events, same warm-up rule):
    config 4 (segmentation grid 256 x 256, batch 4, fp32) and config 2's
    fp16-feature variant (det grid, batch 8, fp16 features and gradients)."""
    O = torch.ops.bfb_b200
    peak, _ = measured_peak()
    res = {}
    for name, mk, S, dt in (('seg_batch4_fp32', synth.seg_bev_pool_case, 4, torch.float32),
                            ('det_batch8_fp16', synth.det_bev_pool_case, 8, torch.float16)):
        first, _ = shard.shard_samples(S * ws, ws, rank)
        case = mk(S, device='cuda', sample_offset=first, dtype=dt)
        B, D, H, W = case.B, case.D, case.H, case.W
        up = torch.cat([upstream_grad(first + i, case, 'cuda') for i in range(S)]).to(dt)
        n = case.feats.size(0)
        es = torch.empty((), dtype=dt).element_size()
        dhw = D * H * W
        r = case.coords[:, 3] * dhw + (case.coords[:, 2] * H + case.coords[:, 0]) * W + case.coords[:, 1]
        U = int(torch.unique(r).numel())
        alg = (n * C * es + n * 32 + B * C * dhw * es) + (n * C * es + n * 32 + U * C * es)

        def step():
            plan = O.bev_pool_plan(case.coords, B, D, H, W)
            O.bev_pool_forward_planned(case.feats, plan, B, D, H, W)
            O.bev_pool_backward(up, plan, n, B, D, H, W)

        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        barrier(ws)
        k = max(3, min(args.steps, 20))
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(k):
            step()
        s1.record()
        torch.cuda.synchronize()
        barrier(ws)
        ms = max_over_ranks(s0.elapsed_time(s1), ws) / k
        res[name] = {'ms_per_sample': round(ms / (S * ws), 5), 'ms_per_step': round(ms, 4), 'samples_per_gpu': S,
                     'points_per_sample': n // S, 'gbs_per_gpu': round(alg / (ms * 1e-3) / 1e9, 1),
                     'hbm_frac': round(alg / (ms * 1e-3) / 1e9 / peak, 4)}
        del case, up
        torch.cuda.empty_cache()
    res['note'] = ('plan + forward + backward of bev_pool per step, inputs resident in HBM; bytes are the '
                   'path-level algorithmic bytes (feats, int64 coords, output, gradient rows)')
    return res


def lidar_sites(wl):
    """(b, x, y, z) int32 rows of the rank's voxelised LiDAR samples."""
    vn = wl.vn.tolist()
    return torch.cat([torch.cat((torch.full((int(vn[b]), 1), b, dtype=torch.int32, device=wl.vcoors.device),
                                 wl.vcoors[b, :int(vn[b])]), 1) for b in range(wl.S)]).contiguous()


SPCONV_LAYERS = [
    # name, rulebook, cin, cout, dtype
    ('subm_k3_16x16_f16', 'subm', 16, 16, torch.float16),
    ('subm_k3_64x64_f16', 'subm', 64, 64, torch.float16),
    ('subm_k3_64x64_bf16', 'subm', 64, 64, torch.bfloat16),
    ('subm_k3_64x64_f32', 'subm', 64, 64, torch.float32),
    ('down_k3_s2_32x64_f16', 'down', 32, 64, torch.float16),
]


def run_spconv(args, wl, ws):
    """Sparse convolution over the rank's voxelised LiDAR samples (the sparse
    encoder's submanifold and strided 3x3x3 layers at full resolution),
    device-resident, forward and backward (input + filter gradients), ours
    beside the reference's own GPU path (Triton gather, one matmul per rule,
    Triton atomic scatter; installed unmodified under baseline/_ref).  ms per
    call of all S samples, max over ranks; useful TFLOP/s = 2 * pairs * Cin *
    Cout per pass (forward; the backward does twice that)."""
    from bevfusion_triton_b200.ops.spconv import get_indice_pairs, indice_conv, indice_conv_backward
    sys.path.insert(0, str(ROOT / 'baseline'))
    import ref_triton
    try:
        rsc = ref_triton.load_spconv()
    except Exception as e:  # the reference copy is optional for this leg
        rsc, why = None, str(e)
    idx = lidar_sites(wl)
    shape = [1440, 1440, 41]
    books = {'subm': get_indice_pairs(idx, wl.S, shape, ksize=3, padding=1, subm=True),
             'down': get_indice_pairs(idx, wl.S, shape, ksize=3, stride=2, padding=1)}
    g = torch.Generator(device='cuda').manual_seed(7)
    k = max(3, min(args.steps, 10))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(ws)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(k):
            fn()
        s1.record()
        torch.cuda.synchronize()
        barrier(ws)
        return max_over_ranks(s0.elapsed_time(s1), ws) / k

    res = {'sites': int(idx.size(0)), 'reference': 'triton (baseline/_ref)' if rsc else f'unavailable: {why}'}
    for name, book, cin, cout, dt in SPCONV_LAYERS:
        outids, pairs, num = books[book]
        n_in, n_out = idx.size(0), outids.size(0)
        x = torch.randn(n_in, cin, device='cuda', generator=g).to(dt)
        w = (torch.randn(27, cin, cout, device='cuda', generator=g) / (27 * cin) ** 0.5).to(dt)
        gy = torch.randn(n_out, cout, device='cuda', generator=g).to(dt)
        npairs = int(num.sum())
        flop = 2.0 * npairs * cin * cout
        fwd = timed(lambda: indice_conv(x, w, pairs, num, n_out))
        bwd = timed(lambda: indice_conv_backward(x, w, gy, pairs, num))
        r = {'pairs': npairs, 'out_sites': n_out, 'fwd_ms': round(fwd, 4), 'bwd_ms': round(bwd, 4),
             'fwd_tflops': round(flop / fwd / 1e9, 2), 'bwd_tflops': round(2 * flop / bwd / 1e9, 2)}
        if rsc is not None:
            rf = timed(lambda: rsc.indice_conv(x, w, pairs, num, n_out))
            rb = timed(lambda: rsc.indice_conv_backward(x, w, gy, pairs, num))
            y, yr = indice_conv(x, w, pairs, num, n_out).float(), rsc.indice_conv(x, w, pairs, num, n_out).float()
            r.update({'ref_fwd_ms': round(rf, 4), 'ref_bwd_ms': round(rb, 4),
                      'fwd_speedup': round(rf / fwd, 2), 'bwd_speedup': round(rb / bwd, 2),
                      'max_rel_diff_vs_ref': float(((y - yr).abs() / yr.abs().clamp(min=1.0)).max())})
        res[name] = r
    return res


def run_sparse_encoder(args, wl, ws):
    """A LiDAR sparse-encoder stack shaped like BEVFusion's SparseEncoder
    default configuration (models/backbones/sparse_encoder.py: 5 -> 16 input
    conv, stages of channels (16, 16, 32), (32, 32, 64), (64, 64, 128),
    (128, 128) with residual submanifold blocks and strided 3x3x3 downsampling,
    the (1, 1, 3) output conv to 128 channels, batch norm + ReLU after each
    conv), built from this library's module layer, over the rank's voxelised
    LiDAR samples (mean voxel features), fp32 and under fp16 autocast.  The
    same stack composed from the reference's own GPU functions
    (spconv_triton, installed unmodified) is timed for the forward.  ms per
    call of all S samples, max over ranks."""
    from torch import nn
    from bevfusion_triton_b200.ops import spconv as S
    sys.path.insert(0, str(ROOT / 'baseline'))
    import ref_triton
    try:
        rsc = ref_triton.load_spconv()
    except Exception:
        rsc = None
    # the voxelisation's packed mean features and (b, x, y, z) sites
    vf, vc, _, total = torch.ops.bfb_b200.voxelize_mean_epilogue(wl.voxels, wl.vcoors, wl.vnum, wl.vn)
    m = int(total.item())
    feats, idx = vf[:m].contiguous(), vc[:m].contiguous()
    shape = [1440, 1440, 41]

    class Block(S.SparseModule):  # residual block of two submanifold convs
        def __init__(self, c, key):
            super().__init__()
            self.c1, self.b1 = S.SubMConv3d(c, c, 3, padding=1, bias=False, indice_key=key), nn.BatchNorm1d(c, 1e-3)
            self.c2, self.b2 = S.SubMConv3d(c, c, 3, padding=1, bias=False, indice_key=key), nn.BatchNorm1d(c, 1e-3)

        def forward(self, x):
            y = self.c1(x)
            y.features = torch.relu(self.b1(y.features))
            y = self.c2(y)
            y.features = torch.relu(self.b2(y.features) + x.features)
            return y

    def cbr(conv, c):
        return [conv, nn.BatchNorm1d(c, eps=1e-3), nn.ReLU()]

    torch.manual_seed(0)
    layers = cbr(S.SubMConv3d(5, 16, 3, padding=1, bias=False, indice_key='subm1'), 16)
    chans = ((16, 16, 32), (32, 32, 64), (64, 64, 128), (128, 128))
    pads = ((0, 0, 1), (0, 0, 1), (0, 0, (1, 1, 0)), (0, 0))
    cin = 16
    for i, blocks in enumerate(chans):
        for j, c in enumerate(blocks):
            if j == len(blocks) - 1 and i != len(chans) - 1:
                layers += cbr(S.SparseConv3d(cin, c, 3, stride=2, padding=pads[i][j], bias=False,
                                             indice_key=f'spconv{i + 1}'), c)
            else:
                layers.append(Block(c, f'subm{i + 1}'))
            cin = c
    layers += cbr(S.SparseConv3d(128, 128, (1, 1, 3), stride=(1, 1, 2), padding=0, bias=False,
                                 indice_key='spconv_down2'), 128)
    net = S.SparseSequential(*layers).cuda()

    def ours(autocast, backward):
        x = feats.detach().requires_grad_(backward)
        with torch.autocast('cuda', dtype=torch.float16, enabled=autocast):
            out = net(S.SparseConvTensor(x, idx, shape, wl.S))
        if backward:
            out.features.float().sum().backward()
        return out

    def ref_forward():
        """The stack's calls, composed from the reference's functions."""
        f, ind, shp, cache = feats, idx, shape, {}

        def conv(m, f, ind, shp):
            if m.indice_key in cache:
                outids, _, pairs, num, _ = cache[m.indice_key]
                oshp = shp
            else:
                outids, pairs, num = rsc.get_indice_pairs(ind, wl.S, shp, m.kernel_size, m.stride, m.padding,
                                                          m.dilation, m.output_padding, m.subm, m.transposed)
                cache[m.indice_key] = (outids, ind, pairs, num, shp)
                oshp = shp if m.subm else S.get_conv_output_size(shp, m.kernel_size, m.stride, m.padding, m.dilation)
            return rsc.indice_conv(f, m.weight, pairs, num, outids.shape[0], False, m.subm), outids, oshp

        with torch.no_grad():
            for m in net:
                if isinstance(m, Block):
                    y, _, _ = conv(m.c1, f, ind, shp)
                    y = torch.relu(m.b1(y))
                    y, _, _ = conv(m.c2, y, ind, shp)
                    f = torch.relu(m.b2(y) + f)
                elif isinstance(m, S.SparseConvolution):
                    f, ind, shp = conv(m, f, ind, shp)
                else:
                    f = m(f)
        return f

    def timed(fn, k=max(3, min(args.steps, 10)), warm=2):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        barrier(ws)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(k):
            fn()
        s1.record()
        torch.cuda.synchronize()
        barrier(ws)
        return round(max_over_ranks(s0.elapsed_time(s1), ws) / k, 3)

    net.eval()
    res = {'sites': int(idx.size(0)), 'layers': sum(isinstance(m, S.SparseConvolution) for m in net.modules()),
           'fwd_fp32_ms': timed(lambda: ours(False, False)), 'fwd_fp16_autocast_ms': timed(lambda: ours(True, False))}
    net.train()
    res['fwd_bwd_fp32_ms'] = timed(lambda: ours(False, True))
    res['fwd_bwd_fp16_autocast_ms'] = timed(lambda: ours(True, True))
    net.eval()
    if rsc is not None:
        res['reference_fwd_fp32_ms'] = timed(ref_forward, k=3, warm=1)  # seconds per call: 3 are plenty
        with torch.no_grad():
            a, b = ours(False, False).features, ref_forward()
        res['fwd_fp32_speedup'] = round(res['reference_fwd_fp32_ms'] / res['fwd_fp32_ms'], 2)
        res['max_abs_diff_vs_reference'] = float((a - b).abs().max())
    return res


def run_rulebook(args, wl, ws):
    """Sparse-convolution rulebooks of the sparse encoder's layer kinds over
    the rank's voxelised LiDAR samples (the voxel sites of the step above,
    (b, x, y, z) on the (1440, 1440, 41) sparse shape), device-resident: ms
    per get_indice_pairs call, including its one host read of the output
    count as in the reference."""
    from bevfusion_triton_b200.ops.spconv import get_indice_pairs
    S = wl.S
    idx = lidar_sites(wl)
    shape = [1440, 1440, 41]
    layers = {'subm_k3': dict(ksize=3, stride=1, padding=1, subm=True),
              'down_k3_s2': dict(ksize=3, stride=2, padding=1),
              'out_k113_s112': dict(ksize=(1, 1, 3), stride=(1, 1, 2), padding=0)}
    res = {'sites': int(idx.size(0)), 'sparse_shape': shape}
    for name, kw in layers.items():
        for _ in range(3):
            get_indice_pairs(idx, S, shape, **kw)
        torch.cuda.synchronize()
        barrier(ws)
        k = max(3, min(args.steps, 20))
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(k):
            o, pr, nm = get_indice_pairs(idx, S, shape, **kw)
        s1.record()
        torch.cuda.synchronize()
        res[name] = {'ms_per_call': round(max_over_ranks(s0.elapsed_time(s1), ws) / k, 4),
                     'out_sites': int(o.size(0)), 'pairs': int(nm.sum())}
    return res


def run_fused(args, rank, ws):
    """The camera branch from depth distribution and context to BEV (fwd+bwd)
    over the rank's det samples: unfused (depth x context product, flatten,
    in-grid filter, bev_pool, as models/vtransforms/depth_lss.py + base.py do)
    vs the fused op that never materialises the feature tensor; and both
    again starting from the camera parameters (geometry + quantise + filter
    in torch, against the geometry plan)."""
    from bevfusion_triton_b200.ops.bev_pool import bev_pool, bev_pool_depth_context, bev_pool_geometry_plan
    S = args.samples_per_gpu
    first, _ = shard.shard_samples(S * ws, ws, rank)
    case = synth.depth_context_case(S, synth.DET_GRID, device='cuda', sample_offset=first)
    shape = (case.B, case.D, case.H, case.W)
    up = torch.randn((case.B, C, case.D, case.H, case.W), device='cuda')
    kidx = torch.nonzero(case.kept).squeeze(1)
    kcoords = case.coords[kidx]

    def unfused():
        d = case.depth.detach().requires_grad_(True)
        c = case.context.detach().requires_grad_(True)
        x = (d.unsqueeze(2) * c.unsqueeze(3)).permute(0, 1, 3, 4, 5, 2).reshape(-1, C)
        bev_pool(x[kidx], kcoords, *shape).backward(up)

    def fused():
        d = case.depth.detach().requires_grad_(True)
        c = case.context.detach().requires_grad_(True)
        bev_pool_depth_context(d, c, case.coords, *shape).backward(up)

    # the same branch from the camera parameters: the reference geometry,
    # quantise and filter in torch, then the unfused pooling; against the
    # geometry plan feeding the fused pooling (no coordinate tensor at all)
    rig = synth.camera_rig(S, augment=True, seed=first, device='cuda')
    bounds = {k: synth.DET_GRID[k] for k in ('xbound', 'ybound', 'zbound')}

    def unfused_camera():
        coords, kept, shp = synth.lss_coords(synth.lss_geometry(**rig), **bounds)
        kidx = torch.nonzero(kept).squeeze(1)
        d = case.depth.detach().requires_grad_(True)
        c = case.context.detach().requires_grad_(True)
        x = (d.unsqueeze(2) * c.unsqueeze(3)).permute(0, 1, 3, 4, 5, 2).reshape(-1, C)
        bev_pool(x[kidx], coords[kidx], *shp).backward(up)

    def fused_camera():
        plan, shp = bev_pool_geometry_plan(**rig, **bounds)
        d = case.depth.detach().requires_grad_(True)
        c = case.context.detach().requires_grad_(True)
        bev_pool_depth_context(d, c, None, *shp, plan=plan).backward(up)

    res = {}
    for name, fn in (('unfused', unfused), ('fused', fused), ('unfused_from_camera', unfused_camera),
                     ('fused_from_camera', fused_camera)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(ws)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k = max(3, min(args.steps, 10))
        s0.record()
        for _ in range(k):
            fn()
        s1.record()
        torch.cuda.synchronize()
        barrier(ws)
        res[name + '_ms_per_sample'] = round(max_over_ranks(s0.elapsed_time(s1), ws) / k / S, 4)
    res['speedup'] = round(res['unfused_ms_per_sample'] / res['fused_ms_per_sample'], 2)
    res['speedup_from_camera'] = round(res['unfused_from_camera_ms_per_sample'] / res['fused_from_camera_ms_per_sample'], 2)
    res['note'] = ('det grid, softmax depth (118 bins) x context (C=80), fp32, forward + backward; *_from_camera '
                   'also computes the frustum geometry, quantisation and filter from the camera parameters '
                   '(augmented rig)')
    return res


# ------------------------------------------------------------------ CPU
def cpu_reference_sample(threads: int, det=None, clouds=None):
    """One bounded sample of the reference's CPU algorithms: det bev_pool
    fwd+bwd of one camera sample (torch CPU, `threads` threads) and hard
    voxelisation of `threads` LiDAR samples in parallel.  Returns
    (ms per sample, description)."""
    from oracle import ref_cpu
    torch.set_num_threads(threads)
    if det is None:
        det = synth.det_bev_pool_case(1, device='cpu')
        g = torch.Generator().manual_seed(5)
        det.up = torch.randn((1, C, det.D, det.H, det.W), generator=g)
    if clouds is None:
        clouds = [synth.lidar_sweeps(i) for i in range(threads)]
    t = time.perf_counter()
    ref_cpu.bev_pool_fwd_bwd_cpu(det.feats, det.coords, det.B, det.D, det.H, det.W, det.up)
    t_bev = time.perf_counter() - t
    t = time.perf_counter()
    ref_cpu.hard_voxelize_many(clouds, list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE),
                               synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS, threads=threads)
    t_vox = (time.perf_counter() - t) / len(clouds)
    return (t_bev + t_vox) * 1e3, det, clouds, t_bev * 1e3, t_vox * 1e3


def cpu_baseline(args):
    threads = os.cpu_count() or 1
    cpu_reference_sample(threads)  # warm
    ms, det, clouds, tb, tv = cpu_reference_sample(threads)
    return {'value': round(ms, 2), 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': (f'1 det sample bev_pool fwd+bwd via torch CPU index_add_ ({tb:.1f} ms, {threads} threads) + '
                       f'{len(clouds)} LiDAR samples hard_voxelize via the C restatement of the reference loop, '
                       f'one per thread ({tv:.1f} ms/sample)')}


def run_reference(args, ws, rank):
    """--impl reference: the reference's own CPU algorithms on the host cores
    (rank 0 only; other ranks exit without work)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    ms0, det, clouds, _, _ = cpu_reference_sample(threads)
    vals, tbs, tvs = [], [], []
    steps = max(1, min(args.steps, args.ref_steps))
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_reference_sample(threads, det, clouds)
    for _ in range(steps):
        ms, _, _, tb, tv = cpu_reference_sample(threads, det, clouds)
        vals.append(ms)
        tbs.append(tb)
        tvs.append(tv)
    v = statistics.median(vals)
    sample = (f'per step: 1 det sample bev_pool fwd+bwd via torch CPU index_add_ ({statistics.median(tbs):.1f} ms, '
              f'{threads} threads) + {len(clouds)} LiDAR samples hard_voxelize via the C restatement of the '
              f'reference loop, one per thread ({statistics.median(tvs):.1f} ms/sample)')
    line = {
        'metric': METRIC, 'value': round(v, 3), 'unit': UNIT, 'n_gpus': ws, 'steps': steps,
        'warmup': args.warmup, 'ms_per_step': round(v, 3), 'higher_is_better': False, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic', 'impl': 'reference',
        'config': {'workload': 'det bev_pool fwd+bwd + LiDAR hard_voxelize, one sample each, reference CPU '
                               'algorithms on the host cores', 'samples_per_gpu': args.samples_per_gpu},
        'cpu_baseline': {'value': round(v, 3), 'unit': UNIT, 'cores': threads, 'kind': 'port', 'sample': sample},
        'e2e': {'value': round(v, 3), 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=50)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--samples-per-gpu', type=int, default=SAMPLES_PER_GPU)
    ap.add_argument('--e2e-steps', type=int, default=5)
    ap.add_argument('--ref-steps', type=int, default=3)
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-fused', action='store_true')
    ap.add_argument('--no-rulebook', action='store_true')
    ap.add_argument('--no-spconv', action='store_true', help='skip the sparse-convolution timings')
    ap.add_argument('--no-triton', action='store_true', help='skip timing the reference Triton GPU path')
    ap.add_argument('--no-extra', action='store_true', help='skip the config-4 and fp16 bev_pool timings')
    ap.add_argument('--lidar-beside', choices=('plan', 'gather'), default='plan',
                    help='start the concurrent voxelisation with the plan or after it, beside the gathers')
    ap.add_argument('--lidar-priority', action='store_true', help='run the LiDAR stream at high priority')
    ap.add_argument('--serial', action='store_true', help='run the LiDAR voxelisation after the camera branch on one stream')
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == 'ours':
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    ws, rank, local = dist_setup(args)
    try:
        if args.impl == 'reference':
            run_reference(args, ws, rank)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
