"""Generates the golden fixtures in this folder from the REFERENCE implementation.

Run only where the reference checkout is available (it is not on the GPU
box; the fixtures travel instead):

    python tests/golden/make_golden.py /path/to/bevfusion-triton

The reference's CPU paths are imported read-only, without executing its
package ``__init__`` files (which would pull in unrelated ops), through stub
package modules:

* ops/bev_pool/src/bev_pool_triton.py            ``bev_pool`` (CPU path: ``_bev_pool_cpu``)
* ops/voxel/src/voxelization_triton.py           ``dynamic_voxelize``, ``hard_voxelize``
* ops/voxel/src/scatter_points_triton.py         ``dynamic_point_to_voxel_forward/backward``
* ops/spconv/src/spconv_triton.py                ``_get_indice_pairs_impl`` (rulebooks, with the
                                                 GPU path's output order: cuda_ordering=True);
                                                 ``indice_conv``, ``fused_indice_conv``,
                                                 ``indice_conv_backward``, ``indice_maxpool(_backward)``
                                                 on CPU tensors (their CPU gather / index_add_ path)
* models/vtransforms/base.py                     ``BaseTransform.get_geometry`` and the quantise +
                                                 in-grid filter of ``BaseTransform.bev_pool``
                                                 (with models/helper/amp.py ``force_fp32``)

``--only spconv`` / ``--only spconv_conv`` / ``--only geometry`` regenerate only
that fixture.

Cases mirror the reference tests (tests/test_ops/test_bev_pool.py:24-84,
tests/test_ops/test_voxel.py:27-79) plus seeded larger cases and full-size
digests of the benchmark configurations.
"""
from __future__ import annotations

import hashlib
import json
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.dont_write_bytecode = True

from tests import synth  # noqa: E402


def import_reference(ref: Path):
    for name, sub in [('ops', 'ops'), ('ops.bev_pool', 'ops/bev_pool'), ('ops.bev_pool.src', 'ops/bev_pool/src'),
                      ('ops.voxel', 'ops/voxel'), ('ops.voxel.src', 'ops/voxel/src'), ('ops.spconv', 'ops/spconv'),
                      ('ops.spconv.src', 'ops/spconv/src')]:
        m = types.ModuleType(name)
        m.__path__ = [str(ref / sub)]
        sys.modules[name] = m
    import ops.bev_pool.src.bev_pool_triton as bpt
    import ops.voxel.src.scatter_points_triton as spt
    import ops.voxel.src.voxelization_triton as vt
    return bpt, vt, spt


def import_spconv():
    import ops.spconv.src.spconv_triton as sct
    return sct


SPCONV_CASES = [
    # spatial shape, ksize, stride, padding, dilation, subm, transpose
    ([8, 8], [3, 3], [1, 1], [1, 1], [1, 1], True, False),
    ([9, 7], [3, 3], [2, 2], [1, 1], [1, 1], False, False),
    ([6, 5, 7], [3, 3, 3], [2, 2, 2], [0, 1, 1], [1, 1, 1], False, False),
    ([6, 5, 7], [1, 1, 3], [1, 1, 2], [0, 0, 0], [1, 1, 1], False, False),
    ([6, 5, 7], [3, 3, 3], [1, 1, 1], [1, 1, 1], [1, 1, 1], True, False),
    ([5, 6], [3, 3], [2, 2], [1, 1], [1, 1], False, True),
    ([8, 9], [3, 3], [1, 1], [2, 2], [2, 2], False, False),
    ([4, 3, 3, 5], [3, 1, 3, 2], [1, 1, 1, 1], [1, 0, 1, 0], [1, 1, 1, 1], False, False),
    ([20, 20, 6], [3, 3, 3], [2, 2, 2], [1, 1, 1], [1, 1, 1], False, False),
]


def import_base_transform(ref: Path):
    """models/vtransforms/base.py with stub ``models`` / ``models.helper``
    packages (only helper/amp.py is executed) and ``ops.bev_pool`` bound to
    the reference bev_pool module (CPU path)."""
    import importlib.util
    for name, sub in [('models', 'models'), ('models.helper', 'models/helper'),
                      ('models.vtransforms', 'models/vtransforms')]:
        m = types.ModuleType(name)
        m.__path__ = [str(ref / sub)]
        sys.modules[name] = m
    spec = importlib.util.spec_from_file_location('models.helper.amp', ref / 'models/helper/amp.py')
    amp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(amp)
    sys.modules['models.helper'].force_fp32 = amp.force_fp32
    import ops.bev_pool.src.bev_pool_triton as bpt
    sys.modules['ops.bev_pool'].bev_pool = bpt.bev_pool
    import models.vtransforms.base as base
    return base


EDGE = 1e-4  # cells: a point this close to a cell edge may round either way


def geometry_cases(base):
    """Per frustum point, the cell rank ((b*D + z)*H + x)*W + y the reference
    gives it (get_geometry, then the trunc quantise and in-grid filter of
    BaseTransform.bev_pool, base.py:82-158), -1 when filtered out.  The
    points whose quantiser input lies within EDGE cells of an integer are
    listed with their reference cells (the GPU producer's fp32 association
    may round them either way); all other points are pinned by a digest of
    the cell array with the listed points set to -2."""
    out, dig = {}, {}
    cases = [('det_plain', synth.DET_GRID, 1, False), ('det_aug', synth.DET_GRID, 2, True),
             ('seg_plain', synth.SEG_GRID, 1, False), ('seg_aug', synth.SEG_GRID, 1, True)]
    for name, grid, batch, augment in cases:
        rig = synth.camera_rig(batch, augment=augment, seed=5)
        bt = base.BaseTransform(80, 80, synth.IMAGE_SIZE, synth.FEATURE_SIZE, grid['xbound'], grid['ybound'],
                                grid['zbound'], synth.DBOUND)
        bt.frustum.data.copy_(rig['frustum'])
        extra = {k: rig[k] for k in ('extra_rots', 'extra_trans') if k in rig}
        geom = bt.get_geometry(rig['camera2lidar_rots'], rig['camera2lidar_trans'], rig['intrins'],
                               rig['post_rots'], rig['post_trans'], **extra)
        B, N, D, H, W, _ = geom.shape
        n = B * N * D * H * W
        captured = {}

        def capture(x, g, b_, d_, h_, w_):
            captured['idx'] = x[:, 0].long()
            captured['coords'] = g.clone()
            captured['grid'] = (b_, int(d_), int(h_), int(w_))
            return torch.zeros((b_, x.size(1), int(d_), int(h_), int(w_)))

        saved = base.bev_pool
        base.bev_pool = capture
        try:  # the point index rides through the filter as the one feature channel
            x = torch.arange(n, dtype=torch.float32).view(B, N, D, H, W, 1)
            bt.bev_pool(geom, x)
        finally:
            base.bev_pool = saved
        Bg, Dg, Hg, Wg = captured['grid']
        c = captured['coords']
        cells = torch.full((n,), -1, dtype=torch.int64)
        cells[captured['idx']] = ((c[:, 3] * Dg + c[:, 2]) * Hg + c[:, 0]) * Wg + c[:, 1]
        q = (geom - (bt.bx - bt.dx / 2.0)) / bt.dx  # the quantiser input, as base.py:139 forms it
        q = q.reshape(-1, 3).double()
        near = torch.nonzero(((q - q.round()).abs() < EDGE).any(1)).squeeze(1)
        masked = cells.clone()
        masked[near] = -2
        out[f'{name}_near_idx'] = near.numpy().astype(np.int32)
        out[f'{name}_near_cells'] = cells[near].numpy()
        out[f'{name}_grid'] = np.array([Bg, Dg, Hg, Wg], dtype=np.int64)
        dig[f'geometry_{name}_masked_cells'] = sha(masked.numpy())
        dig[f'geometry_{name}_kept'] = int((cells >= 0).sum())
    save('geometry_cells', **out)
    return dig


def spconv_cases(sct):
    """Rulebooks of small sparse tensors (2 samples, unique random sites),
    tests/test_ops/test_spconv/test_spconv_ops.py shapes and the sparse
    encoder's layer kinds (submanifold 3x3x3, strided 3x3x3, (1, 1, 3)
    stride (1, 1, 2))."""
    g = torch.Generator().manual_seed(11)
    out = {}
    for i, (shape, k, st, pd, dl, subm, tr) in enumerate(SPCONV_CASES):
        B = 2
        n = min(60, B * int(np.prod(shape)) // 3)
        cells = torch.randperm(B * int(np.prod(shape)), generator=g)[:n]
        f, cols = cells.clone(), []
        for d in reversed(shape):
            cols.append(f % d)
            f //= d
        idx = torch.stack([f] + cols[::-1], 1).int()
        _, ks, ss, ps, ds, _, outs = sct._prepare_indice_pair_args(idx, B, shape, ksize=k, stride=st, padding=pd,
                                                                   dilation=dl, subm=subm, transpose=tr)
        o, pr, nm = sct._get_indice_pairs_impl(idx, B, outs, ks, ss, ps, ds, subm=subm, transpose=tr,
                                               cuda_ordering=True, grid=None)
        out.update({f'c{i}_indices': idx, f'c{i}_cfg': np.array(shape + k + st + pd + dl + [int(subm), int(tr), B]),
                    f'c{i}_outshape': np.array(outs), f'c{i}_outids': o, f'c{i}_pairs': pr, f'c{i}_num': nm})
    save('spconv_cases', **out)


SPCONV_CONV_CASES = [
    # rulebook case of SPCONV_CASES, cin, cout, inverse
    (4, 16, 32, False),   # submanifold 3x3x3
    (2, 16, 16, False),   # strided 3x3x3
    (8, 5, 16, False),    # strided, odd input channels (the encoder's first layer width)
    (5, 32, 16, False),   # transposed
    (2, 16, 16, True),    # strided rulebook used inverse (SparseInverseConv3d)
]


def spconv_conv_cases(sct):
    """Sparse convolution, its backward and sparse max-pooling run by the
    reference on CPU tensors over the rulebooks of ``spconv_cases`` (read back
    from spconv_cases.npz), seeded fp32 features / filters / gradients."""
    rb = np.load(HERE / 'spconv_cases.npz')
    g = torch.Generator().manual_seed(23)
    out = {}
    for j, (c, cin, cout, inverse) in enumerate(SPCONV_CONV_CASES):
        pairs = torch.from_numpy(rb[f'c{c}_pairs'])
        num = torch.from_numpy(rb[f'c{c}_num'])
        n_idx = rb[f'c{c}_indices'].shape[0]
        n_out_ids = rb[f'c{c}_outids'].shape[0]
        n_in, n_out = (n_out_ids, n_idx) if inverse else (n_idx, n_out_ids)
        K = pairs.shape[0]
        x = torch.randn(n_in, cin, generator=g)
        w = torch.randn(K, cin, cout, generator=g) * 0.2
        bias = torch.randn(cout, generator=g)
        gy = torch.randn(n_out, cout, generator=g)
        y = sct.indice_conv(x, w, pairs, num, n_out, inverse=inverse)
        yb = sct.fused_indice_conv(x, w, bias, pairs, num, n_out, inverse, False)
        gx, gw = sct.indice_conv_backward(x, w, gy, pairs, num, inverse=inverse)
        out.update({f'v{j}_case': np.array([c, cin, cout, int(inverse), n_in, n_out]), f'v{j}_x': x, f'v{j}_w': w,
                    f'v{j}_bias': bias, f'v{j}_gy': gy, f'v{j}_y': y, f'v{j}_yb': yb, f'v{j}_gx': gx, f'v{j}_gw': gw})
        if not inverse:
            xp = torch.randn(n_in, cin, generator=g)
            xp[:, 0] = -xp[:, 0].abs()  # an all-negative channel: pooled into zeros
            yp = sct.indice_maxpool(xp, pairs, num, n_out)
            gyp = torch.randn(n_out, cin, generator=g)
            gxp = sct.indice_maxpool_backward(xp, yp, gyp, pairs, num)
            out.update({f'v{j}_xp': xp, f'v{j}_yp': yp, f'v{j}_gyp': gyp, f'v{j}_gxp': gxp})
    save('spconv_conv_cases', **out)


def sha(a) -> str:
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.tobytes()).hexdigest()


def save(name, **arrays):
    np.savez_compressed(HERE / f'{name}.npz', **{k: np.asarray(v) for k, v in arrays.items()})


def bev_cases(bpt):
    # known-answer case, tests/test_ops/test_bev_pool.py:57-84
    feats = torch.tensor([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]])
    coords = torch.tensor([[0, 0, 0, 0], [0, 0, 0, 0], [1, 0, 0, 0]], dtype=torch.int32)
    out = bpt.bev_pool(feats, coords, 1, 1, 2, 1)
    save('bev_known', feats=feats, coords=coords, shape=[1, 1, 2, 1], out=out)

    def rand_case(name, n, c, B, D, H, W, seed, cdtype, fdtype, hot=None):
        g = torch.Generator().manual_seed(seed)
        feats = torch.randn((n, c), generator=g).to(fdtype)
        coords = torch.stack([
            torch.randint(0, H, (n,), generator=g), torch.randint(0, W, (n,), generator=g),
            torch.randint(0, D, (n,), generator=g), torch.randint(0, B, (n,), generator=g)], 1)
        if hot is not None:  # pile `hot` points into a few cells (long segments)
            idx = torch.randperm(n, generator=g)[:hot]
            cells = torch.tensor([[1, 2, 0, 0], [1, 3, 0, 0], [H - 1, W - 1, D - 1, B - 1]])
            coords[idx] = cells[torch.randint(0, 3, (hot,), generator=g)]
        coords = coords.to(cdtype)
        x = feats.clone().requires_grad_(True)
        out = bpt.bev_pool(x, coords, B, D, H, W)
        up = torch.randn(out.shape, generator=g).to(fdtype)
        (out * up).sum().backward()
        save(name, feats=feats.float(), coords=coords, shape=[B, D, H, W], out=out.detach().float(),
             upstream=up.float(), grad=x.grad.float(), fdtype=str(fdtype))

    # tests/test_ops/test_bev_pool.py:87-105 shapes, on CPU with a CPU generator
    rand_case('bev_rand_small_f32', 64, 8, 2, 3, 4, 5, 0, torch.int32, torch.float32)
    rand_case('bev_rand_small_f16', 64, 8, 2, 3, 4, 5, 0, torch.int32, torch.float16)
    rand_case('bev_rand_medium_i64', 12000, 8, 2, 2, 30, 41, 1, torch.int64, torch.float32, hot=7000)
    rand_case('bev_rand_odd_c', 3000, 5, 3, 1, 17, 33, 2, torch.int64, torch.float32)

    # full-size det B=1 with exactly-summable features: order-independent digest
    case = synth.det_bev_pool_case(1, dyadic=True)
    out = bpt.bev_pool(case.feats, case.coords, case.B, case.D, case.H, case.W)
    return {
        'det_b1_dyadic': {
            'coords_sha': sha(case.coords.numpy()), 'feats_sha': sha(case.feats.numpy()),
            'n': int(case.coords.shape[0]), 'shape': [case.B, case.D, case.H, case.W],
            'out_sha': sha(out.numpy()), 'out_sum': float(out.double().sum()),
        }
    }


VOXEL_SIZE = [1.0, 1.0, 1.0]
COORS_RANGE = [0.0, 0.0, 0.0, 4.0, 4.0, 4.0]
POINTS8 = [[0.2, 0.3, 0.1, 1.0], [0.7, 0.9, 0.8, 2.0], [1.2, 1.1, 1.0, 3.0], [1.9, 1.8, 1.7, 4.0],
           [2.2, 2.4, 2.1, 5.0], [3.9, 3.7, 3.8, 6.0], [-0.2, 0.1, 0.1, 7.0], [4.2, 0.1, 0.1, 8.0]]


def hard(vt, points, vsize, crange, mp, mv):
    voxels = torch.zeros((mv, mp, points.size(1)), dtype=points.dtype)
    coors = torch.zeros((mv, 3), dtype=torch.int32)
    num = torch.zeros((mv,), dtype=torch.int32)
    vn = vt.hard_voxelize(points, voxels, coors, num, vsize, crange, mp, mv, 3, True)
    return voxels, coors, num, vn


def voxel_cases(vt):
    # the 8-point fixture, tests/test_ops/test_voxel.py:27-45
    pts = torch.tensor(POINTS8, dtype=torch.float32)
    coors = torch.zeros((8, 3), dtype=torch.int32)
    vt.dynamic_voxelize(pts, coors, VOXEL_SIZE, COORS_RANGE, 3)
    res = {}
    for mp, mv in [(2, 8), (3, 8), (1, 2)]:
        v, c, nump, vn = hard(vt, pts, VOXEL_SIZE, COORS_RANGE, mp, mv)
        res[f'mp{mp}_mv{mv}'] = (v, c, nump, vn)
    save('voxel_points8', points=pts, dyn_coors=coors,
         **{f'{k}_voxels': v[0] for k, v in res.items()}, **{f'{k}_coors': v[1] for k, v in res.items()},
         **{f'{k}_num': v[2] for k, v in res.items()}, **{f'{k}_vn': v[3] for k, v in res.items()})

    # non-cubic grid, voxel overflow and the max_voxels cap; values on cell edges
    g = torch.Generator().manual_seed(3)
    vsize = [0.25, 0.2, 0.5]
    crange = [-3.0, -2.0, -1.0, 3.0, 2.0, 1.0]
    n = 4000
    pts = torch.empty((n, 5))
    pts[:, 0] = torch.rand(n, generator=g) * 7.0 - 3.5
    pts[:, 1] = torch.rand(n, generator=g) * 5.0 - 2.5
    pts[:, 2] = torch.rand(n, generator=g) * 2.6 - 1.3
    pts[:, 3:] = torch.randn((n, 2), generator=g)
    edge = torch.randperm(n, generator=g)[:600]  # exact multiples of the voxel size
    pts[edge, 0] = (torch.randint(-14, 15, (600,), generator=g).float() * 0.25)
    pts[edge, 1] = (torch.randint(-12, 13, (600,), generator=g).float() * 0.2)
    pts[edge[:300], 2] = (torch.randint(-3, 4, (300,), generator=g).float() * 0.5)
    hot = torch.randperm(n, generator=g)[:500]  # crowd a few voxels past max_points
    pts[hot, :3] = torch.tensor([0.1, 0.1, 0.1]) + 0.01 * torch.rand((500, 3), generator=g)
    coors = torch.zeros((n, 3), dtype=torch.int32)
    vt.dynamic_voxelize(pts, coors, vsize, crange, 3)
    out = {'points': pts, 'dyn_coors': coors, 'vsize': torch.tensor(vsize), 'crange': torch.tensor(crange)}
    for mp, mv in [(5, 300), (5, 100000), (32, 50)]:
        v, c, nump, vn = hard(vt, pts, vsize, crange, mp, mv)
        out.update({f'mp{mp}_mv{mv}_voxels': v, f'mp{mp}_mv{mv}_coors': c, f'mp{mp}_mv{mv}_num': nump,
                    f'mp{mp}_mv{mv}_vn': vn})
    save('voxel_rand_noncubic', **out)

    # full-size LiDAR sample (config 3): digests only (the Python loop takes ~10 s)
    pts = synth.lidar_sweeps(0)
    v, c, nump, vn = hard(vt, pts, list(synth.LIDAR_VOXEL_SIZE), list(synth.LIDAR_RANGE),
                          synth.LIDAR_MAX_POINTS, synth.LIDAR_MAX_VOXELS)
    return {
        'lidar_s0': {
            'points_sha': sha(pts.numpy()), 'n': int(pts.shape[0]), 'voxel_num': int(vn),
            'voxels_sha': sha(v[:vn].numpy()), 'coors_sha': sha(c[:vn].numpy()),
            'num_sha': sha(nump[:vn].numpy()), 'points_stored': int(nump[:vn].sum()),
        }
    }


def scatter_cases(spt):
    feats = torch.tensor([[1.0, 2.0, -1.0], [3.0, 0.5, -2.0], [4.0, -1.0, 5.0], [2.0, 3.0, 0.0],
                          [8.0, 1.0, -3.0], [6.0, 4.0, 7.0], [9.0, 9.0, 9.0]])
    coors = torch.tensor([[0, 0, 0], [0, 0, 0], [1, 1, 1], [1, 1, 1], [2, 2, 2], [2, 2, 2], [-1, -1, -1]],
                         dtype=torch.int32)
    g = torch.Generator().manual_seed(4)
    n = 300
    rf = torch.randn((n, 6), generator=g)
    rf[::7] = rf[3]  # ties for the max backward
    rc = torch.randint(-1, 4, (n, 3), generator=g).to(torch.int32)
    out = {}
    for name, (f, c) in {'fix': (feats, coors), 'rand': (rf, rc)}.items():
        out[f'{name}_feats'] = f
        out[f'{name}_coors'] = c
        for red in ('sum', 'mean', 'max'):
            vf, vc, mp, cnt = spt.dynamic_point_to_voxel_forward(f, c, red)
            up = torch.linspace(0.1, 1.0, vf.numel()).view_as(vf)
            gf = torch.zeros_like(f)
            spt.dynamic_point_to_voxel_backward(gf, up.contiguous(), f, vf, mp, cnt, red)
            out.update({f'{name}_{red}_vf': vf, f'{name}_{red}_vc': vc, f'{name}_{red}_map': mp,
                        f'{name}_{red}_cnt': cnt, f'{name}_{red}_up': up, f'{name}_{red}_grad': gf})
    save('scatter_cases', **out)


def main():
    if len(sys.argv) < 2:
        raise SystemExit('usage: make_golden.py <path to the bevfusion-triton checkout>')
    ref = Path(sys.argv[1]).resolve()
    bpt, vt, spt = import_reference(ref)
    only = sys.argv[sys.argv.index('--only') + 1] if '--only' in sys.argv else None
    if only == 'spconv':
        spconv_cases(import_spconv())
        return
    if only == 'spconv_conv':
        spconv_conv_cases(import_spconv())
        return
    if only == 'geometry':
        digests = json.loads((HERE / 'digests.json').read_text())
        digests.update(geometry_cases(import_base_transform(ref)))
        (HERE / 'digests.json').write_text(json.dumps(digests, indent=1, sort_keys=True) + '\n')
        return
    torch.set_num_threads(8)
    digests = {}
    digests.update(bev_cases(bpt))
    digests.update(voxel_cases(vt))
    scatter_cases(spt)
    spconv_cases(import_spconv())
    spconv_conv_cases(import_spconv())
    digests.update(geometry_cases(import_base_transform(ref)))
    (HERE / 'digests.json').write_text(json.dumps(digests, indent=1, sort_keys=True) + '\n')
    print(json.dumps(digests, indent=1))


if __name__ == '__main__':
    main()
