"""Seeded synthetic inputs for the grid scatter-reduce hot path.

The nuScenes data the reference trains on is not available, so these
generators stand in for it with the same shapes, sizes and value
distributions:

* ``det_bev_pool_case`` / ``seg_bev_pool_case`` follow the reference camera
  branch: frustum (models/vtransforms/base.py:67-80), geometry
  (base.py:82-126), quantise + filter (base.py:131-158) and the depth x context
  features (models/vtransforms/depth_lss.py:80-94).  Six pinhole cameras on a
  ring (yaw 0, +-55, +-110, 180 degrees), 1.6 m above the ground.
* ``lidar_sweeps`` builds a 32-beam, 10-sweep spinning-LiDAR point cloud whose
  points feed hard voxelisation (ops/voxel/voxelize.py:12-71).

Sample ``i`` of a batch depends only on ``(seed, i)`` so that any shard of a
batch reproduces the rows of the full batch.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

# --------------------------------------------------------------------------
# camera rig
# --------------------------------------------------------------------------

IMAGE_SIZE = (256, 704)
FEATURE_SIZE = (32, 88)
DBOUND = (1.0, 60.0, 0.5)
FX = FY = 560.0
CX, CY = 352.0, 128.0
CAM_HEIGHT = 1.6
CAM_YAWS_DEG = (0.0, 55.0, -55.0, 110.0, -110.0, 180.0)
CHANNELS = 80

DET_GRID = dict(xbound=(-54.0, 54.0, 0.3), ybound=(-54.0, 54.0, 0.3), zbound=(-10.0, 10.0, 20.0))
SEG_GRID = dict(xbound=(-51.2, 51.2, 0.4), ybound=(-51.2, 51.2, 0.4), zbound=(-10.0, 10.0, 20.0))


def _frustum() -> torch.Tensor:
    """[D, fH, fW, 3] of (u, v, depth); base.py:67-80."""
    ih, iw = IMAGE_SIZE
    fh, fw = FEATURE_SIZE
    ds = torch.arange(*DBOUND, dtype=torch.float32)
    d = ds.numel()
    xs = torch.linspace(0, iw - 1, fw, dtype=torch.float32).view(1, 1, fw).expand(d, fh, fw)
    ys = torch.linspace(0, ih - 1, fh, dtype=torch.float32).view(1, fh, 1).expand(d, fh, fw)
    dd = ds.view(d, 1, 1).expand(d, fh, fw)
    return torch.stack((xs, ys, dd), -1)


def _cam_to_lidar() -> tuple[torch.Tensor, torch.Tensor]:
    """Rotations [6,3,3] (float64) and translations [6,3] (fp32) of the six
    ring cameras.

    Camera axes: x right, y down, z forward.  LiDAR axes: x forward, y left,
    z up.  Each camera is the forward camera turned by its yaw about z.
    """
    base = torch.tensor([[0.0, 0.0, 1.0], [-1.0, 0.0, 0.0], [0.0, -1.0, 0.0]], dtype=torch.float64)
    rots = []
    for yaw in CAM_YAWS_DEG:
        a = math.radians(yaw)
        rz = torch.tensor(
            [[math.cos(a), -math.sin(a), 0.0], [math.sin(a), math.cos(a), 0.0], [0.0, 0.0, 1.0]],
            dtype=torch.float64,
        )
        rots.append(rz @ base)
    rots = torch.stack(rots)
    trans = torch.tensor([[0.0, 0.0, CAM_HEIGHT]] * len(CAM_YAWS_DEG), dtype=torch.float32)
    return rots, trans


def frustum_geometry() -> torch.Tensor:
    """LiDAR-frame frustum points [6, D, fH, fW, 3] (fp32); base.py:82-126.

    post_rots = I and post_trans = 0, so the image-augmentation undo is the
    identity; the remaining steps are (u*d, v*d, d) followed by
    ``cam2lidar_rot @ K^-1`` and the camera translation.  The 3x3 product is
    formed in float64 and applied with explicit element-wise fp32 ops (no
    BLAS), so the result is bitwise identical on every x86 host.
    """
    fr = _frustum()
    pts = torch.cat((fr[..., :2] * fr[..., 2:3], fr[..., 2:3]), -1)  # [D,fH,fW,3]
    kinv = torch.tensor([[1.0 / FX, 0.0, -CX / FX], [0.0, 1.0 / FY, -CY / FY], [0.0, 0.0, 1.0]],
                        dtype=torch.float64)
    rots, trans = _cam_to_lidar()
    outs = []
    for cam in range(rots.size(0)):
        comb = (rots[cam].double() @ kinv).float()
        cols = []
        for i in range(3):
            v = pts[..., 0] * comb[i, 0]
            v = v + pts[..., 1] * comb[i, 1]
            v = v + pts[..., 2] * comb[i, 2]
            cols.append(v + trans[cam, i])
        outs.append(torch.stack(cols, -1))
    return torch.stack(outs).contiguous()


def camera_rig(batch: int, *, augment: bool = False, seed: int = 0, device='cpu') -> dict:
    """Inputs of ``BaseTransform.get_geometry`` (models/vtransforms/base.py:82-126)
    for ``batch`` samples of the six-camera ring: ``frustum`` [D, fH, fW, 3]
    and per camera ``camera2lidar_rots`` / ``intrins`` / ``post_rots``
    [B, 6, 3, 3], ``camera2lidar_trans`` / ``post_trans`` [B, 6, 3], all fp32.

    ``augment`` draws, per sample and seeded, the training-time perturbations
    the reference pipeline applies: image resize 0.9-1.1 and rotation
    +-5.4 degrees with a crop shift (post_rots / post_trans), a few pixels of
    intrinsics jitter, +-2 degrees of camera yaw, and a lidar augmentation
    (``extra_rots`` yaw +-22.5 degrees with scale 0.95-1.05, ``extra_trans``
    +-0.5 m), returned as two more entries.
    """
    g = torch.Generator().manual_seed(seed * 1_000_003 + 17)
    ncam = len(CAM_YAWS_DEG)
    rots64, trans = _cam_to_lidar()
    k = torch.tensor([[FX, 0.0, CX], [0.0, FY, CY], [0.0, 0.0, 1.0]], dtype=torch.float64)
    rots = rots64.unsqueeze(0).repeat(batch, 1, 1, 1)
    intr = k.view(1, 1, 3, 3).repeat(batch, ncam, 1, 1)
    prots = torch.eye(3, dtype=torch.float64).view(1, 1, 3, 3).repeat(batch, ncam, 1, 1)
    ptrans = torch.zeros((batch, ncam, 3), dtype=torch.float64)
    out = {}
    if augment:
        def u(lo, hi, *shape):
            return lo + (hi - lo) * torch.rand(shape, generator=g, dtype=torch.float64)

        yaw = torch.deg2rad(u(-2.0, 2.0, batch, ncam))
        rz = torch.zeros((batch, ncam, 3, 3), dtype=torch.float64)
        rz[..., 0, 0], rz[..., 0, 1], rz[..., 1, 0], rz[..., 1, 1] = yaw.cos(), -yaw.sin(), yaw.sin(), yaw.cos()
        rz[..., 2, 2] = 1.0
        rots = rz @ rots
        intr = intr.clone()
        intr[..., 0, 0] += u(-5.0, 5.0, batch, ncam)
        intr[..., 1, 1] = intr[..., 0, 0]
        intr[..., 0, 2] += u(-4.0, 4.0, batch, ncam)
        intr[..., 1, 2] += u(-4.0, 4.0, batch, ncam)
        sc = u(0.9, 1.1, batch, ncam)
        th = torch.deg2rad(u(-5.4, 5.4, batch, ncam))
        prots = prots.clone()
        prots[..., 0, 0], prots[..., 0, 1] = sc * th.cos(), -sc * th.sin()
        prots[..., 1, 0], prots[..., 1, 1] = sc * th.sin(), sc * th.cos()
        ptrans[..., 0] = u(-30.0, 30.0, batch, ncam)
        ptrans[..., 1] = u(-30.0, 30.0, batch, ncam)
        ey = torch.deg2rad(u(-22.5, 22.5, batch))
        es = u(0.95, 1.05, batch)
        er = torch.zeros((batch, 3, 3), dtype=torch.float64)
        er[:, 0, 0], er[:, 0, 1], er[:, 1, 0], er[:, 1, 1] = es * ey.cos(), -es * ey.sin(), es * ey.sin(), es * ey.cos()
        er[:, 2, 2] = es
        out['extra_rots'] = er.float().to(device)
        out['extra_trans'] = u(-0.5, 0.5, batch, 3).float().to(device)
    out.update(
        frustum=_frustum().to(device),
        camera2lidar_rots=rots.float().to(device),
        camera2lidar_trans=trans.view(1, ncam, 3).repeat(batch, 1, 1).to(device),
        intrins=intr.float().to(device),
        post_rots=prots.float().to(device),
        post_trans=ptrans.float().to(device),
    )
    return out


def lss_geometry(frustum, camera2lidar_rots, camera2lidar_trans, intrins, post_rots, post_trans, extra_rots=None,
                 extra_trans=None):
    """``BaseTransform.get_geometry`` (models/vtransforms/base.py:82-126) as
    the reference computes it, in torch: [B, N, D, fH, fW, 3] LiDAR-frame
    points of every frustum point."""
    B, N, _ = camera2lidar_trans.shape
    points = frustum - post_trans.view(B, N, 1, 1, 1, 3)
    points = post_rots.transpose(-1, -2).reshape(B, N, 1, 1, 1, 3, 3).matmul(points.unsqueeze(-1))
    points = torch.cat((points[:, :, :, :, :, :2] * points[:, :, :, :, :, 2:3], points[:, :, :, :, :, 2:3]), 5)
    combine = torch.linalg.solve(intrins.transpose(-1, -2), camera2lidar_rots.transpose(-1, -2)).transpose(-1, -2)
    points = combine.reshape(B, N, 1, 1, 1, 3, 3).matmul(points).squeeze(-1)
    points = points + camera2lidar_trans.view(B, N, 1, 1, 1, 3)
    if extra_rots is not None:
        points = extra_rots.view(B, 1, 1, 1, 1, 3, 3).expand(B, N, 1, 1, 1, 3, 3).matmul(
            points.unsqueeze(-1)).squeeze(-1)
    if extra_trans is not None:
        points = points + extra_trans.view(B, 1, 1, 1, 1, 3)
    return points


def lss_coords(geom, xbound, ybound, zbound):
    """Quantise + in-grid filter of ``BaseTransform.bev_pool``
    (models/vtransforms/base.py:138-158): (x, y, z, b) int64 coords of every
    frustum point, the kept mask and the grid (B, D, H, W)."""
    B = geom.size(0)
    dx, bx, nx = grid_params(xbound, ybound, zbound)
    dx, bx = dx.to(geom.device), bx.to(geom.device)
    g = ((geom - (bx - dx / 2.0)) / dx).long().reshape(-1, 3)
    b = torch.arange(B, device=geom.device).repeat_interleave(geom[0].numel() // 3).view(-1, 1)
    g = torch.cat((g, b), 1)
    kept = ((g[:, 0] >= 0) & (g[:, 0] < nx[0]) & (g[:, 1] >= 0) & (g[:, 1] < nx[1]) & (g[:, 2] >= 0)
            & (g[:, 2] < nx[2]))
    return g, kept, (B, nx[2], nx[0], nx[1])


def grid_params(xbound, ybound, zbound):
    """dx, lower edge and cell counts; gen_dx_bx (base.py:19-23)."""
    rows = [xbound, ybound, zbound]
    dx = torch.tensor([r[2] for r in rows], dtype=torch.float32)
    bx = torch.tensor([r[0] + r[2] / 2.0 for r in rows], dtype=torch.float32)
    nx = [int((r[1] - r[0]) / r[2]) for r in rows]
    return dx, bx, nx


def quantize_geometry(geom: torch.Tensor, xbound, ybound, zbound):
    """Cell coordinates (x, y, z) int64 and the kept mask; base.py:138-158.

    ``.long()`` truncates toward zero, exactly like the reference caller.
    """
    dx, bx, nx = grid_params(xbound, ybound, zbound)
    g = ((geom.reshape(-1, 3) - (bx - dx / 2.0)) / dx).long()
    kept = (
        (g[:, 0] >= 0) & (g[:, 0] < nx[0]) & (g[:, 1] >= 0) & (g[:, 1] < nx[1])
        & (g[:, 2] >= 0) & (g[:, 2] < nx[2])
    )
    return g, kept, nx


@dataclass
class BevPoolCase:
    feats: torch.Tensor  # [N, C]
    coords: torch.Tensor  # [N, 4] int64 (x, y, z, b)
    B: int
    D: int  # = nz
    H: int  # = nx
    W: int  # = ny


def _dyadic_feats(sample: int, seed: int, n: int, device, dtype) -> torch.Tensor:
    """Integers / 64 in [-16, 16): every partial sum over a cell is exact in
    fp32, so the pooled result does not depend on summation order."""
    g = torch.Generator()
    g.manual_seed(seed * 1_000_003 + sample)
    k = torch.randint(-1024, 1024, (n, CHANNELS), generator=g, dtype=torch.int32)
    return (k.float() / 64.0).to(dtype).to(device)


def _sample_feats(sample: int, seed: int, n_keep_idx: torch.Tensor, device, dtype) -> torch.Tensor:
    """softmax(depth logits) x context for one sample, kept rows only.

    depth_lss.py:91-94: depth [6, D, fH, fW] softmax over D, context
    [6, C, fH, fW]; the product is laid out (n, d, h, w, c).
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1_000_003 + sample)
    ncam = len(CAM_YAWS_DEG)
    d = int(round((DBOUND[1] - DBOUND[0]) / DBOUND[2]))
    fh, fw = FEATURE_SIZE
    logits = torch.randn((ncam, d, fh, fw), generator=g, device=device, dtype=torch.float32)
    ctx = torch.randn((ncam, CHANNELS, fh, fw), generator=g, device=device, dtype=torch.float32)
    depth = logits.softmax(dim=1)
    # (n, d, h, w, c) = depth[n, d, h, w] * ctx[n, c, h, w]
    x = depth.unsqueeze(-1) * ctx.permute(0, 2, 3, 1).unsqueeze(1)
    x = x.reshape(-1, CHANNELS)[n_keep_idx]
    return x.to(dtype).contiguous()


def bev_pool_case(batch: int, grid: dict, *, seed: int = 0, device='cpu', dtype=torch.float32,
                  sample_offset: int = 0, dyadic: bool = False) -> BevPoolCase:
    """Batch of ``batch`` camera samples, concatenated in sample order.

    Every sample uses the same rig (same geometry, hence the same kept
    points and cell coordinates) with fresh features.  ``sample_offset``
    selects rows ``sample_offset .. sample_offset + batch - 1`` of a larger
    batch; the batch column is re-based to start at 0.  ``dyadic`` replaces the
    depth x context features by exactly-summable values (golden tests).
    """
    geom = frustum_geometry()
    g, kept, nx = quantize_geometry(geom, **grid)
    keep_idx = torch.nonzero(kept).squeeze(1)
    cell = g[keep_idx]
    feats, coords = [], []
    for i in range(batch):
        s = sample_offset + i
        if dyadic:
            feats.append(_dyadic_feats(s, seed, keep_idx.numel(), device, dtype))
        else:
            feats.append(_sample_feats(s, seed, keep_idx.to(device), device, dtype))
        b = torch.full((cell.size(0), 1), i, dtype=torch.int64)
        coords.append(torch.cat((cell, b), 1))
    feats = torch.cat(feats, 0)
    coords = torch.cat(coords, 0).to(device)
    return BevPoolCase(feats, coords, batch, nx[2], nx[0], nx[1])


def det_bev_pool_case(batch: int = 1, **kw) -> BevPoolCase:
    return bev_pool_case(batch, DET_GRID, **kw)


def seg_bev_pool_case(batch: int = 1, **kw) -> BevPoolCase:
    return bev_pool_case(batch, SEG_GRID, **kw)


# --------------------------------------------------------------------------
# LiDAR
# --------------------------------------------------------------------------

LIDAR_VOXEL_SIZE = (0.075, 0.075, 0.2)
LIDAR_RANGE = (-54.0, -54.0, -5.0, 54.0, 54.0, 3.0)
LIDAR_MAX_POINTS = 10
LIDAR_MAX_VOXELS = 120000


def lidar_sweeps(sample: int = 0, seed: int = 0, device='cpu') -> torch.Tensor:
    """[346880, 5] fp32 points (x, y, z, intensity, dt) of one sample.

    32 beams with elevation linspace(-30, +10) degrees, 1084 azimuth steps,
    10 sweeps 0.05 s apart.  Beams below the horizon hit the ground plane at
    z = -1.8 m (capped at 70 m); the rest return at 70 m.  In every sweep 20%
    of rays are replaced by obstacle hits at U(2, 50) m.
    """
    g = torch.Generator()
    g.manual_seed(seed * 1_000_003 + sample)
    el = torch.deg2rad(torch.linspace(-30.0, 10.0, 32, dtype=torch.float64))
    az = torch.linspace(-math.pi, math.pi, 1085, dtype=torch.float64)[:-1]
    el_g, az_g = torch.meshgrid(el, az, indexing='ij')
    ground = torch.where(el_g < 0, 1.8 / torch.tan(-el_g).clamp_min(1e-9), torch.full_like(el_g, 70.0))
    base_r = ground.clamp(max=70.0)
    sweeps = []
    for s in range(10):
        hit = torch.rand(el_g.shape, generator=g, dtype=torch.float64) < 0.2
        obst = 2.0 + 48.0 * torch.rand(el_g.shape, generator=g, dtype=torch.float64)
        r = torch.where(hit, obst, base_r)
        xyz = torch.stack(
            (r * torch.cos(el_g) * torch.cos(az_g), r * torch.cos(el_g) * torch.sin(az_g), r * torch.sin(el_g)),
            -1,
        ).reshape(-1, 3)
        inten = 255.0 * torch.rand((xyz.size(0), 1), generator=g, dtype=torch.float64)
        dt = torch.full((xyz.size(0), 1), 0.05 * s, dtype=torch.float64)
        sweeps.append(torch.cat((xyz, inten, dt), 1))
    return torch.cat(sweeps, 0).float().contiguous().to(device)


@dataclass
class DepthContextCase:
    depth: torch.Tensor    # [B, 6, D_bins, fH, fW] softmax over depth bins
    context: torch.Tensor  # [B, 6, C, fH, fW]
    coords: torch.Tensor   # [B*6*D_bins*fH*fW, 4] int64 (x, y, z, b), unfiltered
    kept: torch.Tensor     # [B*6*D_bins*fH*fW] bool, the caller's in-grid filter
    B: int
    D: int
    H: int
    W: int


def depth_context_case(batch: int, grid: dict, *, seed: int = 0, device='cpu', sample_offset: int = 0):
    """Inputs of the fused camera-branch pooling: the depth distribution and
    context of depth_lss.py:91-92 before their product, and one cell per
    frustum point (out-of-grid points kept, with their out-of-range cells)."""
    geom = frustum_geometry()
    g, kept, nx = quantize_geometry(geom, **grid)
    ncam = len(CAM_YAWS_DEG)
    d = int(round((DBOUND[1] - DBOUND[0]) / DBOUND[2]))
    fh, fw = FEATURE_SIZE
    deps, ctxs, coords, keeps = [], [], [], []
    for i in range(batch):
        gen = torch.Generator(device=device)
        gen.manual_seed(seed * 1_000_003 + sample_offset + i)
        logits = torch.randn((ncam, d, fh, fw), generator=gen, device=device, dtype=torch.float32)
        deps.append(logits.softmax(dim=1))
        ctxs.append(torch.randn((ncam, CHANNELS, fh, fw), generator=gen, device=device, dtype=torch.float32))
        coords.append(torch.cat((g, torch.full((g.size(0), 1), i, dtype=torch.int64)), 1))
        keeps.append(kept)
    return DepthContextCase(torch.stack(deps), torch.stack(ctxs), torch.cat(coords).to(device),
                            torch.cat(keeps).to(device), batch, nx[2], nx[0], nx[1])
