"""Seeded synthetic scenes and cameras for the five benchmark configurations.

No public dataset is involved; these generators produce raw (pre-activation)
Gaussian parameters with the distributions the benchmark configurations
specify, and pinhole cameras in the reference's conventions: world_to_camera
is a row-major 4x4 mapping world to camera space with +z forward, +x right,
+y down; intrinsic is [[fx, 0, cx], [0, fy, cy], [0, 0, 1]].

The activations (exp scales, normalised quaternions, sigmoid opacities) are
applied by `activate`, as scripts/train.py:135-140 of the reference does.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SceneConfig:
    name: str
    n: int
    width: int
    height: int
    focal: float
    extent: float          # means ~ U[-extent, extent]^3 (unless clustered)
    log_scale_mean: float
    log_scale_std: float
    opacity_logit_mean: float
    opacity_logit_std: float
    camera_distance: float
    clusters: int = 0      # > 0: isotropic clusters (config 3)
    cluster_std: float = 0.0


CONFIGS = {
    0: SceneConfig("cfg0", 20_000, 256, 256, 300.0, 1.0, math.log(0.02), 0.3, 0.0, 1.0, 4.0),
    1: SceneConfig("cfg1", 1_000_000, 1920, 1080, 1100.0, 3.0, math.log(0.02), 0.3, 0.0, 1.0, 8.0),
    2: SceneConfig("cfg2", 3_000_000, 1600, 1064, 1200.0, 5.0, math.log(0.02), 0.3, 0.0, 1.0, 10.0),
    3: SceneConfig("cfg3", 2_000_000, 3840, 2160, 2400.0, 2.0, math.log(0.08), 0.4, 1.0, 0.5, 14.0,
                   clusters=64, cluster_std=0.3),
    4: SceneConfig("cfg4", 6_000_000, 1920, 1080, 1100.0, 6.0, math.log(0.02), 0.3, 0.0, 1.0, 12.0),
}


def make_gaussians(cfg: SceneConfig, seed: int = 0, n: int | None = None, device="cpu"):
    """Raw parameters: means (N,3), scales (log, N,3), quaternions (raw, N,4),
    opacities (logits, N), sh_coeffs_dc (N,3), sh_coeffs_rest (N,15,3)."""
    n = cfg.n if n is None else int(n)
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    if cfg.clusters > 0:
        centres = (torch.rand(cfg.clusters, 3, generator=g) * 2 - 1) * cfg.extent
        which = torch.randint(0, cfg.clusters, (n,), generator=g)
        means = centres[which] + torch.randn(n, 3, generator=g) * cfg.cluster_std
    else:
        means = (torch.rand(n, 3, generator=g) * 2 - 1) * cfg.extent
    scales = torch.randn(n, 3, generator=g) * cfg.log_scale_std + cfg.log_scale_mean
    quats = torch.randn(n, 4, generator=g)
    opac = torch.randn(n, generator=g) * cfg.opacity_logit_std + cfg.opacity_logit_mean
    dc = torch.randn(n, 3, generator=g) * 0.3
    rest = torch.randn(n, 15, 3, generator=g) * 0.05
    out = dict(means=means, scales=scales, quaternions=quats, opacities=opac, sh_coeffs_dc=dc,
               sh_coeffs_rest=rest)
    return {k: v.to(device=device, dtype=torch.float32).contiguous() for k, v in out.items()}


def activate(raw):
    """exp scales, unit quaternions, sigmoid opacities (scripts/train.py:135-140)."""
    q = raw["quaternions"]
    return dict(
        means=raw["means"],
        scales=torch.exp(raw["scales"]),
        quaternions=q / torch.norm(q, dim=1, keepdim=True).clamp_min(1e-12),
        opacities=torch.sigmoid(raw["opacities"]),
        sh_coeffs_dc=raw["sh_coeffs_dc"],
        sh_coeffs_rest=raw["sh_coeffs_rest"],
    )


def look_at(eye, target=(0.0, 0.0, 0.0)):
    """world_to_camera (4x4) for a camera at `eye` looking at `target`, with
    camera +y pointing towards world +y ("down" in image space)."""
    eye = torch.tensor(eye, dtype=torch.float64)
    tgt = torch.tensor(target, dtype=torch.float64)
    fwd = tgt - eye
    fwd = fwd / fwd.norm()
    down = torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64)
    if abs(float(fwd @ down)) > 0.999:
        down = torch.tensor([0.0, 0.0, 1.0], dtype=torch.float64)
    right = torch.linalg.cross(down, fwd)
    right = right / right.norm()
    dn = torch.linalg.cross(fwd, right)
    R = torch.stack([right, dn, fwd])
    w2c = torch.eye(4, dtype=torch.float64)
    w2c[:3, :3] = R
    w2c[:3, 3] = -R @ eye
    return w2c.to(torch.float32)


def intrinsic_for(cfg: SceneConfig, width=None, height=None):
    w = cfg.width if width is None else width
    h = cfg.height if height is None else height
    return torch.tensor([[cfg.focal, 0.0, w / 2.0], [0.0, cfg.focal, h / 2.0], [0.0, 0.0, 1.0]],
                        dtype=torch.float32)


def orbit_cameras(cfg: SceneConfig, count: int, seed: int = 0, sphere: bool = False):
    """`count` world_to_camera matrices at distance cfg.camera_distance looking
    at the origin. View 0 of the orbit is the camera at (0, 0, -distance);
    with sphere=True directions are seeded-uniform on the sphere."""
    r = cfg.camera_distance
    mats = []
    if sphere:
        g = torch.Generator(device="cpu").manual_seed(int(seed) + 7919)
        d = torch.randn(count, 3, generator=g, dtype=torch.float64)
        d = d / d.norm(dim=1, keepdim=True)
        for k in range(count):
            mats.append(look_at(tuple((d[k] * r).tolist())))
    else:
        for k in range(count):
            a = 2.0 * math.pi * k / max(count, 1)
            mats.append(look_at((r * math.sin(a), 0.0, -r * math.cos(a))))
    return torch.stack(mats)


def primary_camera(cfg: SceneConfig):
    """The configuration's single camera: at (0, 0, -distance) looking +z."""
    w2c = torch.eye(4, dtype=torch.float32)
    w2c[2, 3] = cfg.camera_distance
    return w2c
