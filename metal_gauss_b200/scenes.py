"""Seeded synthetic scenes and cameras for the benchmark configurations.

The reference trains on COLMAP / NeRF-synthetic captures that are not
available here; the benchmark configurations are defined on seeded synthetic
inputs with the shapes and value distributions they state:

  cfg1  10k Gaussians, means U[-1,1]^3, log-scales N(ln 0.02, 0.3), quats
        normalise(N(0, I4)), opacity logits N(0,1), SH degree 0 with the DC
        colour U[0,1]; one camera at radius 4 looking at the origin, fov 50,
        128x128, white background, L1 against a U[0,1] target.
  cfg2  100k Gaussians, same distributions, SH degree 3 (bands 1+ N(0,0.05)),
        800x800, fov 40, camera on a radius-4 sphere.
  cfg3  1M Gaussians near the surfaces of 20 random ellipsoids (normal
        jitter N(0, 0.01)), otherwise as cfg2; 100 cameras on a radius-4
        hemisphere; a batch of 8 views per step.
  cfg4  3M Gaussians with log-scales N(ln 0.01, 0.8), SH 3, 1920x1080, fov 60,
        antialiasing on, 256 orbit views, forward only.
  cfg5  6M Gaussians uniform in a 20x20x5 box plus a dense near-ground layer,
        SH 3, 1600x1200, 64 views per step.

Parameters are returned in the trainer's storage form (train.py:117-164):
means, quats (wxyz, unnormalised), log_scales, logit_opac, sh_dc (N,1,3) and
sh_rest (N,15,3), all fp32, on the requested device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

SH_C0 = 0.28209479177387814


@dataclass
class View:
    """One pinhole camera: K (3,3) and world->camera viewmat (4,4), both on
    the host, as the reference's trainer keeps them (train.py:232-246)."""

    K: torch.Tensor
    viewmat: torch.Tensor
    width: int
    height: int


def intrinsics(W: int, H: int, fov_deg: float) -> torch.Tensor:
    """Square pixels, horizontal field of view `fov_deg`, centred principal
    point."""
    f = 0.5 * W / math.tan(math.radians(fov_deg) / 2)
    K = torch.eye(3)
    K[0, 0], K[1, 1], K[0, 2], K[1, 2] = f, f, W / 2, H / 2
    return K


def look_at(pos, target=(0.0, 0.0, 0.0), down=(0.0, 0.0, -1.0)) -> torch.Tensor:
    """World->camera (x right, y down, z forward) for a camera at `pos` looking
    at `target`; `down` is the world direction that should point down-image."""
    p = torch.tensor(pos, dtype=torch.float64)
    t = torch.tensor(target, dtype=torch.float64)
    f = t - p
    f = f / f.norm()
    d = torch.tensor(down, dtype=torch.float64)
    x = torch.linalg.cross(d, f)
    if x.norm() < 1e-9:  # looking straight along `down`
        x = torch.linalg.cross(torch.tensor([0.0, 1.0, 0.0], dtype=torch.float64), f)
    x = x / x.norm()
    y = torch.linalg.cross(f, x)
    R = torch.stack([x, y, f])
    vm = torch.eye(4, dtype=torch.float64)
    vm[:3, :3] = R
    vm[:3, 3] = -R @ p
    return vm.float()


def sphere_views(n: int, radius: float, W: int, H: int, fov: float, seed: int,
                 hemisphere: bool = False) -> list[View]:
    """`n` cameras at distance `radius` looking at the origin, directions drawn
    uniformly on the sphere (upper hemisphere, z > 0.1, when asked)."""
    g = torch.Generator().manual_seed(seed)
    K = intrinsics(W, H, fov)
    views = []
    while len(views) < n:
        d = torch.randn(3, generator=g, dtype=torch.float64)
        d = d / d.norm()
        if hemisphere:
            if d[2] < 0.1:
                continue
        views.append(View(K.clone(), look_at((radius * d).tolist()), W, H))
    return views


def orbit_views(n: int, radius: float, height: float, W: int, H: int, fov: float) -> list[View]:
    """`n` cameras evenly spaced on a horizontal circle, looking at the origin."""
    K = intrinsics(W, H, fov)
    out = []
    for i in range(n):
        a = 2 * math.pi * i / n
        out.append(View(K.clone(), look_at((radius * math.cos(a), radius * math.sin(a), height)),
                        W, H))
    return out


def _base_params(means: torch.Tensor, g: torch.Generator, sh_degree: int, log_scale_mu: float,
                 log_scale_sigma: float) -> dict:
    n = means.shape[0]
    quats = torch.randn(n, 4, generator=g)
    quats = quats / quats.norm(dim=1, keepdim=True)
    log_scales = torch.randn(n, 3, generator=g) * log_scale_sigma + log_scale_mu
    logit_opac = torch.randn(n, generator=g)
    dc = torch.rand(n, 3, generator=g)
    sh_dc = ((dc - 0.5) / SH_C0)[:, None, :]
    sh_rest = torch.zeros(n, 15, 3)
    if sh_degree > 0:
        nb = (sh_degree + 1) ** 2 - 1
        sh_rest[:, :nb] = torch.randn(n, nb, 3, generator=g) * 0.05
    return dict(means=means, quats=quats, log_scales=log_scales, logit_opac=logit_opac,
                sh_dc=sh_dc, sh_rest=sh_rest)


def uniform_cube(n: int, seed: int, sh_degree: int, log_scale_mu: float = math.log(0.02),
                 log_scale_sigma: float = 0.3) -> dict:
    """cfg1 / cfg2 Gaussians: means U[-1,1]^3."""
    g = torch.Generator().manual_seed(seed)
    means = torch.rand(n, 3, generator=g) * 2 - 1
    return _base_params(means, g, sh_degree, log_scale_mu, log_scale_sigma)


def ellipsoid_surfaces(n: int, seed: int, n_ellipsoids: int = 20, jitter: float = 0.01,
                       sh_degree: int = 3) -> dict:
    """cfg3 Gaussians: points near the surfaces of random ellipsoids inside
    [-1,1]^3 (centres U[-0.6,0.6]^3, semi-axes U[0.1,0.4], random rotation),
    displaced along the normal by N(0, jitter)."""
    g = torch.Generator().manual_seed(seed)
    centres = torch.rand(n_ellipsoids, 3, generator=g) * 1.2 - 0.6
    axes = torch.rand(n_ellipsoids, 3, generator=g) * 0.3 + 0.1
    q = torch.randn(n_ellipsoids, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    w, x, y, z = q.unbind(1)
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                     2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                     2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)],
                    1).reshape(-1, 3, 3)
    which = torch.randint(0, n_ellipsoids, (n,), generator=g)
    d = torch.randn(n, 3, generator=g)
    d = d / d.norm(dim=1, keepdim=True)
    a = axes[which]
    local = d * a                                   # on the ellipsoid surface
    normal = d / a
    normal = normal / normal.norm(dim=1, keepdim=True)
    local = local + normal * (torch.randn(n, 1, generator=g) * jitter)
    means = torch.einsum("nij,nj->ni", R[which], local) + centres[which]
    return _base_params(means, g, sh_degree, math.log(0.02), 0.3)


def heavy_tailed(n: int, seed: int) -> dict:
    """cfg4 Gaussians: means U[-1,1]^3, log-scales N(ln 0.01, 0.8), SH 3."""
    return uniform_cube(n, seed, 3, math.log(0.01), 0.8)


def box_with_ground(n: int, seed: int) -> dict:
    """cfg5 Gaussians: 70% uniform in a 20x20x5 box (z in [0,5]), 30% in a
    dense layer z in [0, 0.2]."""
    g = torch.Generator().manual_seed(seed)
    n_ground = int(0.3 * n)
    box = torch.rand(n - n_ground, 3, generator=g) * torch.tensor([20.0, 20.0, 5.0]) \
        - torch.tensor([10.0, 10.0, 0.0])
    ground = torch.rand(n_ground, 3, generator=g) * torch.tensor([20.0, 20.0, 0.2]) \
        - torch.tensor([10.0, 10.0, 0.0])
    means = torch.cat([box, ground])
    return _base_params(means, g, 3, math.log(0.02), 0.3)


def config(name: str, n: int | None = None, seed: int = 0):
    """(params, views, spec) for a benchmark configuration by name."""
    if name == "cfg1":
        p = uniform_cube(n or 10_000, seed, 0)
        K = intrinsics(128, 128, 50.0)
        views = [View(K, look_at((0.0, -4.0 * math.sin(0.35), -4.0 * math.cos(0.35)),
                                 down=(0.0, 1.0, 0.0)), 128, 128)]
        spec = dict(sh_degree=0, background=(1.0, 1.0, 1.0), loss="l1", batch=1)
    elif name == "cfg2":
        p = uniform_cube(n or 100_000, seed, 3)
        views = sphere_views(1, 4.0, 800, 800, 40.0, seed + 1)
        spec = dict(sh_degree=3, background=(0.0, 0.0, 0.0), loss="l1_ssim", batch=1)
    elif name == "cfg3":
        p = ellipsoid_surfaces(n or 1_000_000, seed)
        views = sphere_views(100, 4.0, 800, 800, 40.0, seed + 1, hemisphere=True)
        spec = dict(sh_degree=3, background=(0.0, 0.0, 0.0), loss="l1_ssim", batch=8)
    elif name == "cfg4":
        p = heavy_tailed(n or 3_000_000, seed)
        views = orbit_views(256, 4.0, 1.0, 1920, 1080, 60.0)
        spec = dict(sh_degree=3, background=(0.0, 0.0, 0.0), loss=None, batch=32,
                    antialias=True)
    elif name == "cfg5":
        p = box_with_ground(n or 6_000_000, seed)
        views = orbit_views(64, 12.0, 4.0, 1600, 1200, 60.0)
        spec = dict(sh_degree=3, background=(0.0, 0.0, 0.0), loss="l1_ssim", batch=64)
    else:
        raise ValueError(f"unknown configuration {name!r}")
    return p, views, spec


def random_target(W: int, H: int, seed: int) -> torch.Tensor:
    """Seeded U[0,1] target image (H,W,3)."""
    g = torch.Generator().manual_seed(seed)
    return torch.rand(H, W, 3, generator=g)
