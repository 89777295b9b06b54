"""Seeded synthetic scenes of the benchmark configurations C0-C4.

No public dataset is involved on this path; every input is generated here
with numpy's PCG64 (seed = config index unless given), in float32:

* C0: 10k Gaussians, means N(0, 0.5^2), colours U(0,1) as SH degree 0,
  scales exp(U(-4.5, -3)), quats normalised N(0,1)^4, opacity sigmoid(N(0,1)),
  look_at from (0,0,-4), 256x256, fov 60.
* C1: 100k, SH3 (DC from U(0,1), rest N(0, 0.05^2)), means N(0,1),
  scales exp(N(-4, 0.5^2)), eye radius 4 at azimuth 30 / elevation 20 deg,
  1280x720, fov 60.
* C2: 1M, SH3, means 80% U([-5,5]^3) + 20% from 8 clusters (sigma 0.3,
  centres U([-4,4]^3)), scales exp(N(-4.5, 0.7^2)), opacity sigmoid(N(0, 1.5^2)),
  eye radius 7, 1920x1080, fov 50, antialias.
* C3: 3M as C2 over [-8,8]^3 (centres U([-7,7]^3)); 64 views on a Fibonacci
  sphere of radius 6 (points within 5 deg of the poles dropped), 1600x1060,
  fov 55.
* C4: 6M as C3; 256 views on an orbit of radius 8 at elevation 15 deg,
  3840x2160, fov 60, antialias, depth output.

Parameters are returned raw, as :class:`GaussianModel` stores them
(log-scales, opacity logits, ``sh_dc`` (N,1,3), ``sh_rest`` (N,K-1,3)).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from .cameras import Camera

SH_C0 = 0.28209479177387814


@dataclass
class SceneConfig:
    index: int
    n: int
    width: int
    height: int
    fov: float
    sh_degree: int
    antialias: bool
    n_views: int
    with_depth: bool = False
    loss: str = "l2"
    description: str = ""


CONFIGS = {
    0: SceneConfig(0, 10_000, 256, 256, 60.0, 0, False, 1, loss="l2", description="10k, 256x256, SH0"),
    1: SceneConfig(1, 100_000, 1280, 720, 60.0, 3, False, 1, loss="l1", description="100k, 1280x720, SH3"),
    2: SceneConfig(2, 1_000_000, 1920, 1080, 50.0, 3, True, 1, loss="l1", description="1M, 1920x1080, SH3, AA"),
    3: SceneConfig(3, 3_000_000, 1600, 1060, 55.0, 3, False, 64, loss="l1_ssim",
                   description="3M, 64 views 1600x1060, SH3, train step"),
    4: SceneConfig(4, 6_000_000, 3840, 2160, 60.0, 3, True, 256, with_depth=True, loss="none",
                   description="6M, 256 views 3840x2160, SH3, AA, depth, forward only"),
}


@dataclass
class Scene:
    config: SceneConfig
    params: dict[str, np.ndarray]
    cameras: list[Camera] = field(default_factory=list)
    seed: int = 0

    def torch_params(self, device="cuda", requires_grad=False) -> dict[str, torch.Tensor]:
        out = {}
        for k, v in self.params.items():
            t = torch.from_numpy(v).to(device)
            if requires_grad:
                t.requires_grad_(True)
            out[k] = t
        return out

    def target(self, view: int = 0, device="cuda") -> torch.Tensor:
        """U(0,1) target image of one view (seeded by config, seed and view)."""
        rng = np.random.Generator(np.random.PCG64([self.seed, 1000 + view]))
        c = self.config
        return torch.from_numpy(rng.random((c.height, c.width, 3), dtype=np.float32)).to(device)


def _eye_from_angles(radius: float, azim_deg: float, elev_deg: float) -> list[float]:
    a, e = math.radians(azim_deg), math.radians(elev_deg)
    return [radius * math.sin(a) * math.cos(e), radius * math.sin(e), -radius * math.cos(a) * math.cos(e)]


def _clustered_means(rng, n, half, centre_half):
    n_uni = int(round(0.8 * n))
    uni = rng.uniform(-half, half, size=(n_uni, 3))
    centres = rng.uniform(-centre_half, centre_half, size=(8, 3))
    which = rng.integers(0, 8, size=n - n_uni)
    clus = centres[which] + rng.normal(0.0, 0.3, size=(n - n_uni, 3))
    m = np.concatenate([uni, clus], axis=0)
    return m[rng.permutation(n)]


def _fibonacci_views(count: int, radius: float, min_pole_deg: float = 5.0) -> list[list[float]]:
    """``count`` eyes on a Fibonacci sphere, skipping points within
    ``min_pole_deg`` of the +-y poles (look_at's up vector is +y)."""
    eyes = []
    golden = math.pi * (3.0 - math.sqrt(5.0))
    total = count
    while True:
        eyes = []
        for i in range(total):
            y = 1.0 - 2.0 * (i + 0.5) / total
            r = math.sqrt(max(0.0, 1.0 - y * y))
            th = golden * i
            v = [math.cos(th) * r, y, math.sin(th) * r]
            if math.degrees(math.acos(min(1.0, abs(y)))) < min_pole_deg:
                continue
            eyes.append([radius * c for c in v])
        if len(eyes) >= count:
            return eyes[:count]
        total += 1


def make_scene(index: int, seed: int | None = None, n: int | None = None, views: int | None = None) -> Scene:
    """Generate config ``index`` (optionally with fewer Gaussians / views for
    tests)."""
    cfg = CONFIGS[index]
    seed = index if seed is None else seed
    n = cfg.n if n is None else n
    rng = np.random.Generator(np.random.PCG64(seed))
    K = (cfg.sh_degree + 1) ** 2
    if index == 0:
        means = rng.normal(0.0, 0.5, size=(n, 3))
        log_scales = rng.uniform(-4.5, -3.0, size=(n, 3))
        logits = rng.normal(0.0, 1.0, size=(n,))
    elif index == 1:
        means = rng.normal(0.0, 1.0, size=(n, 3))
        log_scales = rng.normal(-4.0, 0.5, size=(n, 3))
        logits = rng.normal(0.0, 1.0, size=(n,))
    else:
        half, ch = (5.0, 4.0) if index == 2 else (8.0, 7.0)
        means = _clustered_means(rng, n, half, ch)
        log_scales = rng.normal(-4.5, 0.7, size=(n, 3))
        logits = rng.normal(0.0, 1.5, size=(n,))
    q = rng.normal(0.0, 1.0, size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    rgb = rng.uniform(0.0, 1.0, size=(n, 3))
    sh_dc = ((rgb - 0.5) / SH_C0)[:, None, :]
    sh_rest = rng.normal(0.0, 0.05, size=(n, K - 1, 3)) if K > 1 else np.zeros((n, 0, 3))
    params = {
        "means": means.astype(np.float32),
        "scales": log_scales.astype(np.float32),
        "quats": q.astype(np.float32),
        "opacities": logits.astype(np.float32),
        "sh_dc": np.ascontiguousarray(sh_dc, dtype=np.float32),
        "sh_rest": np.ascontiguousarray(sh_rest, dtype=np.float32),
    }
    nv = cfg.n_views if views is None else views
    W, H, fov = cfg.width, cfg.height, cfg.fov
    if index == 0:
        eyes = [[0.0, 0.0, -4.0]]
    elif index in (1, 2):
        eyes = [_eye_from_angles(4.0 if index == 1 else 7.0, 30.0, 20.0)]
    elif index == 3:
        eyes = _fibonacci_views(cfg.n_views, 6.0)[:nv]
    else:
        eyes = [_eye_from_angles(8.0, k * 360.0 / cfg.n_views, 15.0) for k in range(cfg.n_views)][:nv]
    cams = [Camera.look_at(eye=e, at=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0), fov=fov, width=W, height=H) for e in eyes]
    return Scene(cfg, params, cams, seed)
