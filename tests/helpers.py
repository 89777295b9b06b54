"""Shared fixtures for the test suite (seeded numpy inputs; the reference's
MLX random streams cannot be reproduced without MLX)."""

from __future__ import annotations

import numpy as np
import torch

from mlx3d_b200.cameras import Camera


def random_scene(seed: int = 0, n: int = 300):
    """The reference's ``random_scene`` fixture (tests/test_splatting.py:30-40):
    N=300, means N(0, 0.5^2), quats N(0,1)^4, scales exp(0.3 N - 2.5),
    opacity sigmoid(N), colours U(0,1), 96x64 at fov 50 from (0,0,-4)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    means = (rng.normal(size=(n, 3)) * 0.5).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    scales = np.exp(rng.normal(size=(n, 3)) * 0.3 - 2.5).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(size=(n,))))).astype(np.float32)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    cam = Camera.look_at(eye=(0, 0, -4.0), at=(0, 0, 0), width=96, height=64, fov=50.0)
    return cam, means, quats, scales, opac, colors


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_rel(a, b) -> float:
    """The reference's gradient metric: max|a - b| / max|b| (test_splatting.py:412-414)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-12))


def t64(a, grad=False):
    t = torch.tensor(np.asarray(a), dtype=torch.float64)
    return t.requires_grad_(grad)
