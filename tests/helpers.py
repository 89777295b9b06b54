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


def ico_sphere(level: int = 1, radius: float = 1.0):
    """Icosphere (vertices (V, 3) float32, faces (F, 3) int32): the 12-vertex
    icosahedron, each subdivision splitting every triangle into four with
    edge midpoints pushed to the sphere."""
    t = (1.0 + 5.0 ** 0.5) / 2.0
    v = [(-1, t, 0), (1, t, 0), (-1, -t, 0), (1, -t, 0), (0, -1, t), (0, 1, t), (0, -1, -t), (0, 1, -t),
         (t, 0, -1), (t, 0, 1), (-t, 0, -1), (-t, 0, 1)]
    f = [(0, 11, 5), (0, 5, 1), (0, 1, 7), (0, 7, 10), (0, 10, 11), (1, 5, 9), (5, 11, 4), (11, 10, 2), (10, 7, 6),
         (7, 1, 8), (3, 9, 4), (3, 4, 2), (3, 2, 6), (3, 6, 8), (3, 8, 9), (4, 9, 5), (2, 4, 11), (6, 2, 10),
         (8, 6, 7), (9, 8, 1)]
    verts = [np.array(p, dtype=np.float64) / np.linalg.norm(p) for p in v]
    for _ in range(level):
        mid = {}

        def m(a, b):
            key = (min(a, b), max(a, b))
            if key not in mid:
                p = verts[a] + verts[b]
                verts.append(p / np.linalg.norm(p))
                mid[key] = len(verts) - 1
            return mid[key]

        nf = []
        for a, b, c in f:
            ab, bc, ca = m(a, b), m(b, c), m(c, a)
            nf += [(a, ab, ca), (b, bc, ab), (c, ca, bc), (ab, bc, ca)]
        f = nf
    return (np.array(verts) * radius).astype(np.float32), np.array(f, dtype=np.int32)
