"""Generates ``reference_outputs.npz``: outputs of the reference's own Python
source (mlx3D 0.2.0) on seeded inputs, used to pin the oracle and the CUDA
path to the reference itself.

MLX has no Linux wheel (the reference pins mlx 0.31.2, macOS arm64 only), so
``mlx.core`` is replaced by the float32 numpy stand-in ``mlx_numpy.py``; the
reference modules are imported unmodified from its checkout:

* ``cameras/cameras.py``  ``Camera.look_at`` -> R, t, fx, cx, ...
* ``splatting/projection.py``  ``project_gaussians`` (antialias off and on)
* ``splatting/sh.py``  ``eval_sh`` (degrees 0-3)
* ``splatting/tiles.py``  ``bin_gaussians`` (plain and ``conics`` refinement)
* ``splatting/reference.py``  ``render_gaussians_reference`` (the naive
  O(N H W) renderer the reference's tests use as their oracle)
* ``splatting/model.py``  ``GaussianModel.densify_and_prune`` and
  ``relocate_mcmc`` (density control; numpy's global generator seeded, the
  split draws stored beside the outputs)

What this pins: the float32 operation order of those modules (every output
but the naive renderer's is compared bit for bit).  What it cannot pin:
MLX's own kernels (its exp, its reduction order, argsort's tie order) and
the Metal compositors.

Run from the repository root in a checkout that has the reference beside it:
``python tests/golden/make_golden.py /path/to/mlx3D``.  Inputs are seeded
numpy PCG64 draws and are stored in the file with the outputs.
"""

from __future__ import annotations

import importlib
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_outputs.npz"


def install_reference(ref_root: Path):
    """Import the reference's camera / splatting modules on the stand-in."""
    sys.path.insert(0, str(HERE))
    import mlx_numpy

    mlx = types.ModuleType("mlx")
    mlx.core = mlx_numpy
    sys.modules["mlx"] = mlx
    sys.modules["mlx.core"] = mlx_numpy
    src = ref_root / "src" / "mlx3d"
    # Package stubs: mlx3d/__init__.py and splatting/__init__.py import the
    # whole library (Metal kernels included); only leaf modules are needed.
    for name, path in (("mlx3d", src), ("mlx3d.splatting", src / "splatting")):
        m = types.ModuleType(name)
        m.__path__ = [str(path)]
        sys.modules[name] = m
    cams = importlib.import_module("mlx3d.cameras")  # its __init__ imports cameras.py only
    mods = {k: importlib.import_module(f"mlx3d.splatting.{k}") for k in ("projection", "sh", "tiles", "reference")}
    # model.py imports IO, mesh structures and the Metal renderer at module
    # level; density control uses none of them, so they are stubbed.
    for name, attrs in (("mlx3d.io", ("load_ply", "save_ply")), ("mlx3d.structures", ("Meshes",)),
                        ("mlx3d.splatting.render", ("render_gaussian_depth", "render_gaussian_features",
                                                    "render_gaussians"))):
        m = types.ModuleType(name)
        for a in attrs:
            setattr(m, a, None)
        sys.modules[name] = m
    mods["model"] = importlib.import_module("mlx3d.splatting.model")
    return cams, mods


def scene_inputs():
    """(name, eye, fov, W, H, means, quats, scales, opacities, colors)."""
    out = []
    # the reference tests' random_scene fixture shape (tests/test_splatting.py:30-40)
    rng = np.random.Generator(np.random.PCG64(0))
    n = 300
    means = (rng.normal(size=(n, 3)) * 0.5).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    scales = np.exp(rng.normal(size=(n, 3)) * 0.3 - 2.5).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(size=(n,))))).astype(np.float32)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    out.append(("random300", (0.0, 0.0, -4.0), 50.0, 96, 64, means, quats, scales, opac, colors))
    # benchmark config C0's distributions (10k in the benchmark; 2000 here)
    rng = np.random.Generator(np.random.PCG64(100))
    n = 2000
    means = (rng.normal(size=(n, 3)) * 0.5).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    quats /= np.linalg.norm(quats, axis=1, keepdims=True)
    scales = np.exp(rng.uniform(-4.5, -3.0, size=(n, 3))).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(size=(n,))))).astype(np.float32)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    out.append(("c0_2k", (0.0, 0.0, -4.0), 60.0, 256, 256, means, quats, scales, opac, colors))
    # C1-like: wide spread, SH3 view directions, off-axis camera, 320x180
    rng = np.random.Generator(np.random.PCG64(101))
    n = 3000
    means = rng.normal(size=(n, 3)).astype(np.float32)
    quats = rng.normal(size=(n, 4)).astype(np.float32)
    scales = np.exp(rng.normal(-3.5, 0.5, size=(n, 3))).astype(np.float32)
    opac = (1.0 / (1.0 + np.exp(-rng.normal(size=(n,))))).astype(np.float32)
    colors = rng.uniform(size=(n, 3)).astype(np.float32)
    e, a = np.radians(20.0), np.radians(30.0)
    eye = (4 * np.cos(e) * np.sin(a), 4 * np.sin(e), -4 * np.cos(e) * np.cos(a))
    out.append(("c1_3k", tuple(float(v) for v in eye), 60.0, 320, 180, means, quats, scales, opac, colors))
    return out


def density_params(seed: int, n: int):
    """Seeded raw parameters (SH degree 1) with a spread of scales and opacities."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return {
        "means": rng.normal(size=(n, 3)).astype(np.float32),
        "scales": rng.normal(-3.0, 1.0, size=(n, 3)).astype(np.float32),
        "quats": rng.normal(size=(n, 4)).astype(np.float32),
        "opacities": rng.normal(0.0, 3.0, size=(n,)).astype(np.float32),
        "sh_dc": rng.normal(size=(n, 1, 3)).astype(np.float32),
        "sh_rest": rng.normal(0, 0.1, size=(n, 3, 3)).astype(np.float32),
    }, rng


def density_cases(model_m, data):
    """densify_and_prune and relocate_mcmc of model.py:406-531 on the stand-in."""
    import mlx_numpy as mx

    names = ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest")
    # densify: 600 rows, a third above the gradient threshold
    params, rng = density_params(200, 600)
    grad_accum = rng.uniform(0.0, 0.0006, size=(600,)).astype(np.float32)
    grad_count = rng.integers(0, 4, size=(600,)).astype(np.float32)
    m = model_m.GaussianModel({k: mx.array(v) for k, v in params.items()}, sh_degree=1)
    np.random.seed(1234)
    stats = m.densify_and_prune(mx.array(grad_accum), mx.array(grad_count), grad_threshold=0.0002,
                                scene_extent=3.0, percent_dense=0.02, min_opacity=0.005,
                                return_optimizer_state=True)
    np.random.seed(1234)
    z = np.random.normal(size=(2 * stats["split"], 3))
    p = "density/"
    for k in names:
        data[p + "in_" + k] = params[k]
        data[p + "out_" + k] = np.asarray(m.params[k])
    data[p + "grad_accum"], data[p + "grad_count"] = grad_accum, grad_count
    data[p + "split_samples"] = z
    data[p + "keep_idx"] = np.asarray(stats["_keep_idx"], np.int32)
    data[p + "counts"] = np.array([stats["cloned"], stats["split"], stats["pruned"]], np.int64)
    # relocation: 500 rows, some never visible or nearly transparent, no jitter
    params, rng = density_params(201, 500)
    grad_accum = rng.uniform(0.0, 0.001, size=(500,)).astype(np.float32)
    grad_count = rng.integers(0, 3, size=(500,)).astype(np.float32)
    m = model_m.GaussianModel({k: mx.array(v) for k, v in params.items()}, sh_degree=1)
    st = m.relocate_mcmc(mx.array(grad_accum), mx.array(grad_count), relocate_frac=0.05, min_opacity=0.01,
                         jitter_scale=0.0)
    p = "mcmc/"
    for k in names:
        data[p + "in_" + k] = params[k]
        data[p + "out_" + k] = np.asarray(m.params[k])
    data[p + "grad_accum"], data[p + "grad_count"] = grad_accum, grad_count
    data[p + "moved_idx"] = np.sort(np.asarray(st["_moved_idx"], np.int64))
    data[p + "relocated"] = np.array([st["relocated"]], np.int64)


def main(ref_root: str):
    cams, mods = install_reference(Path(ref_root))
    import mlx_numpy as mx

    proj_m, sh_m, tiles_m, ref_m = mods["projection"], mods["sh"], mods["tiles"], mods["reference"]
    data = {}
    for name, eye, fov, W, H, means, quats, scales, opac, colors in scene_inputs():
        cam = cams.Camera.look_at(eye=eye, fov=fov, width=W, height=H)
        p = f"{name}/"
        data[p + "eye"] = np.array(eye, np.float64)
        data[p + "fov_wh"] = np.array([fov, W, H], np.float64)
        for k, v in (("means", means), ("quats", quats), ("scales", scales), ("opacities", opac),
                     ("colors", colors)):
            data[p + k] = v
        data[p + "R"] = np.asarray(cam.R, np.float32)
        data[p + "t"] = np.asarray(cam.t, np.float32)
        data[p + "intrinsics"] = np.array([cam.fx, cam.fy, cam.cx, cam.cy, cam.znear], np.float64)
        data[p + "camera_center"] = np.asarray(cam.camera_center, np.float32)
        for aa in (False, True):
            pr = proj_m.project_gaussians(cam, mx.array(means), mx.array(quats), mx.array(scales), antialias=aa)
            for k in ("means2d", "conics", "depths", "radii", "compensation"):
                data[p + f"proj_aa{int(aa)}/{k}"] = np.asarray(pr[k])
        pr = proj_m.project_gaussians(cam, mx.array(means), mx.array(quats), mx.array(scales))
        ids, ranges, tx, ty = tiles_m.bin_gaussians(pr["means2d"], pr["radii"], pr["depths"], W, H)
        data[p + "bin/sorted_ids"] = np.asarray(ids, np.int32)
        data[p + "bin/tile_ranges"] = np.asarray(ranges, np.int32)
        data[p + "bin/tiles_xy"] = np.array([tx, ty], np.int32)
        ids, ranges, _, _ = tiles_m.bin_gaussians(pr["means2d"], pr["radii"], pr["depths"], W, H,
                                                  conics=pr["conics"])
        data[p + "bin_refined/sorted_ids"] = np.asarray(ids, np.int32)
        data[p + "bin_refined/tile_ranges"] = np.asarray(ranges, np.int32)
        # SH: coefficients from a seeded draw for the first 400 Gaussians,
        # directions as render.py:77-79 forms them
        rng = np.random.Generator(np.random.PCG64(7))
        n = min(400, means.shape[0])
        sh = np.zeros((n, 16, 3), np.float32)
        sh[:, 0] = (colors[:n] - 0.5) / np.float32(0.28209479177387814)
        sh[:, 1:] = (rng.normal(size=(n, 15, 3)) * 0.1).astype(np.float32)
        center = np.asarray(cam.camera_center, np.float32)
        d = means[:n] - center
        nrm = np.sqrt((d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1]) + d[:, 2] * d[:, 2])
        dirs = (d / np.maximum(nrm, np.float32(1e-8))[:, None]).astype(np.float32)
        data[p + "sh"] = sh
        data[p + "dirs"] = dirs
        for deg in range(4):
            data[p + f"eval_sh_deg{deg}"] = np.asarray(sh_m.eval_sh(deg, mx.array(sh), mx.array(dirs)))
        # naive renderer (O(N H W)): the two scenes with small images; antialias
        # on the reference fixture only (keeps the file small)
        if W * H <= 320 * 180:
            for aa in ((False, True) if name == "random300" else (False,)):
                bg = np.array([0.1, 0.2, 0.3], np.float32)
                r = ref_m.render_gaussians_reference(cam, mx.array(means), mx.array(quats), mx.array(scales),
                                                     mx.array(opac), mx.array(colors), background=mx.array(bg),
                                                     antialias=aa)
                data[p + f"naive_aa{int(aa)}/image"] = np.asarray(r["image"], np.float32)
                data[p + f"naive_aa{int(aa)}/final_T"] = np.asarray(r["final_T"], np.float32)
    density_cases(mods["model"], data)
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB, {len(data)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the mlx3D checkout>")
    main(sys.argv[1])
