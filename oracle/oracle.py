"""CPU ORACLE — TEST INFRASTRUCTURE ONLY (Python side).

ctypes wrapper of ``oracle/_build/libgs_oracle.so`` (the C++ restatement in
gs_oracle.cpp) plus numpy pipelines that chain its stages the way
src/mlx3d/splatting/render.py:29-112 chains the reference's.  Used by tests/,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline only; the product
package never imports it.
"""

from __future__ import annotations

import ctypes
import subprocess
from ctypes import c_float, c_int, c_int64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libgs_oracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(LIB_PATH))
        P = c_void_p
        lib.or_project.argtypes = [P, P, P, P, c_int64, c_float, c_int, P, P, P, P, P, c_int]
        lib.or_eval_sh.argtypes = [c_int, P, c_int64, c_int, c_int, P, P]
        lib.or_sh_colors.argtypes = [P, c_int, P, P, c_int64, c_int, P, c_int]
        lib.or_activate.argtypes = [P, P, c_int64, P, P]
        lib.or_bin_count.argtypes = [P, P, P, c_int64, c_int, c_int, P]
        lib.or_bin_count.restype = c_int64
        lib.or_bin_fill.argtypes = [P, P, P, P, c_int64, c_int, c_int, c_int64, P, P]
        lib.or_rasterize_fwd.argtypes = [P, P, P, c_int, P, P, P, P, P, c_int, c_int, P, P, P, P, c_int, P]
        lib.or_rasterize_bwd.argtypes = [P, P, P, c_int, P, c_int64, P, P, P, c_int, c_int, P, P, P, P, P, P, P, P,
                                         c_int]
        lib.or_project_ut.argtypes = [P, P, P, P, P, c_int64, c_float, c_int, P, P, P, P, P]
        lib.or_mesh_rasterize.argtypes = [P, P, P, P, c_int, c_int, c_float, P, P]
        lib.or_expf.argtypes = [c_float]
        lib.or_expf.restype = c_float
        lib.or_expf_nonpos_mismatches.argtypes = []
        lib.or_expf_nonpos_mismatches.restype = ctypes.c_int64
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _p(a):
    return None if a is None else a.ctypes.data_as(c_void_p)


def expf(x: float) -> float:
    return load().or_expf(x)


def expf_nonpos_mismatches() -> int:
    """Exhaustive count of floats in [-87, 0] where the compositors'
    exponential differs bitwise from gs_expf."""
    return int(load().or_expf_nonpos_mismatches())


def activate(log_scales, logits):
    """exp / sigmoid activations with the shared exponential (model.py:116-122)."""
    ls, lg = _f32(log_scales), _f32(logits)
    s = np.empty_like(ls)
    o = np.empty_like(lg)
    load().or_activate(_p(ls), _p(lg), lg.shape[0], _p(s), _p(o))
    return s, o


def project(cam, means, quats, scales, blur=0.3, antialias=False, threads=0):
    """project_gaussians (projection.py:24-146); ``cam`` is a GsCamera."""
    means, quats, scales = _f32(means), _f32(quats), _f32(scales)
    n = means.shape[0]
    out = {
        "means2d": np.empty((n, 2), np.float32),
        "conics": np.empty((n, 3), np.float32),
        "depths": np.empty((n,), np.float32),
        "radii": np.empty((n,), np.float32),
        "compensation": np.empty((n,), np.float32),
    }
    load().or_project(ctypes.byref(cam), _p(means), _p(quats), _p(scales), n, blur, int(antialias and blur > 0),
                      *(_p(out[k]) for k in ("means2d", "conics", "depths", "radii", "compensation")), threads)
    return out


def project_ut(camera, means, quats, scales, blur=0.3, antialias=False):
    """project_gaussians_ut (projection.py:149-205) for a mlx3d_b200 Camera."""
    means, quats, scales = _f32(means), _f32(quats), _f32(scales)
    n = means.shape[0]
    out = {k: np.empty(s, np.float32) for k, s in (("means2d", (n, 2)), ("conics", (n, 3)), ("depths", (n,)),
                                                  ("radii", (n,)), ("compensation", (n,)))}
    cam, lens = camera.to_native(), camera.lens_native()
    load().or_project_ut(ctypes.byref(cam), ctypes.byref(lens), _p(means), _p(quats), _p(scales), n, blur,
                         int(antialias and blur > 0),
                         *(_p(out[k]) for k in ("means2d", "conics", "depths", "radii", "compensation")))
    return out


def eval_sh(degree, sh, dirs):
    sh, dirs = _f32(sh), _f32(dirs)
    n, k, c = sh.shape
    out = np.empty((n, c), np.float32)
    load().or_eval_sh(degree, _p(sh), n, k, c, _p(dirs), _p(out))
    return out


def sh_colors(cam, degree, means, sh, threads=0):
    """max(eval_sh(degree, sh, normalised view dirs), 0) (render.py:77-80)."""
    means, sh = _f32(means), _f32(sh)
    n, k, _ = sh.shape
    out = np.empty((n, 3), np.float32)
    load().or_sh_colors(ctypes.byref(cam), degree, _p(means), _p(sh), n, k, _p(out), threads)
    return out


def bin_gaussians(means2d, radii, depths, width, height, conics=None):
    """(counts, sorted_ids, tile_ranges, tiles_x, tiles_y) (tiles.py:19-182);
    ``conics`` turns on the tile refinement (tiles.py:91-164)."""
    means2d, radii, depths = _f32(means2d), _f32(radii), _f32(depths)
    conics = None if conics is None else _f32(conics)
    n = means2d.shape[0]
    counts = np.empty((n,), np.int32)
    lib = load()
    d = lib.or_bin_count(_p(means2d), _p(radii), _p(conics), n, width, height, _p(counts))
    tx, ty = (width + 15) // 16, (height + 15) // 16
    ids = np.empty((d,), np.int32)
    ranges = np.empty((tx * ty, 2), np.int32)
    lib.or_bin_fill(_p(means2d), _p(radii), _p(depths), _p(conics), n, width, height, d, _p(ids), _p(ranges))
    return counts, ids, ranges, tx, ty


def mesh_rasterize(tri_xy, tri_z, ids, ranges, width, height, znear):
    """Hard z-buffer over binned triangles (renderer/rasterizer.py:29-79):
    (pix_to_face (H, W) int32, zbuf (H, W))."""
    tri_xy, tri_z, ids, ranges = _f32(tri_xy), _f32(tri_z), _i32(ids), _i32(ranges)
    p2f = np.empty((height, width), np.int32)
    zb = np.empty((height, width), np.float32)
    load().or_mesh_rasterize(_p(tri_xy), _p(tri_z), _p(ids), _p(ranges), width, height, float(znear), _p(p2f),
                             _p(zb))
    return p2f, zb


def rasterize_fwd(means2d, conics, colors, opac, ids, ranges, width, height, background=None, depths=None,
                  threads=0):
    """Forward compositor (rasterize.py:28-98) and depth (rasterize.py:223-290)."""
    means2d, conics, opac = _f32(means2d), _f32(conics), _f32(opac)
    colors = None if colors is None else _f32(colors)
    c = 0 if colors is None else colors.shape[1]
    ids, ranges = _i32(ids), _i32(ranges)
    bg = None if background is None else _f32(background)
    dz = None if depths is None else _f32(depths)
    image = np.empty((height, width, max(c, 1)), np.float32)
    final_T = np.empty((height, width), np.float32)
    n_contrib = np.empty((height, width), np.int32)
    depth = np.empty((height, width), np.float32) if depths is not None else None
    stats = np.zeros(2, np.int64)
    load().or_rasterize_fwd(_p(means2d), _p(conics), _p(colors), c, _p(opac), _p(dz), _p(ids), _p(ranges), _p(bg),
                            width, height, _p(image), _p(final_T), _p(n_contrib), _p(depth), threads, _p(stats))
    out = {"final_T": final_T, "alpha": 1.0 - final_T, "n_contrib": n_contrib,
           "pairs_evaluated": int(stats[0]), "pairs_composited": int(stats[1])}
    if c:
        out["image"] = image
    if depth is not None:
        out["depth"] = depth
    return out


def rasterize_bwd(means2d, conics, colors, opac, ids, ranges, width, height, background, final_T, n_contrib,
                  grad_image, grad_final_T=None, threads=0):
    """Backward compositor (rasterize.py:100-221)."""
    means2d, conics, colors, opac = _f32(means2d), _f32(conics), _f32(colors), _f32(opac)
    n, c = colors.shape
    ids, ranges = _i32(ids), _i32(ranges)
    bg = None if background is None else _f32(background)
    final_T, n_contrib, gi = _f32(final_T), _i32(n_contrib), _f32(grad_image)
    gT = None if grad_final_T is None else _f32(grad_final_T)
    g = {
        "means2d": np.empty((n, 2), np.float32),
        "conics": np.empty((n, 3), np.float32),
        "colors": np.empty((n, c), np.float32),
        "opacities": np.empty((n,), np.float32),
    }
    load().or_rasterize_bwd(_p(means2d), _p(conics), _p(colors), c, _p(opac), n, _p(ids), _p(ranges), _p(bg), width,
                            height, _p(final_T), _p(n_contrib), _p(gi), _p(gT), _p(g["means2d"]), _p(g["conics"]),
                            _p(g["colors"]), _p(g["opacities"]), threads)
    return g


def render(cam, width, height, means, quats, scales, opacities, colors=None, sh=None, sh_degree=3, background=None,
           antialias=False, with_depth=False, threads=0, refine_tiles=False):
    """render_gaussians (render.py:29-112) on the oracle: projection,
    opacity * compensation, SH colour, binning, compositing."""
    proj = project(cam, means, quats, scales, antialias=antialias, threads=threads)
    opac = (_f32(opacities) * proj["compensation"]).astype(np.float32)
    if sh is not None:
        colors = sh_colors(cam, sh_degree, means, sh, threads=threads)
    colors = _f32(colors)
    counts, ids, ranges, tx, ty = bin_gaussians(proj["means2d"], proj["radii"], proj["depths"], width, height,
                                                proj["conics"] if refine_tiles else None)
    bg = np.zeros(3, np.float32) if background is None else _f32(background)
    out = rasterize_fwd(proj["means2d"], proj["conics"], colors, opac, ids, ranges, width, height, bg,
                        depths=proj["depths"] if with_depth else None, threads=threads)
    out.update(proj)
    out.update({"colors": colors, "opacities_eff": opac, "tiles_touched": counts, "sorted_ids": ids,
                "tile_ranges": ranges, "tiles_x": tx, "tiles_y": ty, "background": bg})
    return out


def render_grads(camera, means, quats, scales, opacities, colors=None, sh=None, sh_degree=3, background=None,
                 antialias=False, grad_image=None, grad_alpha=None, threads=0, fwd=None):
    """Gradients of render_gaussians for given output cotangents: the C++
    compositor backward (rasterize.py:100-221) chained, through torch float64
    autograd of the restated projection / SH (torch_ref), into the per-Gaussian
    inputs — the path MLX autodiff takes in the reference (rasterize.py:364-403).
    Returns (forward dict, gradient dict)."""
    import torch

    from . import torch_ref

    cam = camera.to_native()
    W, H = camera.width, camera.height
    if fwd is None:
        fwd = render(cam, W, H, means, quats, scales, opacities, colors=colors, sh=sh, sh_degree=sh_degree,
                     background=background, antialias=antialias, threads=threads)
    gT = None if grad_alpha is None else -_f32(grad_alpha)
    g = rasterize_bwd(fwd["means2d"], fwd["conics"], fwd["colors"], fwd["opacities_eff"], fwd["sorted_ids"],
                      fwd["tile_ranges"], W, H, fwd["background"], fwd["final_T"], fwd["n_contrib"], grad_image,
                      gT, threads=threads)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, requires_grad=True)  # noqa: E731
    m, q, s, o = t(means), t(quats), t(scales), t(opacities)
    proj = torch_ref.project(camera, m, q, s, antialias=antialias)
    opac_eff = o * proj["compensation"]
    outs = [proj["means2d"], proj["conics"], opac_eff]
    cots = [g["means2d"], g["conics"], g["opacities"]]
    shv = None
    if sh is not None:
        shv = t(sh)
        dirs = torch_ref.view_dirs(camera, m).detach()
        col = torch.clamp(torch_ref.eval_sh(sh_degree, shv, dirs), min=0.0)
        outs.append(col)
        cots.append(g["colors"])
    torch.autograd.backward(outs, [torch.tensor(c, dtype=torch.float64) for c in cots])
    grads = {"means": m.grad.numpy(), "quats": q.grad.numpy(), "scales": s.grad.numpy(), "opacities": o.grad.numpy(),
             "means2d": g["means2d"], "conics": g["conics"], "colors": g["colors"], "opacities_eff": g["opacities"]}
    if shv is not None:
        grads["sh"] = shv.grad.numpy()
    return fwd, grads
