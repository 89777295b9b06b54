"""Projection + SH + binning + compositing (src/mlx3d/splatting/render.py).

``render_gaussians`` runs the fused path: one per-Gaussian kernel
(projection, opacity x compensation, SH colour, tile counts), the binning
kernels, and one compositor launch; its backward is one compositor-backward
launch plus one per-Gaussian backward launch.  ``render_gaussian_depth`` and
``render_gaussian_features`` compose the standalone differentiable pieces,
like the reference does.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native as nat
from ..cameras import Camera
from .projection import project_gaussians, project_gaussians_ut
from .rasterize import rasterize, rasterize_depth, rasterize_features
from .sh import eval_sh, num_sh_bases
from .tiles import TILE_SIZE, bin_gaussians, bin_with_counts

__all__ = ["render_gaussians", "render_gaussian_depth", "render_gaussian_features"]


@dataclass
class _RenderCfg:
    cam: object  # GsCamera
    width: int
    height: int
    blur: float
    antialias: bool
    flags: int
    sh_degree: int  # -1: colours given directly
    sh_mode: str  # "full" (sh_a = (N, K, 3)), "split" (sh_a = dc (N, 1, 3), sh_b = rest), "colors"
    with_depth: bool
    probe: object = None  # tensor (N, 2) that receives dL/d means2d of the compositor, or None
    refine: bool = False  # AccuTile refinement of the tile duplicates (tiles.py:91-164)
    duplicates: int = 0  # set by the forward: (Gaussian, tile) pairs D of this frame


def _sh_layout(cfg: _RenderCfg, sh_a, sh_b):
    """(dc pointer, dc stride, rest pointer, rest stride) in floats."""
    if cfg.sh_mode == "full":
        k = sh_a.shape[1]
        return nat.ptr(sh_a), 3 * k, (sh_a.data_ptr() + 12) if k > 1 else None, 3 * k
    if cfg.sh_mode == "split":
        k1 = sh_b.shape[1] if sh_b is not None else 0
        return nat.ptr(sh_a), 3, (nat.ptr(sh_b) if k1 > 0 else None), 3 * k1
    return None, 0, None, 0


class _Render(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, opacities, sh_a, sh_b, colors, background, cfg: _RenderCfg):
        n = means.shape[0]
        dev = means.device
        f32 = dict(device=dev, dtype=torch.float32)
        W, H = cfg.width, cfg.height
        tiles_x = (W + TILE_SIZE - 1) // TILE_SIZE
        tiles_y = (H + TILE_SIZE - 1) // TILE_SIZE
        means2d = torch.empty((n, 2), **f32)
        conics = torch.empty((n, 3), **f32)
        depths = torch.empty((n,), **f32)
        radii = torch.empty((n,), **f32)
        comp = torch.empty((n,), **f32)
        opac_out = torch.empty((n,), **f32)
        counts = torch.empty((n,), device=dev, dtype=torch.int32)
        use_sh = cfg.sh_mode != "colors"
        col = torch.empty((n, 3), **f32) if use_sh else colors
        dc, dcs, rest, rests = _sh_layout(cfg, sh_a, sh_b)
        s = nat.stream()
        nat.call(
            "gs_preprocess_forward", cfg.cam, nat.ptr(means), nat.ptr(quats), nat.ptr(scales), nat.ptr(opacities),
            dc, dcs, rest, rests, cfg.sh_degree, n, cfg.blur, int(cfg.antialias), cfg.flags, nat.ptr(means2d),
            nat.ptr(conics), nat.ptr(depths), nat.ptr(radii), nat.ptr(comp), nat.ptr(col) if use_sh else None,
            nat.ptr(opac_out), nat.ptr(counts), s,
        )
        if cfg.refine:
            nat.call("gs_tile_counts_refined", nat.ptr(means2d), nat.ptr(radii), nat.ptr(conics), n, W, H,
                     nat.ptr(counts), s)
        sorted_ids, tile_ranges = bin_with_counts(means2d, radii, depths, counts, W, H,
                                                  conics if cfg.refine else None)
        cfg.duplicates = int(sorted_ids.shape[0])
        image = torch.empty((H, W, 3), **f32)
        final_T = torch.empty((H, W), **f32)
        n_contrib = torch.empty((H, W), device=dev, dtype=torch.int32)
        depth = torch.empty((H, W), **f32) if cfg.with_depth else None
        nat.call(
            "gs_rasterize_forward", nat.ptr(means2d), nat.ptr(conics), nat.ptr(col), 3, nat.ptr(opac_out),
            nat.ptr(depths) if cfg.with_depth else None, nat.ptr(sorted_ids), nat.ptr(tile_ranges),
            nat.ptr(background), W, H, tiles_x, tiles_y, nat.ptr(image), nat.ptr(final_T), nat.ptr(n_contrib),
            nat.ptr(depth), s,
        )
        ctx.cfg = cfg
        ctx.save_for_backward(
            means, quats, scales, opacities, sh_a, sh_b, background, means2d, conics, col, opac_out, sorted_ids,
            tile_ranges, final_T, n_contrib,
        )
        ctx.mark_non_differentiable(radii, n_contrib, counts)
        if depth is not None:
            ctx.mark_non_differentiable(depth)
        ctx.set_materialize_grads(False)
        return image, final_T, n_contrib, means2d, depths, radii, comp, depth, counts

    @staticmethod
    def backward(ctx, g_image, g_final_T, _gn, g_means2d_out, g_depths_out, _gr, g_comp_out, _gd, _gc):
        cfg = ctx.cfg
        (means, quats, scales, opacities, sh_a, sh_b, bg, means2d, conics, col, opac_out, ids, ranges, final_T,
         n_contrib) = ctx.saved_tensors
        n = means.shape[0]
        W, H = cfg.width, cfg.height
        tiles_x = (W + TILE_SIZE - 1) // TILE_SIZE
        tiles_y = (H + TILE_SIZE - 1) // TILE_SIZE
        dev = means.device
        s = nat.stream()
        if g_image is None:
            g_image = torch.zeros((H, W, 3), device=dev, dtype=torch.float32)
        dest = None
        if _screen_hook is not None and _screen_dest is not None and cfg.sh_mode != "colors":
            dest = _screen_dest(n, dev)
        if dest is not None:  # the compositor backward writes where the consumer wants its cotangents
            g_m2d, g_con, g_col, g_op = dest
        else:
            g_m2d = torch.empty_like(means2d)
            g_con = torch.empty_like(conics)
            g_col = torch.empty((n, 3), device=dev, dtype=torch.float32)
            g_op = torch.empty_like(opac_out)
        nat.call(
            "gs_rasterize_backward", nat.ptr(means2d), nat.ptr(conics), nat.ptr(col), 3, nat.ptr(opac_out), n,
            nat.ptr(ids), nat.ptr(ranges), nat.ptr(bg), W, H, tiles_x, tiles_y, nat.ptr(final_T), nat.ptr(n_contrib),
            nat.ptr(g_image.contiguous()), nat.ptr(None if g_final_T is None else g_final_T.contiguous()),
            nat.ptr(g_m2d), nat.ptr(g_con), nat.ptr(g_col), nat.ptr(g_op), s,
        )
        if g_means2d_out is not None:
            g_m2d += g_means2d_out
        if cfg.probe is not None:
            cfg.probe.copy_(g_m2d)
        if _screen_hook is not None and cfg.sh_mode != "colors":
            if g_depths_out is not None or g_comp_out is not None:
                raise ValueError("screen-space gradient exchange: the loss may depend on the image and alpha "
                                 "only (depths / compensation have cotangents)")
            _screen_hook(cfg, (g_m2d, g_con, g_col, g_op), (means, quats, scales, opacities, sh_a, sh_b))
            return None, None, None, None, None, None, None, None, None
        g_means = _grad_like("means", means)
        g_quats = _grad_like("quats", quats)
        g_scales = _grad_like("scales", scales)
        g_opac = _grad_like("opacities", opacities)
        use_sh = cfg.sh_mode != "colors"
        g_sh_a = g_sh_b = None
        g_dc = g_rest = None
        if use_sh:
            nb = num_sh_bases(cfg.sh_degree)
            if cfg.sh_mode == "full":
                k = sh_a.shape[1]
                g_sh_a = _grad_like("sh_a", sh_a, zero=k > nb)
                g_dc, g_rest = g_sh_a.data_ptr(), (g_sh_a.data_ptr() + 12) if k > 1 else None
            else:
                g_sh_a = _grad_like("sh_a", sh_a)
                g_dc = g_sh_a.data_ptr()
                if sh_b is not None:
                    g_sh_b = _grad_like("sh_b", sh_b, zero=sh_b.shape[1] + 1 > nb)
                    g_rest = nat.ptr(g_sh_b) if sh_b.numel() else None
        dc, dcs, rest, rests = _sh_layout(cfg, sh_a, sh_b)
        c = lambda t: None if t is None else t.contiguous()  # noqa: E731
        nat.call(
            "gs_preprocess_backward", cfg.cam, nat.ptr(means), nat.ptr(quats), nat.ptr(scales), nat.ptr(opacities),
            dc, dcs, rest, rests, cfg.sh_degree, n, cfg.blur, int(cfg.antialias), cfg.flags, nat.ptr(g_m2d),
            nat.ptr(g_con), nat.ptr(g_col) if use_sh else None, nat.ptr(g_op), nat.ptr(c(g_depths_out)),
            nat.ptr(c(g_comp_out)), nat.ptr(g_means), nat.ptr(g_quats), nat.ptr(g_scales), nat.ptr(g_opac), g_dc,
            g_rest, s,
        )
        g_colors = None if use_sh else g_col
        return g_means, g_quats, g_scales, g_opac, g_sh_a, g_sh_b, g_colors, None, None


# Optional destination of the next backward's parameter gradients: a
# callable (name, like) -> tensor shaped like `like` (or None for a fresh
# one); names are "means", "quats", "scales", "opacities", "sh_a", "sh_b".
# mlx3d_b200.distributed.GradientReducer installs one for the duration of a
# backward so the gradients are written straight into its flat all-reduce
# buffer.  A module global, not thread-local: autograd runs CUDA backward
# functions on its own device thread.
_grad_sink = None


# Optional consumer of the next backward's screen-space cotangents: a
# callable (cfg, (g_means2d, g_conics, g_colors, g_opacities_out), (means,
# quats, scales, opacities, sh_a, sh_b)).  When set, the fused render's
# backward stops after the compositor backward, hands the cotangents over
# and returns no parameter gradients: the consumer (e.g.
# mlx3d_b200.distributed.ScreenGradientExchange) runs the per-Gaussian
# backward itself.  Module global for the same reason as _grad_sink.
_screen_hook = None
# With the hook, optionally: a callable (n, device) -> (g_means2d (n,2),
# g_conics (n,3), g_colors (n,3), g_opacities_out (n,)) tensors the
# compositor backward writes its cotangents into (e.g. buffers that other
# GPUs read directly), or None for fresh ones.
_screen_dest = None


_SIDE_STREAMS: dict = {}


def side_streams(count: int) -> list:
    """``count`` CUDA streams of the current device, created once and reused:
    the caching allocator keeps freed blocks per stream, so fresh streams on
    every call would never reuse memory (each call would allocate anew)."""
    dev = torch.cuda.current_device()
    have = _SIDE_STREAMS.setdefault(dev, [])
    while len(have) < count:
        have.append(torch.cuda.Stream(device=dev))
    return have[:count]


def set_screen_grad_hook(fn, dest=None) -> None:
    global _screen_hook, _screen_dest
    _screen_hook = fn
    _screen_dest = dest if fn is not None else None


def set_grad_sink(fn) -> None:
    global _grad_sink
    _grad_sink = fn


def _grad_like(name: str, like: torch.Tensor, zero: bool = False) -> torch.Tensor:
    if _grad_sink is not None:
        t = _grad_sink(name, like)
        if t is not None:
            if zero:
                t.zero_()
            return t
    return torch.zeros_like(like) if zero else torch.empty_like(like)


def _render_fused(
    camera: Camera,
    means,
    quats,
    scales,
    opacities,
    *,
    colors=None,
    sh=None,
    sh_dc=None,
    sh_rest=None,
    sh_degree: int = 3,
    background=None,
    antialias: bool = False,
    flags: int = 0,
    with_depth: bool = False,
    blur: float = 0.3,
    probe: torch.Tensor | None = None,
    refine_tiles: bool = False,
) -> dict[str, torch.Tensor]:
    means = nat.require_cuda("means", means)
    quats = nat.require_cuda("quats", quats)
    scales = nat.require_cuda("scales", scales)
    n = means.shape[0]
    if means.shape != (n, 3) or quats.shape != (n, 4) or scales.shape != (n, 3):
        raise ValueError("means (N, 3), quats (N, 4) and scales (N, 3) must agree.")
    opacities = nat.require_cuda("opacities", opacities).reshape(-1)
    if opacities.shape != (n,):
        raise ValueError("opacities must have shape (N,).")
    dev = means.device
    if background is None:
        background = torch.zeros(3, device=dev)
    background = nat.require_cuda("background", torch.as_tensor(background, device=dev)).reshape(3)
    sh_a = sh_b = None
    if colors is not None:
        colors = nat.require_cuda("colors", colors)
        if colors.shape != (n, 3):
            raise ValueError("colors must have shape (N, 3).")
        mode, degree = "colors", -1
    elif sh is not None:
        sh_a = nat.require_cuda("sh", sh)
        if sh_a.ndim != 3 or sh_a.shape[0] != n or sh_a.shape[2] != 3:
            raise ValueError("sh must have shape (N, K, 3).")
        mode, degree = "full", int(sh_degree)
        if sh_a.shape[1] < num_sh_bases(degree):
            raise ValueError(f"sh has {sh_a.shape[1]} coefficients; degree {degree} needs {num_sh_bases(degree)}.")
    else:
        sh_a = nat.require_cuda("sh_dc", sh_dc).reshape(n, 1, 3)
        sh_b = None if sh_rest is None or sh_rest.shape[1] == 0 else nat.require_cuda("sh_rest", sh_rest)
        mode, degree = "split", int(sh_degree)
        k = 1 + (0 if sh_b is None else sh_b.shape[1])
        if k < num_sh_bases(degree):
            raise ValueError(f"sh has {k} coefficients; degree {degree} needs {num_sh_bases(degree)}.")
    if not 0 <= degree <= 3 and mode != "colors":
        raise ValueError("sh_degree must be in [0, 3].")
    cfg = _RenderCfg(
        cam=camera.to_native(), width=int(camera.width), height=int(camera.height), blur=float(blur),
        antialias=bool(antialias) and blur > 0, flags=int(flags), sh_degree=degree, sh_mode=mode,
        with_depth=bool(with_depth), probe=probe, refine=bool(refine_tiles),
    )
    image, final_T, n_contrib, means2d, depths, radii, comp, depth, counts = _Render.apply(
        means, quats, scales, opacities, sh_a, sh_b, colors, background, cfg
    )
    out = {
        "image": image,
        "alpha": 1.0 - final_T,
        "final_T": final_T,
        "n_contrib": n_contrib,
        "means2d": means2d,
        "depths": depths,
        "radii": radii,
        "compensation": comp,
    }
    if depth is not None:
        out["depth"] = depth
    out["n_duplicates"] = cfg.duplicates
    out["tiles_touched"] = counts
    return out


def _check_projection(projection: str) -> None:
    if projection not in ("ewa", "ut"):
        raise ValueError("projection must be 'ewa' or 'ut'.")


def _project(camera, means, quats, scales, projection, antialias):
    """render.py:14-26."""
    _check_projection(projection)
    fn = project_gaussians if projection == "ewa" else project_gaussians_ut
    return fn(camera, means, quats, scales, antialias=antialias)


def _render_composed(camera, means, quats, scales, opacities, colors=None, sh=None, sh_degree=3, background=None,
                     antialias=False, refine_tiles=False, projection="ut", with_depth=False):
    """render_gaussians as the reference composes it (render.py:56-112), from
    the standalone kernels: used for the unscented projection, whose sigma
    points are not part of the fused per-Gaussian kernel."""
    proj = _project(camera, means, quats, scales, projection, antialias)
    opac = nat.require_cuda("opacities", opacities).reshape(-1) * proj["compensation"]
    if sh is not None:
        m = nat.require_cuda("means", means).detach()
        center = camera.camera_center.to(m.device)
        d = m - center
        d = d / torch.clamp(torch.linalg.norm(d, dim=-1, keepdim=True), min=1e-8)
        raw = eval_sh(sh_degree, sh, d)
        colors = torch.where(raw > 0, raw, torch.zeros_like(raw))
    sorted_ids, tile_ranges, tiles_x, tiles_y = bin_gaussians(
        proj["means2d"], proj["radii"], proj["depths"], camera.width, camera.height,
        conics=proj["conics"] if refine_tiles else None,
    )
    out = rasterize(proj["means2d"], proj["conics"], colors, opac, sorted_ids, tile_ranges, camera.width,
                    camera.height, tiles_x, tiles_y, background=background)
    if with_depth:
        out["depth"] = rasterize_depth(proj["means2d"], proj["conics"], opac, proj["depths"], sorted_ids,
                                       tile_ranges, camera.width, camera.height, tiles_x, tiles_y)["depth"]
    return _extras(out, proj)


def render_gaussians(
    camera: Camera,
    means: torch.Tensor,
    quats: torch.Tensor,
    scales: torch.Tensor,
    opacities: torch.Tensor,
    colors: torch.Tensor | None = None,
    sh: torch.Tensor | None = None,
    sh_degree: int = 3,
    background: torch.Tensor | None = None,
    refine_tiles: bool = False,
    antialias: bool = False,
    projection: str = "ewa",
    render_depth: bool = False,
) -> dict[str, torch.Tensor]:
    """Render 3D Gaussians from a camera, differentiable end to end (render.py:29-112).

    ``scales`` are linear standard deviations and ``opacities`` in [0, 1]
    (activations applied by the caller), exactly one of ``colors`` (N, 3) or
    ``sh`` (N, K, 3).  Returns ``image`` (H, W, 3), ``alpha``, ``final_T``,
    ``n_contrib`` and the projection outputs ``means2d``, ``depths``,
    ``radii``, ``compensation``.  ``render_depth=True`` (an addition to the
    reference API) also composites the expected depth in the same pass.
    """
    if (colors is None) == (sh is None):
        raise ValueError("Provide exactly one of `colors` or `sh`.")
    _check_projection(projection)
    if projection == "ut":
        return _render_composed(camera, means, quats, scales, opacities, colors=colors, sh=sh, sh_degree=sh_degree,
                                background=background, antialias=antialias, refine_tiles=refine_tiles,
                                with_depth=render_depth)
    return _render_fused(
        camera, means, quats, scales, opacities, colors=colors, sh=sh, sh_degree=sh_degree, background=background,
        antialias=antialias, with_depth=render_depth, refine_tiles=refine_tiles,
    )


def _project_and_bin(camera, means, quats, scales, opacities, refine_tiles, antialias, projection):
    proj = _project(camera, means, quats, scales, projection, antialias)
    opac = nat.require_cuda("opacities", opacities).reshape(-1) * proj["compensation"]
    sorted_ids, tile_ranges, tiles_x, tiles_y = bin_gaussians(
        proj["means2d"], proj["radii"], proj["depths"], camera.width, camera.height,
        conics=proj["conics"] if refine_tiles else None,
    )
    return proj, opac, sorted_ids, tile_ranges, tiles_x, tiles_y


def _extras(out, proj):
    out.update({k: proj[k] for k in ("means2d", "depths", "radii", "compensation")})
    return out


def render_gaussian_depth(
    camera: Camera,
    means: torch.Tensor,
    quats: torch.Tensor,
    scales: torch.Tensor,
    opacities: torch.Tensor,
    refine_tiles: bool = False,
    antialias: bool = False,
    projection: str = "ewa",
) -> dict[str, torch.Tensor]:
    """Expected depth and alpha, forward only (render.py:115-161)."""
    proj, opac, ids, ranges, tx, ty = _project_and_bin(
        camera, means, quats, scales, opacities, refine_tiles, antialias, projection
    )
    out = rasterize_depth(proj["means2d"], proj["conics"], opac, proj["depths"], ids, ranges, camera.width,
                          camera.height, tx, ty)
    return _extras(out, proj)


def render_gaussian_features(
    camera: Camera,
    means: torch.Tensor,
    quats: torch.Tensor,
    scales: torch.Tensor,
    opacities: torch.Tensor,
    features: torch.Tensor,
    background: torch.Tensor | float | None = None,
    normalize: bool = False,
    refine_tiles: bool = False,
    antialias: bool = False,
    projection: str = "ewa",
) -> dict[str, torch.Tensor]:
    """Composite arbitrary (N, C) features (render.py:164-220)."""
    if features.ndim != 2:
        raise ValueError("features must have shape (N, C).")
    if features.shape[0] != means.shape[0]:
        raise ValueError("features and means2d must have the same first dimension.")
    proj, opac, ids, ranges, tx, ty = _project_and_bin(
        camera, means, quats, scales, opacities, refine_tiles, antialias, projection
    )
    out = rasterize_features(proj["means2d"], proj["conics"], features, opac, ids, ranges, camera.width,
                             camera.height, tx, ty, background=background, normalize=normalize)
    return _extras(out, proj)
