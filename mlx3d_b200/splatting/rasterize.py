"""Tile compositing on the sm_100a kernels (src/mlx3d/splatting/rasterize.py).

``rasterize`` / ``rasterize_features`` are differentiable in means2d, conics,
colours (features) and opacities through ``gs_rasterize_backward``, the
counterpart of the reference's ``_rasterize_core`` custom function and its
vjp (rasterize.py:345-403).  ``rasterize_depth`` is forward-only, as in the
reference.  Feature rendering composites all C channels in one pass (the
reference loops over chunks of three; channels are independent, so the
values are the same).
"""

from __future__ import annotations

import torch

from .. import _native as nat

__all__ = ["rasterize", "rasterize_depth", "rasterize_features"]


class _Rasterize(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2d, conics, colors, opacities, background, sorted_ids, tile_ranges, dims):
        width, height, tiles_x, tiles_y = dims
        c = colors.shape[1]
        dev = means2d.device
        image = torch.empty((height, width, c), device=dev, dtype=torch.float32)
        final_T = torch.empty((height, width), device=dev, dtype=torch.float32)
        n_contrib = torch.empty((height, width), device=dev, dtype=torch.int32)
        nat.call(
            "gs_rasterize_forward", nat.ptr(means2d), nat.ptr(conics), nat.ptr(colors), c, nat.ptr(opacities), None,
            nat.ptr(sorted_ids), nat.ptr(tile_ranges), nat.ptr(background), width, height, tiles_x, tiles_y,
            nat.ptr(image), nat.ptr(final_T), nat.ptr(n_contrib), None, nat.stream(),
        )
        ctx.save_for_backward(means2d, conics, colors, opacities, background, sorted_ids, tile_ranges, final_T,
                              n_contrib)
        ctx.dims = dims
        ctx.mark_non_differentiable(n_contrib)
        ctx.set_materialize_grads(False)
        return image, final_T, n_contrib

    @staticmethod
    def backward(ctx, g_image, g_final_T, _g_n):
        means2d, conics, colors, opac, bg, ids, ranges, final_T, n_contrib = ctx.saved_tensors
        width, height, tiles_x, tiles_y = ctx.dims
        n, c = colors.shape
        if g_image is None:
            g_image = torch.zeros((height, width, c), device=means2d.device, dtype=torch.float32)
        g_m = torch.empty_like(means2d)
        g_co = torch.empty_like(conics)
        g_col = torch.empty_like(colors)
        g_op = torch.empty_like(opac)
        nat.call(
            "gs_rasterize_backward", nat.ptr(means2d), nat.ptr(conics), nat.ptr(colors), c, nat.ptr(opac), n,
            nat.ptr(ids), nat.ptr(ranges), nat.ptr(bg), width, height, tiles_x, tiles_y, nat.ptr(final_T),
            nat.ptr(n_contrib), nat.ptr(g_image.contiguous()),
            nat.ptr(None if g_final_T is None else g_final_T.contiguous()), nat.ptr(g_m), nat.ptr(g_co),
            nat.ptr(g_col), nat.ptr(g_op), nat.stream(),
        )
        return g_m, g_co, g_col, g_op, None, None, None, None


def _common(means2d, conics, opacities, sorted_ids, tile_ranges, width, height, tiles_x, tiles_y):
    means2d = nat.require_cuda("means2d", means2d)
    conics = nat.require_cuda("conics", conics)
    opacities = nat.require_cuda("opacities", opacities)
    sorted_ids = nat.require_cuda("sorted_ids", sorted_ids, torch.int32)
    tile_ranges = nat.require_cuda("tile_ranges", tile_ranges, torch.int32)
    n = means2d.shape[0]
    if means2d.shape != (n, 2) or conics.shape != (n, 3) or opacities.reshape(-1).shape != (n,):
        raise ValueError("means2d (N, 2), conics (N, 3) and opacities (N,) must agree.")
    if tile_ranges.shape != (tiles_x * tiles_y, 2):
        raise ValueError("tile_ranges must have shape (tiles_x * tiles_y, 2).")
    return means2d, conics, opacities.reshape(n), sorted_ids, tile_ranges


def rasterize(
    means2d: torch.Tensor,
    conics: torch.Tensor,
    colors: torch.Tensor,
    opacities: torch.Tensor,
    sorted_ids: torch.Tensor,
    tile_ranges: torch.Tensor,
    width: int,
    height: int,
    tiles_x: int,
    tiles_y: int,
    background: torch.Tensor | None = None,
) -> dict[str, torch.Tensor]:
    """Alpha-composite binned 2D Gaussians into an image (rasterize.py:406-446).

    Returns ``image`` (H, W, 3), ``alpha`` (H, W) = 1 - final_T, ``final_T``
    and ``n_contrib`` (H, W) int32.
    """
    means2d, conics, opacities, sorted_ids, tile_ranges = _common(
        means2d, conics, opacities, sorted_ids, tile_ranges, width, height, tiles_x, tiles_y
    )
    colors = nat.require_cuda("colors", colors)
    if colors.shape != (means2d.shape[0], 3):
        raise ValueError("colors must have shape (N, 3).")
    if background is None:
        background = torch.zeros(3, device=means2d.device)
    background = nat.require_cuda("background", torch.as_tensor(background, device=means2d.device)).reshape(3)
    image, final_T, n_contrib = _Rasterize.apply(
        means2d, conics, colors, opacities, background, sorted_ids, tile_ranges, (width, height, tiles_x, tiles_y)
    )
    return {"image": image, "alpha": 1.0 - final_T, "final_T": final_T, "n_contrib": n_contrib}


def rasterize_features(
    means2d: torch.Tensor,
    conics: torch.Tensor,
    features: torch.Tensor,
    opacities: torch.Tensor,
    sorted_ids: torch.Tensor,
    tile_ranges: torch.Tensor,
    width: int,
    height: int,
    tiles_x: int,
    tiles_y: int,
    background: torch.Tensor | float | None = None,
    normalize: bool = False,
) -> dict[str, torch.Tensor]:
    """Alpha-composite arbitrary (N, C) feature channels (rasterize.py:449-545).

    ``background`` (C,) or a scalar is ignored when ``normalize``; with
    ``normalize`` the result is ``sum_i alpha_i T_i f_i / alpha`` where
    alpha > 1e-6 and 0 elsewhere.
    """
    if features.ndim != 2:
        raise ValueError("features must have shape (N, C).")
    if features.shape[0] != means2d.shape[0]:
        raise ValueError("features and means2d must have the same first dimension.")
    channels = int(features.shape[1])
    if channels <= 0:
        raise ValueError("features must contain at least one channel.")
    means2d, conics, opacities, sorted_ids, tile_ranges = _common(
        means2d, conics, opacities, sorted_ids, tile_ranges, width, height, tiles_x, tiles_y
    )
    features = nat.require_cuda("features", features)
    dev = means2d.device
    if background is None or normalize:
        bg = torch.zeros((channels,), device=dev)
    else:
        bg = torch.as_tensor(background, dtype=torch.float32, device=dev)
        if bg.ndim == 0:
            bg = bg.expand(channels)
        if tuple(bg.shape) != (channels,):
            raise ValueError(f"background must have shape ({channels},).")
        bg = bg.contiguous()
    image, final_T, n_contrib = _Rasterize.apply(
        means2d, conics, features, opacities, bg, sorted_ids, tile_ranges, (width, height, tiles_x, tiles_y)
    )
    alpha = 1.0 - final_T
    feat = image
    if normalize:
        a = alpha[..., None]
        feat = torch.where(a > 1e-6, feat / torch.clamp(a, min=1e-6), torch.zeros_like(feat))
    return {"features": feat, "alpha": alpha, "final_T": final_T, "n_contrib": n_contrib}


def rasterize_depth(
    means2d: torch.Tensor,
    conics: torch.Tensor,
    opacities: torch.Tensor,
    depths: torch.Tensor,
    sorted_ids: torch.Tensor,
    tile_ranges: torch.Tensor,
    width: int,
    height: int,
    tiles_x: int,
    tiles_y: int,
) -> dict[str, torch.Tensor]:
    """Forward-only expected depth ``sum w_i z_i / (1 - T)`` (rasterize.py:548-578)."""
    means2d, conics, opacities, sorted_ids, tile_ranges = _common(
        means2d, conics, opacities, sorted_ids, tile_ranges, width, height, tiles_x, tiles_y
    )
    depths = nat.require_cuda("depths", depths).reshape(-1)
    dev = means2d.device
    depth = torch.empty((height, width), device=dev, dtype=torch.float32)
    final_T = torch.empty((height, width), device=dev, dtype=torch.float32)
    with torch.no_grad():
        nat.call(
            "gs_rasterize_forward", nat.ptr(means2d.detach()), nat.ptr(conics.detach()), None, 0,
            nat.ptr(opacities.detach()), nat.ptr(depths.detach()), nat.ptr(sorted_ids), nat.ptr(tile_ranges), None,
            width, height, tiles_x, tiles_y, None, nat.ptr(final_T), None, nat.ptr(depth), nat.stream(),
        )
    return {"depth": depth, "alpha": 1.0 - final_T, "final_T": final_T}
