"""Tile binning (src/mlx3d/splatting/tiles.py:19-182) on the sm_100a kernels.

Same outputs as the reference: ``sorted_ids`` (D,) int32 Gaussian ids in
(tile, depth) render order and ``tile_ranges`` (tiles, 2) int32 [start, end)
with empty tiles at [0, 0).  Like the reference (tiles.py:68), the duplicate
total D is read back to the host once per call to size the outputs.
"""

from __future__ import annotations

import threading

import torch

from .. import _native as nat

TILE_SIZE = 16

__all__ = ["TILE_SIZE", "bin_gaussians", "bin_with_counts"]

_PINNED: dict = {}


def _pinned_d() -> torch.Tensor:
    """A pinned host int64 for the duplicate count (one per thread and device)."""
    key = (threading.get_ident(), torch.cuda.current_device())
    t = _PINNED.get(key)
    if t is None:
        t = torch.empty((1,), dtype=torch.int64).pin_memory()
        _PINNED[key] = t
    return t


def bin_with_counts(
    means2d: torch.Tensor,
    radii: torch.Tensor,
    depths: torch.Tensor,
    tiles_touched: torch.Tensor,
    width: int,
    height: int,
    conics: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Depth order, duplicates, tile sort and ranges, given per-Gaussian tile
    counts already computed (by the fused preprocess kernel, gs_tile_counts, or
    gs_tile_counts_refined when ``conics`` is given for the tile refinement)."""
    n = means2d.shape[0]
    dev = means2d.device
    tiles_x = (width + TILE_SIZE - 1) // TILE_SIZE
    tiles_y = (height + TILE_SIZE - 1) // TILE_SIZE
    lib = nat.load()
    s = nat.stream()
    ws_n = torch.empty((max(1, lib.gs_bin_workspace_n_bytes(n)),), device=dev, dtype=torch.uint8)
    d_total = torch.empty((2,), device=dev, dtype=torch.int64)
    # D first (it does not depend on the depth order): its copy to the host
    # overlaps the depth sort, so the host sizes the D buffers and queues the
    # rest of the frame while the GPU is still sorting.
    nat.call("gs_bin_total", nat.ptr(tiles_touched), n, nat.ptr(d_total), s)
    d_host = _pinned_d()
    d_host.copy_(d_total[:1], non_blocking=True)
    ready = torch.cuda.Event()
    ready.record()
    nat.call("gs_bin_begin", nat.ptr(depths), nat.ptr(tiles_touched), n, nat.ptr(ws_n), ws_n.numel(),
             nat.ptr(d_total[1:]), s)
    ready.synchronize()
    d = int(d_host[0])
    ws_d = torch.empty((max(1, lib.gs_bin_workspace_d_bytes(d)),), device=dev, dtype=torch.uint8)
    sorted_ids = torch.empty((d,), device=dev, dtype=torch.int32)
    tile_ranges = torch.empty((tiles_x * tiles_y, 2), device=dev, dtype=torch.int32)
    if conics is None:
        nat.call(
            "gs_bin_end", nat.ptr(means2d), nat.ptr(radii), n, d, width, height, nat.ptr(ws_n), ws_n.numel(),
            nat.ptr(ws_d), ws_d.numel(), nat.ptr(sorted_ids) if d else None, nat.ptr(tile_ranges), s,
        )
    else:
        nat.call(
            "gs_bin_end_refined", nat.ptr(means2d), nat.ptr(radii), nat.ptr(conics), n, d, width, height,
            nat.ptr(ws_n), ws_n.numel(), nat.ptr(ws_d), ws_d.numel(), nat.ptr(sorted_ids) if d else None,
            nat.ptr(tile_ranges), s,
        )
    return sorted_ids, tile_ranges


def bin_gaussians(
    means2d: torch.Tensor,
    radii: torch.Tensor,
    depths: torch.Tensor,
    width: int,
    height: int,
    conics: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, int, int]:
    """Assign Gaussians to 16x16 tiles and sort by (tile, depth) (tiles.py:19-182).

    Returns ``(sorted_ids, tile_ranges, tiles_x, tiles_y)``.  With ``conics``
    (N, 3), duplicates whose tile rectangle cannot reach the Gaussian's
    conic distance 12 are dropped (tiles.py:91-164).  No gradients flow
    through binning (the reference stop-gradients its inputs).
    """
    means2d = nat.require_cuda("means2d", means2d.detach())
    radii = nat.require_cuda("radii", radii.detach())
    depths = nat.require_cuda("depths", depths.detach())
    n = means2d.shape[0]
    if means2d.shape != (n, 2) or radii.shape != (n,) or depths.shape != (n,):
        raise ValueError("means2d must be (N, 2); radii and depths (N,).")
    tiles_x = (width + TILE_SIZE - 1) // TILE_SIZE
    tiles_y = (height + TILE_SIZE - 1) // TILE_SIZE
    counts = torch.empty((n,), device=means2d.device, dtype=torch.int32)
    if conics is None:
        nat.call("gs_tile_counts", nat.ptr(means2d), nat.ptr(radii), n, width, height, nat.ptr(counts),
                 nat.stream())
    else:
        conics = nat.require_cuda("conics", conics.detach())
        if conics.shape != (n, 3):
            raise ValueError("conics must have shape (N, 3).")
        nat.call("gs_tile_counts_refined", nat.ptr(means2d), nat.ptr(radii), nat.ptr(conics), n, width, height,
                 nat.ptr(counts), nat.stream())
    sorted_ids, tile_ranges = bin_with_counts(means2d, radii, depths, counts, width, height, conics)
    return sorted_ids, tile_ranges, tiles_x, tiles_y
