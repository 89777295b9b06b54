"""Tile binning (src/mlx3d/splatting/tiles.py:19-182) on the sm_100a kernels.

Same outputs as the reference: ``sorted_ids`` (D,) int32 Gaussian ids in
(tile, depth) render order and ``tile_ranges`` (tiles, 2) int32 [start, end)
with empty tiles at [0, 0).  Like the reference (tiles.py:68), the duplicate
total D is read back to the host once per call to size the outputs.
"""

from __future__ import annotations

import ctypes
import threading

import torch

from .. import _native as nat

TILE_SIZE = 16

__all__ = ["TILE_SIZE", "bin_gaussians", "bin_with_counts", "check_pending_status"]

_PINNED: dict = {}
# (thread, device) -> (event, pinned status word) of the previous binning
# whose status was copied to the host without waiting for it.
_PENDING: dict = {}


def _pinned_d() -> torch.Tensor:
    """A pinned host int64 for the duplicate count (one per thread and device)."""
    key = (threading.get_ident(), torch.cuda.current_device())
    t = _PINNED.get(key)
    if t is None:
        t = torch.empty((1,), dtype=torch.int64).pin_memory()
        _PINNED[key] = t
    return t


def _raise_status(v: int) -> None:
    raise RuntimeError(
        f"binning: a bounded device wait gave up (status 0x{v:x}); every tile range was left empty, so the "
        "frame rendered no Gaussians"
    )


def check_pending_status() -> None:
    """Raise if a binning on this thread and device, whose status was copied
    to the host without waiting, reported a device wait that gave up.  Status
    copies that have not completed yet are left for a later check."""
    key = (threading.get_ident(), torch.cuda.current_device())
    pend = _PENDING.get(key)
    if pend is None or not pend[0].query():
        return
    del _PENDING[key]
    v = int(pend[1][0])
    if v:
        _raise_status(v)


def bin_with_counts(
    means2d: torch.Tensor,
    radii: torch.Tensor,
    depths: torch.Tensor,
    tiles_touched: torch.Tensor,
    width: int,
    height: int,
    conics: torch.Tensor | None = None,
    check: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Depth order, duplicates, tile sort and ranges, given per-Gaussian tile
    counts already computed (by the fused preprocess kernel, gs_tile_counts, or
    gs_tile_counts_refined when ``conics`` is given for the tile refinement).

    The binning's look-backs are bounded device waits; one that gives up
    leaves every tile range empty and sets a status word.  With ``check`` the
    status is read synchronously and a failure raises ``RuntimeError`` here;
    otherwise it is copied to the host asynchronously and raised by the next
    binning call on this thread and device (whose own synchronisation on D
    comes after it), or by ``check_pending_status``."""
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
    check_pending_status()
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
    if n == 0:
        return sorted_ids, tile_ranges
    off = lib.gs_bin_status_offset(n)
    if check:
        st = ctypes.c_uint32(0)
        status = lib.gs_bin_status(nat.ptr(ws_n), ws_n.numel(), n, ctypes.byref(st), s)
        if status == nat.GS_ERR_TIMEOUT:
            _raise_status(st.value)
        if status != nat.GS_OK:
            raise RuntimeError(f"gs_bin_status failed (status {status}): {lib.gs_last_error().decode()}")
    else:
        flag = torch.empty((1,), dtype=torch.int32, pin_memory=True)
        flag.copy_(ws_n[off:off + 4].view(torch.int32), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        _PENDING[(threading.get_ident(), torch.cuda.current_device())] = (ev, flag)
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
    sorted_ids, tile_ranges = bin_with_counts(means2d, radii, depths, counts, width, height, conics, check=True)
    return sorted_ids, tile_ranges, tiles_x, tiles_y
