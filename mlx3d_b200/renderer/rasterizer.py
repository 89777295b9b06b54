"""Hard z-buffer mesh rasterizer (src/mlx3d/renderer/rasterizer.py).

Visibility — the nearest triangle per pixel — is resolved by the sm_100a
kernel behind ``gs_mesh_rasterize`` over the triangles the Gaussian tiler
bins to each 16x16 tile (bounding circle around the screen-space centroid,
ordered by mean depth), exactly like the reference's Metal kernel.  The
barycentric coordinates of the hit are then recomputed with differentiable
torch operations, so gradients reach vertex positions (and, through
:func:`interpolate_face_attributes`, per-vertex attributes) without a
backward kernel.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native as nat
from ..cameras import Camera
from ..splatting.tiles import bin_gaussians

__all__ = ["Fragments", "rasterize_meshes", "interpolate_face_attributes"]

_EPS = 1e-12


@dataclass
class Fragments:
    """Per-pixel rasterizer output (rasterizer.py:84-101).

    ``pix_to_face`` (H, W) int32 nearest face or -1; ``zbuf`` (H, W) its
    camera-space depth (0 where empty); ``bary`` (H, W, 3) barycentrics of the
    hit (differentiable in the vertices, 0 where empty); ``valid`` (H, W)
    covered mask; ``vert_ids`` (H, W, 3) vertex indices of the hit face."""

    pix_to_face: torch.Tensor
    zbuf: torch.Tensor
    bary: torch.Tensor
    valid: torch.Tensor
    vert_ids: torch.Tensor


def _as_verts_faces(mesh_or_verts, faces):
    """(verts, faces) from a one-mesh container with verts_packed() /
    faces_packed(), or from a raw (V, 3) vertex tensor and (F, 3) faces
    (rasterizer.py:109-117)."""
    if hasattr(mesh_or_verts, "verts_packed") and hasattr(mesh_or_verts, "faces_packed"):
        if len(mesh_or_verts) != 1:
            raise ValueError("rasterize_meshes renders one mesh at a time.")
        return mesh_or_verts.verts_packed(), mesh_or_verts.faces_packed()
    if faces is None:
        raise ValueError("faces must be provided when verts are passed directly.")
    return mesh_or_verts, faces


def rasterize_meshes(camera: Camera, mesh_or_verts, faces: torch.Tensor | None = None) -> Fragments:
    """Rasterize one triangle mesh (rasterizer.py:120-196)."""
    verts, faces_idx = _as_verts_faces(mesh_or_verts, faces)
    verts = nat.require_cuda("verts", verts)
    if not isinstance(faces_idx, torch.Tensor):
        faces_idx = torch.as_tensor(faces_idx)
    faces_idx = faces_idx.to(device=verts.device, dtype=torch.long)
    if faces_idx.ndim != 2 or faces_idx.shape[-1] != 3:
        raise ValueError("faces must have shape (F, 3).")
    h, w = int(camera.height), int(camera.width)

    xy, z = camera.project_points(verts)  # (V, 2), (V,)
    tri_xy = xy[faces_idx]  # (F, 3, 2)
    tri_z = z[faces_idx]  # (F, 3)

    # Bin faces into tiles by their bounding circles with the Gaussian tiler.
    sxy = tri_xy.detach()
    centroid = sxy.mean(dim=1)
    radii = torch.sqrt(((sxy - centroid[:, None, :]) ** 2).sum(dim=-1).max(dim=1).values)
    depths = tri_z.detach().mean(dim=1)
    sorted_ids, tile_ranges, _, _ = bin_gaussians(centroid.contiguous(), radii.contiguous(), depths.contiguous(), w, h)

    pix_to_face = torch.empty((h, w), device=verts.device, dtype=torch.int32)
    zbuf = torch.empty((h, w), device=verts.device, dtype=torch.float32)
    nf = int(faces_idx.shape[0])
    nat.call("gs_mesh_rasterize", nat.ptr(sxy.contiguous()), nat.ptr(tri_z.detach().contiguous()), nf,
             nat.ptr(sorted_ids), nat.ptr(tile_ranges), w, h, float(camera.znear),
             nat.ptr(pix_to_face), nat.ptr(zbuf), nat.stream())

    valid = pix_to_face >= 0
    fidx = torch.where(valid, pix_to_face, torch.zeros_like(pix_to_face)).long()
    vert_ids = faces_idx[fidx] if nf else torch.zeros((h, w, 3), device=verts.device, dtype=torch.long)
    if nf:
        # Barycentrics recomputed with differentiable operations (rasterizer.py:171-185).
        tri = xy[vert_ids]  # (H, W, 3, 2)
        ax, ay = tri[..., 0, 0], tri[..., 0, 1]
        bx, by = tri[..., 1, 0], tri[..., 1, 1]
        cxv, cyv = tri[..., 2, 0], tri[..., 2, 1]
        px = (torch.arange(w, device=verts.device, dtype=torch.float32) + 0.5)[None, :]
        py = (torch.arange(h, device=verts.device, dtype=torch.float32) + 0.5)[:, None]
        denom = (by - cyv) * (ax - cxv) + (cxv - bx) * (ay - cyv)
        denom = torch.where(denom.abs() < _EPS, torch.ones_like(denom), denom)
        l0 = ((by - cyv) * (px - cxv) + (cxv - bx) * (py - cyv)) / denom
        l1 = ((cyv - ay) * (px - cxv) + (ax - cxv) * (py - cyv)) / denom
        l2 = 1.0 - l0 - l1
        bary = torch.stack([l0, l1, l2], dim=-1) * valid[..., None]
    else:
        bary = torch.zeros((h, w, 3), device=verts.device, dtype=torch.float32)
    return Fragments(pix_to_face=pix_to_face, zbuf=zbuf, bary=bary, valid=valid, vert_ids=vert_ids)


def interpolate_face_attributes(frag: Fragments, attrs: torch.Tensor) -> torch.Tensor:
    """(H, W, C) barycentric interpolation of per-vertex ``attrs`` (V, C),
    0 on empty pixels (rasterizer.py:199-210); differentiable in ``attrs``
    and, through the barycentrics, in the vertex positions."""
    tri_attr = attrs[frag.vert_ids]  # (H, W, 3, C)
    out = (frag.bary[..., None] * tri_attr).sum(dim=-2)
    return out * frag.valid[..., None]
