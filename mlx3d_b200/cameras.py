"""Pinhole cameras with mlx3D's conventions (src/mlx3d/cameras/cameras.py).

OpenCV / COLMAP frame: +x right, +y down, +z forward; ``X_cam = R @ X_world + t``;
``u = fx * x/z + cx``.  ``R`` and ``t`` are float32 torch tensors; the
intrinsics are Python floats, exactly as in the reference, and
:meth:`Camera.to_native` rounds them to the float32 values the reference's
mixed Python-float / float32-array expressions end up using.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ._native import GsCamera, GsLens

__all__ = ["Camera", "look_at", "look_at_view_transform", "fov_to_focal", "focal_to_fov"]


def fov_to_focal(fov: float, pixels: int) -> float:
    """Focal length in pixels from a field of view in radians (cameras.py:32-34)."""
    return pixels / (2.0 * math.tan(fov / 2.0))


def focal_to_fov(focal: float, pixels: int) -> float:
    """Field of view in radians from a focal length in pixels (cameras.py:37-39)."""
    return 2.0 * math.atan(pixels / (2.0 * focal))


def _as_f32_cpu(v) -> torch.Tensor:
    if isinstance(v, torch.Tensor):
        return v.detach().to(device="cpu", dtype=torch.float32)
    return torch.tensor(v, dtype=torch.float32)


def look_at(eye, at, up) -> tuple[torch.Tensor, torch.Tensor]:
    """OpenCV-convention extrinsics ``(R, t)`` for a camera at ``eye`` looking
    at ``at`` (cameras.py:94-113), computed in float32 on the host."""
    eye, at, up = _as_f32_cpu(eye), _as_f32_cpu(at), _as_f32_cpu(up)
    z = at - eye
    z = z / torch.linalg.norm(z)
    x = torch.linalg.cross(z, up)
    x = x / torch.linalg.norm(x)
    y = torch.linalg.cross(z, x)
    R = torch.stack([x, y, z], dim=0)
    t = -(R @ eye)
    return R, t


def look_at_view_transform(dist=1.0, elev=0.0, azim=0.0, at=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0), degrees=True):
    """Extrinsics for a camera on a sphere around ``at`` (cameras.py:116-136)."""
    if degrees:
        elev = math.radians(elev)
        azim = math.radians(azim)
    x = dist * math.cos(elev) * math.sin(azim)
    y = dist * math.sin(elev)
    z = dist * math.cos(elev) * math.cos(azim)
    eye = [at[0] + x, at[1] + y, at[2] + z]
    return look_at(eye, at, up)


@dataclass
class Camera:
    """A single camera (cameras.py:139-173).  ``orthographic``, ``distortion``
    (Brown-Conrady (k1, k2, p1, p2[, k3]) or, with ``fisheye``, OpenCV fisheye
    (k1, k2, k3, k4)) are honoured by the unscented projection
    (``projection="ut"``); the EWA projection is pinhole, as in the reference."""

    R: torch.Tensor
    t: torch.Tensor
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int
    znear: float = 0.01
    zfar: float = 100.0
    orthographic: bool = False
    distortion: tuple | None = None
    fisheye: bool = False

    @classmethod
    def from_fov(cls, fov: float, width: int, height: int, R=None, t=None, degrees: bool = True, **kw) -> "Camera":
        """Camera from a vertical field of view (cameras.py:209-239)."""
        if degrees:
            fov = math.radians(fov)
        f = fov_to_focal(fov, height)
        R = torch.eye(3) if R is None else _as_f32_cpu(R)
        t = torch.zeros(3) if t is None else _as_f32_cpu(t)
        return cls(R=R, t=t, fx=f, fy=f, cx=width / 2.0, cy=height / 2.0, width=width, height=height, **kw)

    @classmethod
    def look_at(cls, eye, at=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0), fov: float = 60.0, width: int = 512,
                height: int = 512, degrees: bool = True, **kw) -> "Camera":
        """Camera at ``eye`` looking at ``at`` (cameras.py:241-255)."""
        R, t = look_at(eye, at, up)
        return cls.from_fov(fov, width, height, R=R, t=t, degrees=degrees, **kw)

    @property
    def K(self) -> torch.Tensor:
        return torch.tensor([[self.fx, 0.0, self.cx], [0.0, self.fy, self.cy], [0.0, 0.0, 1.0]])

    @property
    def camera_center(self) -> torch.Tensor:
        """(3,) camera position in world coordinates, ``-R^T t`` (cameras.py:270-273)."""
        R = _as_f32_cpu(self.R)
        t = _as_f32_cpu(self.t)
        return -(R.T @ t)

    def world_to_camera(self, points: torch.Tensor) -> torch.Tensor:
        return points @ self.R.to(points).T + self.t.to(points)

    def camera_to_world(self, points: torch.Tensor) -> torch.Tensor:
        """Camera-frame points back to world coordinates (cameras.py:285-287)."""
        return (points - self.t.to(points)) @ self.R.to(points)

    def project_points(self, points: torch.Tensor, eps: float = 1e-8) -> tuple[torch.Tensor, torch.Tensor]:
        """World points (..., 3) to pixel coordinates (..., 2) and camera-frame
        depth (...,) (cameras.py:289-308): pinhole (or orthographic) with the
        camera's lens distortion; differentiable torch operations (a host-side
        utility, e.g. for the mesh rasterizer's vertices)."""
        pc = self.world_to_camera(points)
        z = pc[..., 2]
        if self.orthographic:
            return torch.stack([self.fx * pc[..., 0] + self.cx, self.fy * pc[..., 1] + self.cy], dim=-1), z
        inv_z = 1.0 / torch.where(z.abs() < eps, torch.full_like(z, eps), z)
        x, y = pc[..., 0] * inv_z, pc[..., 1] * inv_z
        x, y = self._distort(x, y)
        return torch.stack([self.fx * x + self.cx, self.fy * y + self.cy], dim=-1), z

    def _distort(self, x: torch.Tensor, y: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Lens distortion of normalised coordinates (cameras.py:42-76)."""
        c = self.distortion
        if c is None:
            return x, y
        if self.fisheye:
            k1, k2, k3, k4 = (list(c) + [0.0, 0.0, 0.0, 0.0])[:4]
            r = torch.sqrt(x * x + y * y)
            th = torch.atan(r)
            th2 = th * th
            thd = th * (1.0 + th2 * (k1 + th2 * (k2 + th2 * (k3 + th2 * k4))))
            sc = thd / torch.clamp(r, min=1e-9)
            return x * sc, y * sc
        k1, k2, p1, p2 = c[0], c[1], c[2], c[3]
        k3 = c[4] if len(c) > 4 else 0.0
        r2 = x * x + y * y
        radial = 1.0 + r2 * (k1 + r2 * (k2 + r2 * k3))
        return (x * radial + 2.0 * p1 * x * y + p2 * (r2 + 2.0 * x * x),
                y * radial + p1 * (r2 + 2.0 * y * y) + 2.0 * p2 * x * y)

    def _undistort(self, x: torch.Tensor, y: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Inverse lens distortion by eight fixed-point iterations
        (cameras.py:53-66 Brown-Conrady, :79-91 fisheye); identity without
        distortion."""
        c = self.distortion
        if c is None:
            return x, y
        if self.fisheye:
            k1, k2, k3, k4 = (list(c) + [0.0, 0.0, 0.0, 0.0])[:4]
            thd = torch.sqrt(x * x + y * y)
            th = thd
            for _ in range(8):
                th2 = th * th
                th = thd / (1.0 + th2 * (k1 + th2 * (k2 + th2 * (k3 + th2 * k4))))
            sc = torch.tan(th) / torch.clamp(thd, min=1e-9)
            return x * sc, y * sc
        k1, k2, p1, p2 = c[0], c[1], c[2], c[3]
        k3 = c[4] if len(c) > 4 else 0.0
        xu, yu = x, y
        for _ in range(8):
            r2 = xu * xu + yu * yu
            radial = 1.0 + r2 * (k1 + r2 * (k2 + r2 * k3))
            dx = 2.0 * p1 * xu * yu + p2 * (r2 + 2.0 * xu * xu)
            dy = p1 * (r2 + 2.0 * yu * yu) + 2.0 * p2 * xu * yu
            xu = (x - dx) / radial
            yu = (y - dy) / radial
        return xu, yu

    def unproject_points(self, xy: torch.Tensor, depth: torch.Tensor) -> torch.Tensor:
        """Pixel coordinates (..., 2) with camera-frame z depths (...,) back to
        world points (..., 3) (cameras.py:327-336); differentiable torch
        operations."""
        xd = (xy[..., 0] - self.cx) / self.fx
        yd = (xy[..., 1] - self.cy) / self.fy
        if self.orthographic:
            return self.camera_to_world(torch.stack([xd, yd, depth], dim=-1))
        x, y = self._undistort(xd, yd)
        return self.camera_to_world(torch.stack([x * depth, y * depth, depth], dim=-1))

    def lens_native(self) -> GsLens:
        """Lens model of this camera for the unscented projection."""
        lens = GsLens()
        lens.orthographic = int(bool(self.orthographic))
        lens.fisheye = int(bool(self.fisheye))
        d = tuple(self.distortion) if self.distortion is not None else ()
        if self.fisheye:
            d = (tuple(d) + (0.0, 0.0, 0.0, 0.0))[:4]
        elif d:
            if len(d) < 4:
                raise ValueError("distortion must be (k1, k2, p1, p2[, k3])")
            d = (tuple(d) + (0.0,))[:5]
        lens.n_dist = len(d) if self.distortion is not None else 0
        for i, v in enumerate(d):
            lens.dist[i] = float(v)
        return lens

    def to_native(self) -> GsCamera:
        """The float32 view of this camera the CUDA kernels consume."""
        R = _as_f32_cpu(self.R).reshape(9).tolist()
        t = _as_f32_cpu(self.t).reshape(3).tolist()
        c = self.camera_center.reshape(3).tolist()
        cam = GsCamera()
        cam.R = type(cam.R)(*R)
        cam.t = type(cam.t)(*t)
        # Python doubles as the reference uses them (projection.py:64-73,83-85,136):
        # each becomes float32 where it meets a float32 array.
        cam.fx, cam.fy = float(self.fx), float(self.fy)
        cam.cx, cam.cy = float(self.cx), float(self.cy)
        cam.neg_fx, cam.neg_fy = -float(self.fx), -float(self.fy)
        tan_fov_x = 0.5 * self.width / self.fx
        tan_fov_y = 0.5 * self.height / self.fy
        cam.clip_x = 1.3 * tan_fov_x
        cam.clip_y = 1.3 * tan_fov_y
        cam.znear = float(self.znear)
        cam.center = type(cam.center)(*c)
        cam.width, cam.height = int(self.width), int(self.height)
        return cam
