"""EWA projection of 3D Gaussians (src/mlx3d/splatting/projection.py:24-146).

Forward and backward are the sm_100a kernels behind ``gs_project_forward`` /
``gs_project_backward``; the backward applies MLX's autodiff conventions for
``maximum`` / ``clip`` / ``where`` (gradient to the first argument only where
it is strictly larger / strictly inside the bounds).
"""

from __future__ import annotations

import torch

from .. import _native as nat
from ..cameras import Camera

__all__ = ["project_gaussians", "project_gaussians_ut", "quat_scale_to_cov3d"]


def _check_gaussians(means, quats, scales):
    if means.ndim != 2 or means.shape[1] != 3:
        raise ValueError("means must have shape (N, 3).")
    n = means.shape[0]
    if quats.shape != (n, 4):
        raise ValueError("quats must have shape (N, 4).")
    if scales.shape != (n, 3):
        raise ValueError("scales must have shape (N, 3).")


class _Project(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, cam_native, blur, antialias):
        n = means.shape[0]
        dev = means.device
        means2d = torch.empty((n, 2), device=dev, dtype=torch.float32)
        conics = torch.empty((n, 3), device=dev, dtype=torch.float32)
        depths = torch.empty((n,), device=dev, dtype=torch.float32)
        radii = torch.empty((n,), device=dev, dtype=torch.float32)
        comp = torch.empty((n,), device=dev, dtype=torch.float32)
        nat.call(
            "gs_project_forward", cam_native, nat.ptr(means), nat.ptr(quats), nat.ptr(scales), n, blur,
            int(antialias), nat.ptr(means2d), nat.ptr(conics), nat.ptr(depths), nat.ptr(radii), nat.ptr(comp),
            nat.stream(),
        )
        ctx.save_for_backward(means, quats, scales)
        ctx.cam, ctx.blur, ctx.aa = cam_native, blur, antialias
        ctx.mark_non_differentiable(radii)
        ctx.set_materialize_grads(False)
        return means2d, conics, depths, radii, comp

    @staticmethod
    def backward(ctx, g_means2d, g_conics, g_depths, _g_radii, g_comp):
        means, quats, scales = ctx.saved_tensors
        n = means.shape[0]
        g_means = torch.empty_like(means)
        g_quats = torch.empty_like(quats)
        g_scales = torch.empty_like(scales)
        c = lambda t: None if t is None else t.contiguous()  # noqa: E731
        g_means2d, g_conics, g_depths, g_comp = c(g_means2d), c(g_conics), c(g_depths), c(g_comp)
        nat.call(
            "gs_project_backward", ctx.cam, nat.ptr(means), nat.ptr(quats), nat.ptr(scales), n, ctx.blur,
            int(ctx.aa), nat.ptr(g_means2d), nat.ptr(g_conics), nat.ptr(g_depths), nat.ptr(g_comp),
            nat.ptr(g_means), nat.ptr(g_quats), nat.ptr(g_scales), nat.stream(),
        )
        return g_means, g_quats, g_scales, None, None, None


def project_gaussians(
    camera: Camera,
    means: torch.Tensor,
    quats: torch.Tensor,
    scales: torch.Tensor,
    blur: float = 0.3,
    antialias: bool = False,
) -> dict[str, torch.Tensor]:
    """Project 3D Gaussians to screen space (projection.py:24-146).

    Returns a dict with ``means2d`` (N, 2), ``conics`` (N, 3) upper-triangular
    inverse 2D covariance, ``depths`` (N,) camera-space z, ``radii`` (N,)
    float pixel radii (0 = culled) and ``compensation`` (N,) (ones unless
    ``antialias``).  Differentiable in means, quats and scales.
    """
    means = nat.require_cuda("means", means)
    quats = nat.require_cuda("quats", quats)
    scales = nat.require_cuda("scales", scales)
    _check_gaussians(means, quats, scales)
    means2d, conics, depths, radii, comp = _Project.apply(
        means, quats, scales, camera.to_native(), float(blur), bool(antialias) and blur > 0
    )
    return {"means2d": means2d, "conics": conics, "depths": depths, "radii": radii, "compensation": comp}


class _ProjectUT(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, quats, scales, cam_native, lens, blur, antialias):
        n = means.shape[0]
        f32 = dict(device=means.device, dtype=torch.float32)
        means2d, conics = torch.empty((n, 2), **f32), torch.empty((n, 3), **f32)
        depths, radii, comp = torch.empty((n,), **f32), torch.empty((n,), **f32), torch.empty((n,), **f32)
        nat.call("gs_project_ut_forward", cam_native, lens, nat.ptr(means), nat.ptr(quats), nat.ptr(scales), n, blur,
                 int(antialias), nat.ptr(means2d), nat.ptr(conics), nat.ptr(depths), nat.ptr(radii), nat.ptr(comp),
                 nat.stream())
        ctx.save_for_backward(means, quats, scales)
        ctx.args = (cam_native, lens, blur, antialias)
        ctx.mark_non_differentiable(radii)
        ctx.set_materialize_grads(False)
        return means2d, conics, depths, radii, comp

    @staticmethod
    def backward(ctx, g_means2d, g_conics, g_depths, _g_radii, g_comp):
        means, quats, scales = ctx.saved_tensors
        cam_native, lens, blur, antialias = ctx.args
        g_means, g_quats, g_scales = torch.empty_like(means), torch.empty_like(quats), torch.empty_like(scales)
        c = lambda t: None if t is None else t.contiguous()  # noqa: E731
        nat.call("gs_project_ut_backward", cam_native, lens, nat.ptr(means), nat.ptr(quats), nat.ptr(scales),
                 means.shape[0], blur, int(antialias), nat.ptr(c(g_means2d)), nat.ptr(c(g_conics)),
                 nat.ptr(c(g_depths)), nat.ptr(c(g_comp)), nat.ptr(g_means), nat.ptr(g_quats), nat.ptr(g_scales),
                 nat.stream())
        return g_means, g_quats, g_scales, None, None, None, None


def project_gaussians_ut(
    camera: Camera,
    means: torch.Tensor,
    quats: torch.Tensor,
    scales: torch.Tensor,
    blur: float = 0.3,
    antialias: bool = False,
) -> dict[str, torch.Tensor]:
    """3DGUT-style unscented projection (projection.py:149-205): six sigma
    points through the camera's own model (``orthographic``, Brown-Conrady
    or fisheye ``distortion``).  Same outputs as :func:`project_gaussians`,
    differentiable in means, quats and scales."""
    means = nat.require_cuda("means", means)
    quats = nat.require_cuda("quats", quats)
    scales = nat.require_cuda("scales", scales)
    _check_gaussians(means, quats, scales)
    means2d, conics, depths, radii, comp = _ProjectUT.apply(
        means, quats, scales, camera.to_native(), camera.lens_native(), float(blur), bool(antialias) and blur > 0
    )
    return {"means2d": means2d, "conics": conics, "depths": depths, "radii": radii, "compensation": comp}


def quat_to_rotmat(quats: torch.Tensor) -> torch.Tensor:
    """Rotation matrices of (normalised) wxyz quaternions, (..., 3, 3); host
    utility with torch ops (transforms.quaternion_to_matrix)."""
    q = quats / torch.linalg.norm(quats, dim=-1, keepdim=True)
    w, x, y, z = q.unbind(-1)
    return torch.stack(
        [
            1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
            2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
            2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
        ],
        dim=-1,
    ).reshape(*quats.shape[:-1], 3, 3)


def quat_scale_to_cov3d(quats: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """3D covariances ``R S S^T R^T`` (projection.py:17-21); a small host-side
    utility (not on the rendering path), computed with torch ops."""
    R = quat_to_rotmat(quats)
    M = R * scales[..., None, :]
    return M @ M.transpose(-1, -2)
