"""The trainable Gaussian scene (src/mlx3d/splatting/model.py).

Raw parameters live in ``self.params`` as torch leaf tensors:
``means`` (N, 3), ``scales`` (N, 3) log standard deviations, ``quats`` (N, 4)
unnormalised wxyz, ``opacities`` (N,) logits, ``sh_dc`` (N, 1, 3) and
``sh_rest`` (N, K-1, 3).  :meth:`render` feeds the raw parameters to the
fused sm_100a kernels, which apply exp / sigmoid themselves and read
``sh_dc`` / ``sh_rest`` in place (no per-frame concatenation).
"""

from __future__ import annotations

import math

import torch

from .. import _native as nat
from ..cameras import Camera
from .render import _check_projection, _render_composed, _render_fused, render_gaussian_depth, render_gaussian_features
from .sh import num_sh_bases, rgb_to_sh

__all__ = ["GaussianModel"]


class GaussianModel:
    def __init__(self, params: dict[str, torch.Tensor], sh_degree: int = 3):
        self.params = params
        self.sh_degree = sh_degree
        # Active degree grows during training, starting at 0 (model.py:33).
        self.active_sh_degree = 0

    @classmethod
    def from_points(
        cls,
        points: torch.Tensor,
        colors: torch.Tensor | None = None,
        sh_degree: int = 3,
        initial_opacity: float = 0.1,
        scale_init_max_ref: int = 10_000,
        scale_init_chunk_size: int = 1024,
        scale_init_max_scale: float | None = None,
    ) -> "GaussianModel":
        """Initialise from a point cloud (model.py:36-105): isotropic scales from
        the mean squared distance to the 3 nearest neighbours (a one-off
        host-side initialisation with torch ops, not the rendering path)."""
        points = points.to(torch.float32)
        dev = points.device
        n = points.shape[0]
        if colors is None:
            colors = torch.full((n, 3), 0.5, device=dev)
        ref_count = min(n, max(1, int(scale_init_max_ref)))
        ref = points[torch.randperm(n, device=dev)[:ref_count]] if n > ref_count else points
        if ref_count <= 1:
            mean_sq = torch.full((n,), 1e-8, device=dev)
        else:
            k = min(4, ref_count)
            d_all = []
            for s in range(0, n, scale_init_chunk_size):
                d = torch.cdist(points[s : s + scale_init_chunk_size], ref) ** 2
                d_all.append(torch.topk(d, k, dim=1, largest=False).values)
            d = torch.cat(d_all)
            self_hit = d[:, 0] <= 1e-12
            nearest = torch.where(self_hit[:, None], d[:, 1:k], d[:, : k - 1])
            mean_sq = torch.clamp(nearest.mean(dim=-1), min=1e-8)
        scales = torch.log(torch.sqrt(mean_sq))[:, None].repeat(1, 3)
        if scale_init_max_scale is not None:
            scales = torch.clamp(scales, max=math.log(max(scale_init_max_scale, 1e-8)))
        quats = torch.zeros((n, 4), device=dev)
        quats[:, 0] = 1.0
        K = num_sh_bases(sh_degree)
        logit = math.log(initial_opacity / (1 - initial_opacity))
        params = {
            "means": points.clone(),
            "scales": scales,
            "quats": quats,
            "opacities": torch.full((n,), logit, device=dev),
            "sh_dc": rgb_to_sh(colors.to(dev, torch.float32))[:, None, :].contiguous(),
            "sh_rest": torch.zeros((n, K - 1, 3), device=dev),
        }
        return cls(params, sh_degree=sh_degree)

    @property
    def num_gaussians(self) -> int:
        return self.params["means"].shape[0]

    def __len__(self) -> int:
        return self.num_gaussians

    @property
    def scales_act(self) -> torch.Tensor:
        return torch.exp(self.params["scales"])

    @property
    def opacities_act(self) -> torch.Tensor:
        return torch.sigmoid(self.params["opacities"])

    @property
    def sh(self) -> torch.Tensor:
        return torch.cat([self.params["sh_dc"], self.params["sh_rest"]], dim=1)

    def render(
        self,
        camera: Camera,
        background: torch.Tensor | None = None,
        antialias: bool = False,
        projection: str = "ewa",
        render_depth: bool = False,
    ) -> dict:
        """``render_gaussians`` on this model's activated parameters
        (model.py:146-164); activations and SH gathering run inside the fused
        kernels.  ``render_depth=True`` adds an expected ``depth`` output."""
        _check_projection(projection)
        p = self.params
        if projection == "ut":
            return _render_composed(camera, p["means"], p["quats"], self.scales_act, self.opacities_act, sh=self.sh,
                                    sh_degree=self.active_sh_degree, background=background, antialias=antialias,
                                    with_depth=render_depth)
        return _render_fused(
            camera,
            p["means"],
            p["quats"],
            p["scales"],
            p["opacities"],
            sh_dc=p["sh_dc"],
            sh_rest=p["sh_rest"],
            sh_degree=self.active_sh_degree,
            background=background,
            antialias=antialias,
            flags=nat.GS_ACT_EXP_SCALES | nat.GS_ACT_SIGMOID_OPACITY,
            with_depth=render_depth,
        )

    def render_depth(self, camera: Camera, antialias: bool = False, projection: str = "ewa") -> dict:
        """Expected depth (model.py:166-180)."""
        p = self.params
        return render_gaussian_depth(camera, p["means"], p["quats"], self.scales_act, self.opacities_act,
                                     antialias=antialias, projection=projection)

    def render_features(
        self,
        camera: Camera,
        features: torch.Tensor,
        background: torch.Tensor | float | None = None,
        normalize: bool = False,
        antialias: bool = False,
        projection: str = "ewa",
    ) -> dict:
        """Arbitrary per-Gaussian features (model.py:182-203)."""
        p = self.params
        return render_gaussian_features(camera, p["means"], p["quats"], self.scales_act, self.opacities_act,
                                        features, background=background, normalize=normalize,
                                        antialias=antialias, projection=projection)

    def save_ply(self, path: str) -> None:
        """Save in the standard 3DGS PLY layout (model.py:338-361)."""
        from ..ply import save_gaussians_ply

        save_gaussians_ply(path, self.params)

    @classmethod
    def load_ply(cls, path: str, sh_degree: int = 3, device="cuda") -> "GaussianModel":
        """Load a 3DGS PLY checkpoint (model.py:363-392); the active SH degree
        is the file's degree."""
        from ..ply import load_gaussians_ply

        params, degree = load_gaussians_ply(path, sh_degree, device=device)
        model = cls(params, sh_degree=degree)
        model.active_sh_degree = degree
        return model

    def one_up_sh_degree(self) -> None:
        if self.active_sh_degree < self.sh_degree:
            self.active_sh_degree += 1
