"""The trainable Gaussian scene (src/mlx3d/splatting/model.py).

Adaptive density control (clone / split / prune, MCMC relocation, compact
checkpoints, opacity reset; model.py:273-545) edits the Gaussian table with
torch tensor operations on the parameters' own device: it is control of the
set between optimisation steps, not part of the rendering path.

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
from .render import (_check_projection, _render_composed, _render_fused, render_gaussian_depth,
                     render_gaussian_features, side_streams)
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

    def render_views(self, cameras, background: torch.Tensor | None = None, antialias: bool = False,
                     render_depth: bool = False, streams: int = 2, on_output=None) -> list:
        """Render several views, pipelined over ``streams`` CUDA streams: view
        i runs on stream i mod ``streams``, so one view's per-Gaussian pass
        and binning (latency bound, and the host's wait for the duplicate
        count) overlap another view's compositor.  Forward only (no
        autograd graph is kept).  ``on_output(i, out)`` is called for every
        view as soon as its work is enqueued, on that view's stream (as the
        current stream); its return value is collected instead of the
        outputs when given (keeping 256 4K outputs alive would need tens of
        GB).  The current stream waits for all views before this returns."""
        cur = torch.cuda.current_stream()
        ss = side_streams(max(1, int(streams)))
        for s in ss:
            s.wait_stream(cur)
        results = []
        with torch.no_grad():
            for i, cam in enumerate(cameras):
                s = ss[i % len(ss)]
                with torch.cuda.stream(s):
                    out = self.render(cam, background=background, antialias=antialias, render_depth=render_depth)
                    results.append(on_output(i, out) if on_output is not None else out)
        for s in ss:
            cur.wait_stream(s)
        if on_output is None:
            for out in results:  # outputs made on side streams are used on the current one
                for v in out.values():
                    if isinstance(v, torch.Tensor) and v.is_cuda:
                        v.record_stream(cur)
        return results

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

    def apply_2dgs_constraints(self, max_thickness: float) -> None:
        """Clamp the third local log-scale to log(max_thickness), turning each
        Gaussian into an oriented disk (2DGS surfels; model.py:128-143)."""
        thickness = max(float(max_thickness), 1e-8)
        lim = math.log(thickness)
        with torch.no_grad():
            s = self.params["scales"]
            s[:, 2:3].clamp_(max=lim)

    def surfel_points(self, min_opacity: float = 0.01, max_points: int | None = None,
                      orient_towards=None) -> tuple[torch.Tensor, torch.Tensor]:
        """Surfel centres and unit normals (the local z axis) of the Gaussians
        with activated opacity >= ``min_opacity`` (model.py:210-254).  At
        most ``max_points`` are kept, ranked by opacity * scale_x * scale_y
        (the row of largest importance survives when none passes the opacity
        test); rows keep index order.  ``orient_towards`` flips each normal to
        face that point."""
        from .projection import quat_to_rotmat

        if max_points is not None and max_points <= 0:
            raise ValueError("max_points must be positive when provided.")
        n = self.num_gaussians
        dev = self.params["means"].device
        if n == 0:
            empty = torch.zeros((0, 3), device=dev)
            return empty, empty
        with torch.no_grad():
            opacity = self.opacities_act
            scales = self.scales_act
            importance = opacity * scales[:, 0] * scales[:, 1]
            keep = opacity >= float(min_opacity)
            if not bool(keep.any()):
                keep[int(torch.argmax(importance))] = True
            keep_idx = torch.nonzero(keep).flatten()
            if max_points is not None and keep_idx.numel() > max_points:
                local = torch.topk(importance[keep_idx], max_points).indices
                keep_idx = keep_idx[local]
            keep_idx = torch.sort(keep_idx).values
            points = self.params["means"][keep_idx].clone()
            normals = quat_to_rotmat(self.params["quats"][keep_idx])[:, :, 2]
            normals = normals / torch.clamp(torch.linalg.norm(normals, dim=-1, keepdim=True), min=1e-8)
            if orient_towards is not None:
                target = torch.as_tensor(orient_towards, dtype=points.dtype, device=dev)
                flip = ((target - points) * normals).sum(-1, keepdim=True) < 0
                normals = torch.where(flip, -normals, normals)
        return points, normals

    def one_up_sh_degree(self) -> None:
        if self.active_sh_degree < self.sh_degree:
            self.active_sh_degree += 1

    # --------------------------------------------------- density control
    def _set_params(self, new: dict[str, torch.Tensor]) -> None:
        """Replace the tables by contiguous leaves, keeping requires_grad."""
        out = {}
        for k, v in new.items():
            t = v.detach().contiguous()
            old = self.params.get(k)
            if old is not None and old.requires_grad:
                t.requires_grad_(True)
            out[k] = t
        self.params = out

    def copy(self) -> "GaussianModel":
        """A detached copy of the Gaussian table (model.py:273-277)."""
        out = GaussianModel({k: v.detach().clone() for k, v in self.params.items()}, self.sh_degree)
        out.active_sh_degree = self.active_sh_degree
        return out

    def select(self, keep_idx) -> None:
        """Keep only the rows ``keep_idx``, in that order (model.py:395-398)."""
        idx = torch.as_tensor(keep_idx, dtype=torch.long, device=self.params["means"].device)
        self._set_params({k: v.detach()[idx] for k, v in self.params.items()})

    def append(self, new_params: dict[str, torch.Tensor]) -> None:
        """Concatenate rows after the existing ones (model.py:400-404)."""
        self._set_params({k: torch.cat([v.detach(), new_params[k].to(v)], dim=0) for k, v in self.params.items()})

    def reset_opacities(self, max_opacity: float = 0.01) -> None:
        """Clamp the opacity logits to logit(max_opacity) (model.py:533-538)."""
        logit = math.log(max_opacity / (1.0 - max_opacity))
        with torch.no_grad():
            self.params["opacities"].clamp_(max=logit)

    def compact(self, min_opacity: float = 0.0, max_gaussians: int | None = None,
                target_sh_degree: int | None = None) -> "GaussianModel":
        """A smaller checkpoint (model.py:279-336): rows with activated opacity
        below ``min_opacity`` dropped (the most important row kept if none
        survives), at most ``max_gaussians`` rows by importance
        opacity * max(scale)^2, original order preserved, SH truncated to
        ``target_sh_degree``; this model is not modified."""
        if max_gaussians is not None and max_gaussians <= 0:
            raise ValueError("max_gaussians must be positive when provided.")
        if target_sh_degree is not None and not (0 <= target_sh_degree <= self.sh_degree):
            raise ValueError("target_sh_degree must be between 0 and the model sh_degree.")
        n = self.num_gaussians
        if n == 0:
            return self.copy()
        with torch.no_grad():
            opacity = self.opacities_act
            max_scale = self.scales_act.max(dim=1).values
            importance = opacity * max_scale * max_scale
            keep = opacity >= float(min_opacity)
            if not bool(keep.any()):
                keep[int(torch.argmax(importance))] = True
            keep_idx = torch.nonzero(keep).flatten()
            if max_gaussians is not None and keep_idx.numel() > max_gaussians:
                local = torch.topk(importance[keep_idx], max_gaussians).indices
                keep_idx = keep_idx[local]
            keep_idx = torch.sort(keep_idx).values
            params = {k: v.detach()[keep_idx].clone() for k, v in self.params.items()}
        sh_degree = self.sh_degree
        if target_sh_degree is not None:
            sh_degree = int(target_sh_degree)
            k = num_sh_bases(sh_degree)
            params["sh_rest"] = params["sh_rest"][:, : max(0, k - 1), :].contiguous()
        out = GaussianModel(params, sh_degree=sh_degree)
        out.active_sh_degree = min(self.active_sh_degree, sh_degree)
        return out

    def densify_and_prune(self, grad_accum: torch.Tensor, grad_count: torch.Tensor,
                          grad_threshold: float = 0.0002, scene_extent: float = 1.0,
                          percent_dense: float = 0.01, min_opacity: float = 0.005,
                          return_optimizer_state: bool = False, generator: torch.Generator | None = None,
                          samples: torch.Tensor | None = None) -> dict:
        """Adaptive density control of the 3DGS paper (model.py:406-480).

        Average screen-space gradient = grad_accum / max(grad_count, 1); rows
        above ``grad_threshold`` are cloned when their largest scale is at
        most ``percent_dense * scene_extent``, otherwise split into two rows
        drawn from the Gaussian (offsets R (s * N(0, 1)), log-scales reduced
        by log 1.6).  Split sources, rows with opacity below ``min_opacity``
        and rows larger than half the scene extent are pruned.  The kept rows
        come first, then the clones, then the split pairs.  Returns the counts
        (and, with ``return_optimizer_state``, the kept indices and the number
        of appended rows, for resizing optimizer moments).  ``samples``
        ((2 * splits, 3) standard normal draws, pair-major) replaces the
        draws from ``generator``."""
        from .projection import quat_to_rotmat

        dev = self.params["means"].device
        with torch.no_grad():
            avg_grad = grad_accum.to(dev) / torch.clamp(grad_count.to(dev), min=1.0)
            scales = self.scales_act.detach()
            max_scale = scales.max(dim=1).values
            high_grad = avg_grad > grad_threshold
            small = max_scale <= percent_dense * scene_extent
            clone_idx = torch.nonzero(high_grad & small).flatten()
            split_idx = torch.nonzero(high_grad & ~small).flatten()
            p = {k: v.detach() for k, v in self.params.items()}
            clones = {k: v[clone_idx] for k, v in p.items()}
            splits = {}
            if split_idx.numel() > 0:
                R = quat_to_rotmat(p["quats"][split_idx])
                s = scales[split_idx]
                if samples is None:
                    samples = torch.randn((split_idx.numel() * 2, 3), device=dev, dtype=s.dtype, generator=generator)
                elif samples.shape != (split_idx.numel() * 2, 3):
                    raise ValueError(f"samples must have shape ({split_idx.numel() * 2}, 3)")
                samples = samples.to(device=dev, dtype=s.dtype)
                samples = samples * s.repeat_interleave(2, dim=0)
                offsets = torch.einsum("nij,nj->ni", R.repeat_interleave(2, dim=0), samples)
                splits = {k: v[split_idx].repeat_interleave(2, dim=0) for k, v in p.items()}
                splits["means"] = splits["means"] + offsets
                splits["scales"] = splits["scales"] - math.log(1.6)
            opac = torch.sigmoid(torch.clamp(p["opacities"], -50.0, 50.0))
            split_mask = high_grad & ~small
            prune = (opac < min_opacity) | split_mask | (max_scale > 0.5 * scene_extent)
            keep_idx = torch.nonzero(~prune).flatten()
            new = {k: torch.cat([v[keep_idx], clones[k]] + ([splits[k]] if splits else []), dim=0)
                   for k, v in p.items()}
        self._set_params(new)
        stats = {"cloned": int(clone_idx.numel()), "split": int(split_idx.numel()), "pruned": int(prune.sum())}
        if return_optimizer_state:
            stats["_keep_idx"] = keep_idx
            stats["_new_count"] = int(clone_idx.numel() + 2 * split_idx.numel())
        return stats

    def relocate_mcmc(self, grad_accum: torch.Tensor, grad_count: torch.Tensor, relocate_frac: float = 0.02,
                      min_opacity: float = 0.01, jitter_scale: float = 0.25,
                      generator: torch.Generator | None = None, noise: torch.Tensor | None = None) -> dict:
        """Fixed-budget relocation (model.py:482-531): up to
        ``relocate_frac * N`` underused rows (opacity below ``min_opacity`` or
        never visible; the least opaque rows when none is underused) are
        overwritten by copies of the highest-gradient other rows, with means
        jittered by ``jitter_scale`` times the source scales, the opacity
        reset to logit(0.05) and log-scales reduced by log 1.6.  N is kept.
        ``noise`` ((k, 3) standard normal draws, in the order of the returned
        ``_moved_idx``) replaces the draws from ``generator``."""
        n = self.num_gaussians
        max_relocate = int(max(0.0, min(relocate_frac, 1.0)) * n)
        if max_relocate <= 0 or n <= 1:
            return {"relocated": 0}
        dev = self.params["means"].device
        with torch.no_grad():
            counts = grad_count.to(dev)
            avg_grad = grad_accum.to(dev) / torch.clamp(counts, min=1.0)
            opac = torch.sigmoid(self.params["opacities"].detach())
            underused = (opac < min_opacity) | (counts <= 0)
            n_under = int(underused.sum())
            k = max_relocate if n_under == 0 else min(max_relocate, n_under)
            k = min(k, n - 1)
            if k == 0:
                return {"relocated": 0}
            target_score = torch.where(underused, 2.0 - opac, -opac)
            dst = torch.topk(target_score, k).indices
            source_score = avg_grad.clone()
            source_score[dst] = -1e30
            src = torch.topk(source_score, k).indices
            source_scales = torch.exp(self.params["scales"].detach()[src])
            new = {}
            for name, arr in self.params.items():
                arr = arr.detach()
                values = arr[src].clone()
                if name == "means" and jitter_scale > 0:
                    z = (torch.randn(values.shape, device=dev, dtype=values.dtype, generator=generator)
                         if noise is None else noise.to(device=dev, dtype=values.dtype).reshape(values.shape))
                    values = values + z * source_scales * float(jitter_scale)
                elif name == "opacities":
                    values = torch.full_like(values, math.log(0.05 / 0.95))
                elif name == "scales":
                    values = values - math.log(1.6)
                out = arr.clone()
                out[dst] = values
                new[name] = out
        self._set_params(new)
        return {"relocated": int(k), "_moved_idx": dst}
