"""The 3DGS optimisation recipe (src/mlx3d/splatting/trainer.py) on sm_100a.

One step: fused render (preprocess, binning, compositing) -> fused
L1 + D-SSIM loss -> fused backward -> one multi-tensor Adam launch over the
six parameter groups.  Learning rates and schedule follow the reference:
per-group Adam with eps = 1e-15 and no bias correction (mlx.optimizers.Adam's
default), ``lr_means`` (times the scene extent) decaying exponentially to
``lr_means_final`` over ``lr_means_max_steps``; update k uses the schedule's
value at k - 1 and ``learning_rates()`` reports the rate of the last update
(the behaviour pinned by the reference's test_trainer_position_lr_decays).

Screen-space positional gradient norms are accumulated for densification
(trainer.py:357-365); every ``densify_every`` steps inside the window the
model's adaptive density control runs (clone / split / prune, or MCMC
relocation with ``method="mcmc"``, trainer.py:366-400) and the Adam moments
follow the surviving rows (new rows start at zero).  The opacity reset and
SH-degree schedule run as in the reference.  ``method="2dgs"`` keeps every
Gaussian a thin surfel (third scale clamped to ``two_d_thickness`` times the
scene extent after each update and density event) and, with its lambdas set,
adds the depth-variance and normal-consistency losses of a second, feature
compositing pass (trainer.py:180-259).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import _native as nat
from ..cameras import Camera
from ..distributed import GradientReducer, world
from ..losses import l1_dssim_loss
from .model import GaussianModel
from .render import _project, _render_fused, side_streams

__all__ = ["TrainerConfig", "GaussianTrainer"]

_GROUPS = ("means", "scales", "quats", "opacities", "sh_dc", "sh_rest")


@dataclass
class TrainerConfig:
    """Fields and defaults of trainer.py:27-76 (densification fields kept for
    API compatibility; only the statistics they gate are computed)."""

    method: str = "vanilla"
    lr_means: float = 1.6e-4
    lr_means_final: float = 1.6e-6
    lr_means_max_steps: int = 30_000
    lr_scales: float = 5e-3
    lr_quats: float = 1e-3
    lr_opacities: float = 5e-2
    lr_sh_dc: float = 2.5e-3
    lr_sh_rest: float = 2.5e-3 / 20.0
    lambda_dssim: float = 0.2
    antialias: bool = False
    projection: str = "ewa"
    lambda_2d_depth_variance: float = 0.0  # 2DGS: ray-depth variance penalty
    lambda_2d_normal_consistency: float = 0.0  # 2DGS: rendered vs depth-map normals
    geometry_min_alpha: float = 0.05  # 2DGS: pixels below this alpha are left out of the geometry losses
    two_d_thickness: float = 1e-4  # 2DGS: surfel thickness as a fraction of the scene extent
    densify_from: int = 500
    densify_until: int = 15000
    densify_every: int = 100
    densify_grad_threshold: float = 0.0002
    mcmc_relocate_frac: float = 0.02
    mcmc_min_opacity: float = 0.01
    mcmc_jitter_scale: float = 0.25
    mcmc_noise_scale: float = 0.01
    opacity_reset_every: int = 3000
    sh_increase_every: int = 1000
    white_background: bool = False
    adam_betas: tuple = (0.9, 0.999)
    adam_eps: float = 1e-15
    adam_bias_correction: bool = False
    max_gaussians: int | None = None
    low_memory: bool = False  # releases torch's cached blocks after density events


class GaussianTrainer:
    """Optimises a :class:`GaussianModel` against posed images (trainer.py:79-421)."""

    def __init__(self, model: GaussianModel, config: TrainerConfig | None = None, scene_extent: float = 1.0):
        self.model = model
        self.config = config or TrainerConfig()
        if self.config.method not in {"vanilla", "mcmc", "2dgs"}:
            raise ValueError("TrainerConfig.method must be 'vanilla', 'mcmc', or '2dgs'")
        if self.config.projection not in {"ewa", "ut"}:
            raise ValueError("TrainerConfig.projection must be 'ewa' or 'ut'")
        self.scene_extent = scene_extent
        self.step_count = 0
        for k in _GROUPS:
            p = model.params[k]
            if not p.is_contiguous() or p.dtype != torch.float32 or p.device.type != "cuda":
                raise ValueError(f"parameter {k} must be a contiguous float32 CUDA tensor")
            p.requires_grad_(True)
        self._m = {k: torch.zeros_like(model.params[k]) for k in _GROUPS}
        self._v = {k: torch.zeros_like(model.params[k]) for k in _GROUPS}
        self._lr_last = self._schedule(0)
        self._reset_grad_accum()
        self._apply_method_constraints()

    # ----------------------------------------------------------- schedules
    def _schedule(self, k: int) -> dict[str, float]:
        c = self.config
        lr0 = c.lr_means * self.scene_extent
        lr1 = c.lr_means_final * self.scene_extent
        if c.lr_means_max_steps > 0 and lr0 > 0 and lr1 > 0:
            lr_means = lr0 * ((lr1 / lr0) ** (1.0 / c.lr_means_max_steps)) ** k
        else:
            lr_means = lr0
        return {"means": lr_means, "scales": c.lr_scales, "quats": c.lr_quats, "opacities": c.lr_opacities,
                "sh_dc": c.lr_sh_dc, "sh_rest": c.lr_sh_rest}

    def learning_rates(self) -> dict[str, float]:
        """Per-parameter rates of the last update (before any update: of the first)."""
        return dict(self._lr_last)

    def _reset_grad_accum(self) -> None:
        n = self.model.num_gaussians
        dev = self.model.params["means"].device
        self.grad_accum = torch.zeros((n,), dtype=torch.float32, device=dev)
        self.grad_count = torch.zeros((n,), dtype=torch.float32, device=dev)

    # ------------------------------------------------------------- pieces
    def _apply_method_constraints(self) -> None:
        """2DGS: keep every Gaussian a thin surfel (trainer.py:180-183)."""
        if self.config.method == "2dgs":
            self.model.apply_2dgs_constraints(self.config.two_d_thickness * max(float(self.scene_extent), 1e-8))

    def _geometry_loss_2dgs(self, camera: Camera):
        """2DGS geometry terms (trainer.py:186-259): a second compositing pass
        of per-Gaussian features [depth, depth^2, normal (3)] (normal = the
        local z axis, flipped towards the camera), normalised by alpha; the
        ray-depth variance E[z^2] - E[z]^2 and 1 - |cos| between the rendered
        normals and the normals of the depth map's unprojected points, both
        averaged over pixels with alpha > geometry_min_alpha.  Returns
        (loss or None, metrics)."""
        from .projection import quat_to_rotmat
        from .rasterize import rasterize_features
        from .tiles import bin_gaussians

        cfg = self.config
        metrics = {"depth_variance": 0.0, "normal_consistency": 0.0}
        if cfg.method != "2dgs" or (cfg.lambda_2d_depth_variance <= 0 and cfg.lambda_2d_normal_consistency <= 0):
            return None, metrics
        p = self.model.params
        W, H = camera.width, camera.height
        dev = p["means"].device
        proj = _project(camera, p["means"], p["quats"], torch.exp(p["scales"]), cfg.projection, cfg.antialias)
        opac = torch.sigmoid(p["opacities"]) * proj["compensation"]
        ids, ranges, tx, ty = bin_gaussians(proj["means2d"], proj["radii"], proj["depths"], W, H)
        depths = proj["depths"]
        normals = quat_to_rotmat(p["quats"])[:, :, 2]
        view = camera.camera_center.to(dev) - p["means"]
        normals = normals / torch.clamp(torch.linalg.norm(normals, dim=-1, keepdim=True), min=1e-8)
        normals = torch.where((normals * view).sum(-1, keepdim=True) < 0, -normals, normals)
        feats = torch.cat([depths[:, None], (depths * depths)[:, None], normals], dim=1)
        geom = rasterize_features(proj["means2d"], proj["conics"], feats, opac, ids, ranges, W, H, tx, ty,
                                  normalize=True)
        valid = (geom["alpha"] > cfg.geometry_min_alpha).float()
        denom = torch.clamp(valid.sum(), min=1.0)
        ed, ed2 = geom["features"][..., 0], geom["features"][..., 1]
        loss = torch.zeros((), device=dev)
        if cfg.lambda_2d_depth_variance > 0:
            dv = (torch.clamp(ed2 - ed * ed, min=0.0) * valid).sum() / denom
            metrics["depth_variance"] = dv.detach()
            loss = loss + float(cfg.lambda_2d_depth_variance) * dv
        if cfg.lambda_2d_normal_consistency > 0 and W > 1 and H > 1:
            u = torch.arange(W, dtype=torch.float32, device=dev) + 0.5
            v = torch.arange(H, dtype=torch.float32, device=dev) + 0.5
            uu, vv = u[None, :].expand(H, W), v[:, None].expand(H, W)
            pts = camera.unproject_points(torch.stack([uu, vv], dim=-1), ed)
            tan_x = pts[:-1, 1:] - pts[:-1, :-1]
            tan_y = pts[1:, :-1] - pts[:-1, :-1]
            dn = torch.linalg.cross(tan_x, tan_y)
            dn = dn / torch.clamp(torch.linalg.norm(dn, dim=-1, keepdim=True), min=1e-8)
            rn = geom["features"][:-1, :-1, 2:5]
            rn = rn / torch.clamp(torch.linalg.norm(rn, dim=-1, keepdim=True), min=1e-8)
            valid4 = valid[:-1, :-1] * valid[:-1, 1:] * valid[1:, :-1] * valid[1:, 1:]
            cos = (rn * dn).sum(-1)
            nc = ((1.0 - cos.abs()) * valid4).sum() / torch.clamp(valid4.sum(), min=1.0)
            metrics["normal_consistency"] = nc.detach()
            loss = loss + float(cfg.lambda_2d_normal_consistency) * nc
        return loss, metrics

    def _view_forward(self, camera: Camera, target: torch.Tensor, probe: torch.Tensor | None):
        """Render + loss of one view (graph kept for the backward)."""
        cfg = self.config
        dev = self.model.params["means"].device
        bg = torch.ones(3, device=dev) if cfg.white_background else torch.zeros(3, device=dev)
        p = self.model.params
        if cfg.projection == "ut":
            out = self.model.render(camera, background=bg, antialias=cfg.antialias, projection="ut")
        else:
            out = _render_fused(
                camera, p["means"], p["quats"], p["scales"], p["opacities"], sh_dc=p["sh_dc"], sh_rest=p["sh_rest"],
                sh_degree=self.model.active_sh_degree, background=bg, antialias=cfg.antialias,
                flags=nat.GS_ACT_EXP_SCALES | nat.GS_ACT_SIGMOID_OPACITY, probe=probe)
        loss, _, _ = l1_dssim_loss(out["image"], target, cfg.lambda_dssim)
        geom, metrics = self._geometry_loss_2dgs(camera)
        if geom is not None:
            loss = loss + geom
        self._geometry = metrics
        return loss, out

    def _view_loss(self, camera: Camera, target: torch.Tensor, probe: torch.Tensor | None, scale: float):
        loss, out = self._view_forward(camera, target, probe)
        (loss * scale).backward()
        return loss.detach(), out

    def _adam_chunked(self, flat: torch.Tensor, chunks: list) -> None:
        """The Adam update of a step whose gradients are the flat buffer
        ``flat`` (parameter order _GROUPS) being all-reduced in ``chunks``
        ((begin, end, work) element ranges): each chunk's parameter rows are
        updated as soon as its sum has arrived, while the later chunks are
        still on the wire (one launch per chunk over the parameters it
        intersects)."""
        self.step_count += 1
        lrs = self._schedule(self.step_count - 1)
        self._lr_last = lrs
        c = self.config
        spans, off = [], 0
        for k in _GROUPS:
            n = self.model.params[k].numel()
            spans.append((k, off, off + n))
            off += n
        for a, b, work in chunks:
            if work is not None:
                work.wait()
            groups = (nat.GsAdamGroup * len(_GROUPS))()
            ng = 0
            for k, lo, hi in spans:
                s0, s1 = max(a, lo), min(b, hi)
                if s0 >= s1:
                    continue
                p, d = self.model.params[k], s0 - lo
                groups[ng] = nat.GsAdamGroup(p.data_ptr() + 4 * d, flat.data_ptr() + 4 * s0,
                                             self._m[k].data_ptr() + 4 * d, self._v[k].data_ptr() + 4 * d,
                                             s1 - s0, lrs[k])
                ng += 1
            nat.call("gs_adam_step", groups, ng, c.adam_betas[0], c.adam_betas[1], c.adam_eps,
                     int(c.adam_bias_correction), self.step_count, nat.stream())
        for k in _GROUPS:
            self.model.params[k].grad = None

    def _adam(self) -> None:
        self.step_count += 1
        lrs = self._schedule(self.step_count - 1)
        self._lr_last = lrs
        c = self.config
        groups = (nat.GsAdamGroup * len(_GROUPS))()
        for i, k in enumerate(_GROUPS):
            p = self.model.params[k]
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            g = p.grad.contiguous()
            p.grad = g
            groups[i] = nat.GsAdamGroup(p.data_ptr(), g.data_ptr(), self._m[k].data_ptr(), self._v[k].data_ptr(),
                                        p.numel(), lrs[k])
        nat.call("gs_adam_step", groups, len(_GROUPS), c.adam_betas[0], c.adam_betas[1], c.adam_eps,
                 int(c.adam_bias_correction), self.step_count, nat.stream())
        for k in _GROUPS:
            self.model.params[k].grad = None

    # ----------------------------------------------------- density control
    def _resize_moments(self, keep_idx: torch.Tensor, new_count: int) -> None:
        """Adam moments of the surviving rows, zeros for appended ones
        (trainer.py:139-159)."""
        for k in _GROUPS:
            for st in (self._m, self._v):
                kept = st[k][keep_idx]
                if new_count > 0:
                    kept = torch.cat([kept, torch.zeros((new_count, *kept.shape[1:]), dtype=kept.dtype,
                                                        device=kept.device)], dim=0)
                st[k] = kept.contiguous()

    def _zero_moment_rows(self, idx: torch.Tensor) -> None:
        """Relocated rows restart their moments (trainer.py:161-179)."""
        if idx is None or idx.numel() == 0:
            return
        for k in _GROUPS:
            self._m[k][idx] = 0.0
            self._v[k][idx] = 0.0

    def _density_event(self) -> dict:
        cfg = self.config
        if cfg.method == "mcmc":
            result = self.model.relocate_mcmc(self.grad_accum, self.grad_count, relocate_frac=cfg.mcmc_relocate_frac,
                                              min_opacity=cfg.mcmc_min_opacity, jitter_scale=cfg.mcmc_jitter_scale)
            self._zero_moment_rows(result.get("_moved_idx"))
        else:
            # At the cap, growth stops (infinite threshold) but pruning goes on.
            at_cap = cfg.max_gaussians is not None and self.model.num_gaussians >= cfg.max_gaussians
            threshold = float("inf") if at_cap else cfg.densify_grad_threshold
            result = self.model.densify_and_prune(self.grad_accum, self.grad_count, grad_threshold=threshold,
                                                  scene_extent=self.scene_extent, return_optimizer_state=True)
            self._resize_moments(result["_keep_idx"], result["_new_count"])
        self._reset_grad_accum()
        if cfg.low_memory and torch.cuda.is_available():
            torch.cuda.empty_cache()
        return {k: v for k, v in result.items() if not str(k).startswith("_")}

    def _mcmc_noise(self) -> None:
        """SGLD-like position noise of the MCMC method (trainer.py:343-350)."""
        cfg = self.config
        if cfg.method != "mcmc" or cfg.mcmc_noise_scale <= 0:
            return
        sigma = cfg.mcmc_noise_scale * self.scene_extent * math.sqrt(max(self.learning_rates()["means"], 0.0))
        if sigma > 0:
            with torch.no_grad():
                m = self.model.params["means"]
                m.add_(torch.randn_like(m) * sigma)

    def _schedules_after_update(self) -> tuple[bool, bool]:
        cfg = self.config
        opacity_reset = sh_changed = False
        if self.step_count % cfg.opacity_reset_every == 0 and self.step_count <= cfg.densify_until:
            self.model.reset_opacities(0.01)
            opacity_reset = True
        if self.step_count % cfg.sh_increase_every == 0:
            self.model.one_up_sh_degree()
            sh_changed = True
        return opacity_reset, sh_changed

    def _info(self, loss: float, opacity_reset: bool, sh_changed: bool, densify: dict | None = None) -> dict:
        return {"loss": loss, "num_gaussians": self.model.num_gaussians, "step": self.step_count,
                "active_sh_degree": self.model.active_sh_degree, "lr_means": self.learning_rates()["means"],
                "method": self.config.method, "densify": densify, "opacity_reset": opacity_reset,
                "sh_degree_changed": sh_changed,
                "geometry": {k: float(v) for k, v in getattr(self, "_geometry", {}).items()}}

    # --------------------------------------------------------------- steps
    def step(self, camera: Camera, target: torch.Tensor) -> dict:
        """One optimisation step on a single view (trainer.py:319-421)."""
        cfg = self.config
        track = cfg.densify_from <= self.step_count + 1 <= cfg.densify_until and cfg.projection == "ewa"
        probe = torch.zeros((self.model.num_gaussians, 2), device=target.device) if track else None
        loss, out = self._view_loss(camera, target, probe, 1.0)
        self._adam()
        self._mcmc_noise()
        self._apply_method_constraints()
        densify = None
        if track:
            with torch.no_grad():
                g = probe * torch.tensor([camera.width / 2.0, camera.height / 2.0], device=probe.device)
                visible = (out["radii"] > 0).float()
                self.grad_accum += g.norm(dim=-1) * visible
                self.grad_count += visible
            if self.step_count % cfg.densify_every == 0 and self.step_count > cfg.densify_from:
                densify = self._density_event()
                self._apply_method_constraints()
        opacity_reset, sh_changed = self._schedules_after_update()
        return self._info(float(loss), opacity_reset, sh_changed, densify)

    def _views_backward(self, cameras, targets, scale: float, streams: int, first_sink=None) -> list:
        """Forward + backward of every view, gradients accumulated in .grad.

        With ``streams`` > 1 the views are pipelined: view i's forward runs
        on stream i mod ``streams`` while view i-1's backward runs on its own
        stream, so the latency-bound per-Gaussian pass and binning of one view
        overlap the compositor backward of the other.  Every backward waits
        for the previous view's backward (an event), so the accumulations
        into .grad stay ordered; the current stream waits for all of them.
        ``first_sink`` (a context manager) is entered around the first view's
        backward (the one that creates .grad).  Returns the detached per-view
        losses (usable on the current stream)."""
        import contextlib

        sink = first_sink if first_sink is not None else contextlib.nullcontext()
        if streams <= 1 or len(cameras) <= 1:
            out = []
            for i, (c, t) in enumerate(zip(cameras, targets)):
                if i == 0:
                    with sink:
                        out.append(self._view_loss(c, t, None, scale)[0])
                else:
                    out.append(self._view_loss(c, t, None, scale)[0])
            return out
        cur = torch.cuda.current_stream()
        ss = side_streams(streams)
        for s in ss:
            s.wait_stream(cur)
        losses, prev_bwd, pending = [], None, None
        for i, (cam, tgt) in enumerate(zip(cameras, targets)):
            s = ss[i % len(ss)]
            with torch.cuda.stream(s):
                loss, _ = self._view_forward(cam, tgt, None)
            if pending is not None:  # previous view's backward, issued after this view's forward
                prev_bwd = self._issue_backward(*pending, prev_bwd, sink if i == 1 else None)
            pending = (loss, scale, s)
            losses.append(loss.detach())
        self._issue_backward(*pending, prev_bwd, sink if len(cameras) == 1 else None)
        for s in ss:
            cur.wait_stream(s)
        for loss in losses:  # made on the side streams, read on the current one
            loss.record_stream(cur)
        return losses

    @staticmethod
    def _issue_backward(loss, scale, s, after, sink=None):
        import contextlib

        with torch.cuda.stream(s), (sink if sink is not None else contextlib.nullcontext()):
            if after is not None:
                s.wait_event(after)
            (loss * scale).backward()
            done = torch.cuda.Event()
            done.record(s)
        return done

    def step_views(self, cameras: list[Camera], targets: list[torch.Tensor], total_views: int | None = None,
                   monitor=None, streams: int = 2) -> dict:
        """One data-parallel step over a batch of views: this rank renders
        ``cameras`` (its shard), the loss is averaged over ``total_views``
        (all ranks' views), gradients are summed over ranks (NCCL all-reduce)
        and one Adam update is applied on every rank.  With a
        :class:`~mlx3d_b200.distributed.PeerMonitor`, the ranks exchange
        heartbeats before anything is launched, so a rank that left makes
        this raise ``PeerLost`` instead of blocking in the all-reduce."""
        if monitor is not None:
            monitor.beat(self.step_count)
        rank, ws = world()
        if total_views is None:
            total_views = len(cameras) * ws
        plist = [self.model.params[k] for k in _GROUPS]
        red = None
        if ws > 1:
            # the first view's backward writes the gradients straight into the
            # flat all-reduce buffer (later views accumulate into them in
            # place), so the all-reduce needs no gathering copy
            if getattr(self, "_reducer", None) is None:
                self._reducer = GradientReducer()
            red = self._reducer
            for p in plist:
                p.grad = None
        losses = self._views_backward(cameras, targets, 1.0 / total_views, streams,
                                      first_sink=red.sink(plist) if red is not None else None)
        loss_sum = torch.stack(losses).sum() if losses else torch.zeros((), device=self.model.params["means"].device)
        if red is not None:
            red.stage(plist)  # copies only gradients that did not land in the buffer
            flat, chunks = red.launch_chunks(4)  # the all-reduce, in four asynchronous pieces
            self._adam_chunked(flat, chunks)  # each piece's rows updated once its sum arrived
        else:
            self._adam()
        self._mcmc_noise()
        self._apply_method_constraints()
        opacity_reset, sh_changed = self._schedules_after_update()
        info = self._info(float(loss_sum) / max(len(cameras), 1), opacity_reset, sh_changed)
        info["views"] = len(cameras)
        return info
