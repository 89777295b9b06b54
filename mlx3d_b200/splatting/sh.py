"""Real spherical harmonics, degrees 0-3 (src/mlx3d/splatting/sh.py)."""

from __future__ import annotations

import torch

from .. import _native as nat

__all__ = ["eval_sh", "rgb_to_sh", "sh_to_rgb", "num_sh_bases", "SH_C0"]

SH_C0 = 0.28209479177387814


def num_sh_bases(degree: int) -> int:
    return (degree + 1) ** 2


def rgb_to_sh(rgb: torch.Tensor) -> torch.Tensor:
    """DC coefficient from RGB in [0, 1] (sh.py:30-32)."""
    return (rgb - 0.5) / SH_C0


def sh_to_rgb(sh_dc: torch.Tensor) -> torch.Tensor:
    """RGB from the DC coefficient (sh.py:35-37)."""
    return sh_dc * SH_C0 + 0.5


class _EvalSH(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sh, dirs, degree):
        n, k, c = sh.shape
        out = torch.empty((n, c), device=sh.device, dtype=torch.float32)
        nat.call("gs_eval_sh_forward", degree, nat.ptr(sh), n, k, c, nat.ptr(dirs), nat.ptr(out), nat.stream())
        ctx.save_for_backward(sh, dirs)
        ctx.degree = degree
        return out

    @staticmethod
    def backward(ctx, g_out):
        sh, dirs = ctx.saved_tensors
        n, k, c = sh.shape
        g_sh = torch.empty_like(sh)
        g_dirs = torch.empty_like(dirs) if ctx.needs_input_grad[1] else None
        nat.call(
            "gs_eval_sh_backward", ctx.degree, nat.ptr(sh), n, k, c, nat.ptr(dirs), nat.ptr(g_out.contiguous()),
            nat.ptr(g_sh), nat.ptr(g_dirs), nat.stream(),
        )
        return g_sh, g_dirs, None


def eval_sh(degree: int, sh: torch.Tensor, dirs: torch.Tensor) -> torch.Tensor:
    """Evaluate SH at unit directions (sh.py:41-78).

    ``sh`` (N, K, C) with K >= (degree+1)^2, ``dirs`` (N, 3).  Returns (N, C)
    colours offset by +0.5 (callers clamp to >= 0).
    """
    if not 0 <= degree <= 3:
        raise ValueError("degree must be in [0, 3].")
    sh = nat.require_cuda("sh", sh)
    dirs = nat.require_cuda("dirs", dirs)
    if sh.ndim != 3 or sh.shape[1] < num_sh_bases(degree):
        raise ValueError(f"sh must have shape (N, K, C) with K >= {num_sh_bases(degree)}.")
    if dirs.shape != (sh.shape[0], 3):
        raise ValueError("dirs must have shape (N, 3).")
    return _EvalSH.apply(sh, dirs, int(degree))
