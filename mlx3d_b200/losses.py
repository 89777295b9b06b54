"""Image losses of the 3DGS training recipe (src/mlx3d/losses/image_metrics.py).

``ssim`` and ``l1_dssim_loss`` run on the fused sm_100a kernels behind
``gs_l1_ssim_forward`` / ``gs_l1_ssim_backward``: one forward kernel for the
five windowed statistics, the SSIM and L1 sums, one backward kernel for the
gradient of both terms.  ``psnr`` and ``l1_loss`` are one-line reductions.
"""

from __future__ import annotations

import torch

from . import _native as nat

__all__ = ["ssim", "l1_loss", "psnr", "l1_dssim_loss"]


def _prep(pred, target):
    if pred.shape != target.shape:
        raise ValueError("pred and target must have the same shape.")
    if pred.ndim == 4:
        if pred.shape[0] != 1:
            raise ValueError("batched SSIM supports a batch of one image (N=1).")
        pred, target = pred[0], target[0]
    if pred.ndim != 3:
        raise ValueError("images must have shape (H, W, C) or (1, H, W, C).")
    return nat.require_cuda("pred", pred), nat.require_cuda("target", target.detach())


class _L1DSSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, lam, max_val, window_size, sigma):
        H, W, C = pred.shape
        lib = nat.load()
        ws = torch.empty((lib.gs_l1_ssim_workspace_bytes(H, W, C),), device=pred.device, dtype=torch.uint8)
        loss = torch.empty((3,), device=pred.device, dtype=torch.float32)
        nat.call("gs_l1_ssim_forward", nat.ptr(pred), nat.ptr(target), H, W, C, lam, max_val, window_size, sigma,
                 nat.ptr(ws), ws.numel(), nat.ptr(loss), nat.stream())
        ctx.save_for_backward(pred, target, ws)
        ctx.args = (lam, max_val, window_size, sigma)
        return loss[0], loss[1], loss[2]

    @staticmethod
    def backward(ctx, g_loss, g_l1, g_ssim):
        pred, target, ws = ctx.saved_tensors
        lam, max_val, window_size, sigma = ctx.args
        H, W, C = pred.shape
        grad = torch.zeros_like(pred)
        # d total = g_loss * d loss + g_l1 * d l1 + g_ssim * d ssim, each term linear in the
        # kernel's (l1 weight, ssim weight) = (1 - lam, -lam): run it once per needed term.
        terms = []
        if g_loss is not None:
            terms.append((g_loss, lam))
        if g_l1 is not None:
            terms.append((g_l1, 0.0))
        if g_ssim is not None:
            terms.append((-g_ssim, 1.0))
        for g, lam_k in terms:
            part = torch.empty_like(pred)
            nat.call("gs_l1_ssim_backward", nat.ptr(pred), nat.ptr(target), H, W, C, lam_k, max_val, window_size,
                     sigma, nat.ptr(ws), ws.numel(), 1.0, nat.ptr(part), nat.stream())
            grad += part * g
        return grad, None, None, None, None, None


def l1_dssim_loss(pred: torch.Tensor, target: torch.Tensor, lambda_dssim: float = 0.2, max_val: float = 1.0,
                  window_size: int = 11, sigma: float = 1.5):
    """``(1 - lambda) * mean|pred - target| + lambda * (1 - ssim(pred, target))``
    (trainer.py:300-305); returns ``(loss, l1, ssim)`` scalar tensors."""
    pred, target = _prep(pred, target)
    return _L1DSSIM.apply(pred, target, float(lambda_dssim), float(max_val), int(window_size), float(sigma))


def ssim(pred: torch.Tensor, target: torch.Tensor, max_val: float = 1.0, window_size: int = 11,
         sigma: float = 1.5) -> torch.Tensor:
    """Mean SSIM with a Gaussian window (image_metrics.py:66-85); differentiable in pred."""
    return l1_dssim_loss(pred, target, 1.0, max_val, window_size, sigma)[2]


def l1_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return (pred - target).abs().mean()


def psnr(pred: torch.Tensor, target: torch.Tensor, max_val: float = 1.0) -> torch.Tensor:
    mse = ((pred - target) ** 2).mean()
    return 10.0 * torch.log10((max_val * max_val) / torch.clamp(mse, min=1e-12))
