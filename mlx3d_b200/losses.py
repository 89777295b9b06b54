"""Image losses of the 3DGS training recipe (src/mlx3d/losses/image_metrics.py).

``ssim`` and ``l1_dssim_loss`` run on the fused sm_100a kernels behind
``gs_l1_ssim_forward`` / ``gs_l1_ssim_backward``: one forward kernel for the
five windowed statistics, the SSIM and L1 sums, one backward kernel for the
gradient of both terms.  ``l1_loss`` runs on ``gs_l1_forward`` /
``gs_l1_backward``; ``psnr`` is a one-line reduction.
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
        grad = torch.empty_like(pred)
        # d total = g_loss * d loss + g_l1 * d l1 + g_ssim * d ssim, each term linear in the
        # kernel's (l1 weight, ssim weight) = (1 - lam, -lam): one launch per needed term, the
        # cotangent read on the device, the later terms accumulated into the first.
        terms = []
        if g_loss is not None:
            terms.append((g_loss, 1.0, lam))
        if g_l1 is not None:
            terms.append((g_l1, 1.0, 0.0))
        if g_ssim is not None:
            terms.append((g_ssim, -1.0, 1.0))
        if not terms:
            return torch.zeros_like(pred), None, None, None, None, None
        for k, (g, sign, lam_k) in enumerate(terms):
            g = g.detach().to(torch.float32).contiguous()
            nat.call("gs_l1_ssim_backward_dev", nat.ptr(pred), nat.ptr(target), H, W, C, lam_k, window_size,
                     sigma, nat.ptr(ws), ws.numel(), nat.ptr(g), sign, int(k > 0), nat.ptr(grad), nat.stream())
        return grad, None, None, None, None, None


class _L1(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target):
        lib = nat.load()
        n = pred.numel()
        ws = torch.empty((lib.gs_l1_workspace_bytes(n),), device=pred.device, dtype=torch.uint8)
        loss = torch.empty((1,), device=pred.device, dtype=torch.float32)
        nat.call("gs_l1_forward", nat.ptr(pred), nat.ptr(target), n, nat.ptr(ws), ws.numel(), nat.ptr(loss),
                 nat.stream())
        ctx.save_for_backward(pred, target)
        return loss[0]

    @staticmethod
    def backward(ctx, g):
        pred, target = ctx.saved_tensors
        grad = torch.empty_like(pred)
        g = g.detach().to(torch.float32).contiguous()
        nat.call("gs_l1_backward", nat.ptr(pred), nat.ptr(target), pred.numel(), nat.ptr(g), nat.ptr(grad),
                 nat.stream())
        return grad, None


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
    """mean |pred - target| on the fused sm_100a kernels (deterministic sum);
    differentiable in pred."""
    if pred.shape != target.shape:
        raise ValueError("pred and target must have the same shape.")
    pred = nat.require_cuda("pred", pred)
    target = nat.require_cuda("target", target.detach())
    return _L1.apply(pred.contiguous(), target.contiguous())


def psnr(pred: torch.Tensor, target: torch.Tensor, max_val: float = 1.0) -> torch.Tensor:
    mse = ((pred - target) ** 2).mean()
    return 10.0 * torch.log10((max_val * max_val) / torch.clamp(mse, min=1e-12))
