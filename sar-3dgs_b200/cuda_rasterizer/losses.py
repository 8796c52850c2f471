"""The training loss of SAR-3DGS (losses.py of the reference) on the fused
sm_100a kernel sarr_combined_loss: L1 (optionally weighted by the target) plus
D-SSIM with a Gaussian window, forward and gradient in two passes over the
images, deterministic.

Same names and return values as the reference's module: l1_loss,
weighted_l1_loss, dssim_loss, combined_loss and CombinedLoss (whose forward
returns the total loss tensor and a dict of Python floats, losses.py:160-219).
"""
from typing import Dict, Tuple

import torch
import torch.nn as nn

from . import _native

__all__ = ["l1_loss", "weighted_l1_loss", "dssim_loss", "combined_loss", "CombinedLoss"]


def _as_batch(x: torch.Tensor) -> torch.Tensor:
    """[H,W], [B,H,W] or [B,C,H,W] -> [V,H,W] (each channel its own image, as
    the reference's grouped convolution treats them)."""
    if x.dim() == 2:
        return x.unsqueeze(0)
    if x.dim() == 3:
        return x
    if x.dim() == 4:
        return x.reshape(-1, x.shape[-2], x.shape[-1])
    raise ValueError(f"input dimension error: dim()={x.dim()}")


def _layout(pred: torch.Tensor, target: torch.Tensor):
    """Both images in one memory order: the loss and its gradient are
    symmetric under transposing both, so a transposed view (the
    rasterizer's azimuth-major images) is passed without a copy."""
    p, t = _as_batch(pred), _as_batch(target)
    if not p.is_contiguous() and p.transpose(-1, -2).is_contiguous() and \
            t.transpose(-1, -2).is_contiguous():
        return p.transpose(-1, -2), t.transpose(-1, -2), True
    return p.contiguous(), t.contiguous(), False


class _CombinedLossFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pred, target, l1_weight, ssim_weight, window_size, l1_mode):
        p, t, transposed = _layout(pred, target)
        losses, grad = _native.combined_loss(p.detach(), t.detach(), l1_weight, ssim_weight,
                                             window_size, l1_mode, want_grad=pred.requires_grad)
        if grad is not None:
            if transposed:
                grad = grad.transpose(-1, -2)
            ctx.save_for_backward(grad.reshape(pred.shape))
        else:
            ctx.save_for_backward(None)
        ctx.mark_non_differentiable(losses)
        total = losses[0].clone()
        return total, losses

    @staticmethod
    def backward(ctx, grad_total, grad_losses):
        (grad,) = ctx.saved_tensors
        g = None if grad is None else grad * grad_total
        return g, None, None, None, None, None


def _combined(pred, target, l1_weight, ssim_weight, window_size, l1_mode):
    return _CombinedLossFunction.apply(pred, target, float(l1_weight), float(ssim_weight),
                                       int(window_size), l1_mode)


def l1_loss(pred: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """mean |pred - target| (losses.py:16-26)."""
    total, _ = _combined(pred, target, 1.0, 0.0, 1, "plain")
    return total


def weighted_l1_loss(pred: torch.Tensor, target: torch.Tensor, mode: str = "linear") -> torch.Tensor:
    """L1 weighted by 1 + f(target / max(target)) (losses.py:29-62)."""
    total, _ = _combined(pred, target, 1.0, 0.0, 1, mode if mode in ("linear", "square", "sqrt")
                         else "linear")
    return total


def dssim_loss(pred: torch.Tensor, target: torch.Tensor, window_size: int = 5) -> torch.Tensor:
    """1 - mean SSIM map (losses.py:80-124)."""
    total, _ = _combined(pred, target, 0.0, 1.0, window_size, "plain")
    return total


class CombinedLoss(nn.Module):
    """L1 + D-SSIM (losses.py:127-219)."""

    def __init__(self, l1_weight: float = 0.9, ssim_weight: float = 0.1, window_size: int = 5,
                 use_weighted_l1: bool = False, l1_weight_mode: str = "linear"):
        super().__init__()
        self.l1_weight = l1_weight
        self.ssim_weight = ssim_weight
        self.window_size = window_size
        self.use_weighted_l1 = use_weighted_l1
        self.l1_weight_mode = l1_weight_mode

    def forward(self, pred: torch.Tensor, target: torch.Tensor) -> Tuple[torch.Tensor, Dict[str, float]]:
        mode = self.l1_weight_mode if self.use_weighted_l1 else "plain"
        if mode not in ("plain", "linear", "square", "sqrt"):
            mode = "linear"
        total, losses = _combined(pred, target, self.l1_weight, self.ssim_weight, self.window_size,
                                  mode)
        vals = losses.tolist()
        return total, {
            "l1": vals[1],
            "dssim": vals[2],
            "total": vals[0],
            "l1_weight": self.l1_weight,
            "dssim_weight": self.ssim_weight,
            "weighted_l1": self.use_weighted_l1,
        }


def combined_loss(pred: torch.Tensor, target: torch.Tensor, l1_weight: float = 0.9,
                  ssim_weight: float = 0.1, window_size: int = 11, use_weighted_l1: bool = False,
                  l1_weight_mode: str = "linear") -> Tuple[torch.Tensor, Dict[str, float]]:
    """Functional form of CombinedLoss (losses.py:222-245)."""
    return CombinedLoss(l1_weight, ssim_weight, window_size, use_weighted_l1, l1_weight_mode)(pred, target)
