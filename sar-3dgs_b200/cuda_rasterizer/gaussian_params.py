"""Gaussian parameters of a training step (GaussianModel of the reference,
gaussian_model.py:261-330) on the sm_100a kernel sarr_gaussian_params: the
covariance Sigma = R diag(exp(s))^2 R^T from log-scales and quaternions in one
pass (the reference builds S with a Python loop over the Gaussians), and the
sigmoid transmittance.

The covariance is detached, as in the reference (its cache holds
Sigma.detach()); the transmittance keeps its gradient (d sigmoid)."""
import torch

from . import _native

__all__ = ["compute_covariance_full", "compute_covariance", "compute_covariance_rasterizer",
           "get_opacity"]

_REF6 = ((0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2))


def compute_covariance_full(scales: torch.Tensor, rotations: torch.Tensor) -> torch.Tensor:
    """[N,3,3] detached covariance (gaussian_model.py:285-328)."""
    cov, _ = _native.gaussian_params(scales.detach(), rotations.detach(), None, _native.SARR_COV33)
    return cov


def compute_covariance(scales: torch.Tensor, rotations: torch.Tensor) -> torch.Tensor:
    """[N,6] upper triangle in the reference's order 00, 01, 02, 11, 12, 22
    (gaussian_model.py:261-283)."""
    full = compute_covariance_full(scales, rotations)
    return torch.stack([full[:, a, b] for a, b in _REF6], dim=1)


def compute_covariance_rasterizer(scales: torch.Tensor, rotations: torch.Tensor) -> torch.Tensor:
    """[N,6] in the rasterizer's order xx, yy, zz, xy, xz, yz (cov_3x3_to_6)."""
    cov, _ = _native.gaussian_params(scales.detach(), rotations.detach(), None, _native.SARR_COV6)
    return cov


class _Sigmoid(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits):
        _, sigma = _native.gaussian_params(None, None, logits.detach())
        sigma = sigma.reshape(logits.shape)
        ctx.save_for_backward(sigma)
        return sigma

    @staticmethod
    def backward(ctx, grad):
        (sigma,) = ctx.saved_tensors
        return grad * sigma * (1.0 - sigma)


def get_opacity(opacity_logits: torch.Tensor) -> torch.Tensor:
    """sigmoid(opacity_logits) with its gradient (gaussian_model.py:330-332)."""
    return _Sigmoid.apply(opacity_logits)
