"""Densification and pruning of the Gaussian set (GaussianModel.densify_and_prune
of the reference, gaussian_model.py:433-566) on the sm_100a kernels
sarr_densify_flags / sarr_densify_apply: flags, counts and a stable scatter in
three passes instead of per-index Python loops; same new set in the same order.
"""
from typing import Tuple

import torch
import torch.nn as nn

from . import _native

__all__ = ["densify_and_prune", "densify_and_prune_tensors"]


def densify_and_prune_tensors(means, scales, rotations, opacities, sh_coeffs, grad_means,
                              grad_threshold=0.0001, size_threshold=0.01, large_scale_threshold=2.0,
                              opacity_threshold=0.05, max_gaussians=500000):
    """Returns ((means, scales, rotations, opacities, sh_coeffs) of the new set,
    (num_clones, num_splits, num_prunes, total_new))."""
    with torch.no_grad():
        return _native.densify_and_prune(means.detach(), scales.detach(), rotations.detach(),
                                         opacities.detach(), sh_coeffs.detach(), grad_means.detach(),
                                         grad_threshold, size_threshold, large_scale_threshold,
                                         opacity_threshold, max_gaussians)


def densify_and_prune(model, grad_means: torch.Tensor, grad_scales: torch.Tensor = None,
                      grad_opacities: torch.Tensor = None, grad_threshold: float = 0.0001,
                      size_threshold: float = 0.01, large_scale_threshold: float = 2.0,
                      opacity_threshold: float = 0.05,
                      max_gaussians: int = 500000) -> Tuple[int, int, int, int]:
    """In place on a GaussianModel-like object (attributes _means, _scales,
    _rotations, _opacities, _sh_coeffs), as the reference's method: the
    parameters are replaced by new nn.Parameters; grad_scales and
    grad_opacities are accepted and unused, as in the reference."""
    out, counts = densify_and_prune_tensors(model._means, model._scales, model._rotations,
                                            model._opacities, model._sh_coeffs, grad_means,
                                            grad_threshold, size_threshold, large_scale_threshold,
                                            opacity_threshold, max_gaussians)
    clones, splits, prunes, new = counts
    if prunes == 0 and new == 0:
        return counts
    for name, t in zip(("_means", "_scales", "_rotations", "_opacities", "_sh_coeffs"), out):
        setattr(model, name, nn.Parameter(t, requires_grad=True))
    return counts
