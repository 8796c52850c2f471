"""Autograd wrapper of the SAR rasterizer; drop-in for
cuda_rasterizer/rasterizer_autograd.py of SAR-3DGS (same classes, functions and
signatures).

Design differences from the reference, none visible in the results:
  - the [N,3,3] covariance is read directly by the kernels and the covariance
    gradient is written directly in [N,3,3] form (the reference packs with
    cov_3x3_to_6 and unpacks with cov_6_to_3x3, :159, :215, :249);
  - Omega is not computed in the autograd forward: the reference computes it
    and drops it (:178);
  - the forward keeps its per-tile lists and sorted tile records in a small
    state buffer that the backward reuses, instead of recomputing the whole
    forward pipeline (rasterizer_impl_v2.cu:1495-1559); the saved inputs are
    version-checked by autograd, so the state always matches them;
  - grad_output is made contiguous before it is read (the reference reads
    grad_output.data_ptr() as a dense image, which is wrong for expanded
    gradients such as the one of image.sum()).
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import _native

__all__ = ["SARRasterizerFunction", "SARRasterizer", "cov_3x3_to_6", "cov_6_to_3x3",
           "quaternion_to_rotation_matrix", "compute_scales_rotations_grad"]


def quaternion_to_rotation_matrix(q: torch.Tensor) -> torch.Tensor:
    """Rotation matrices from (w, x, y, z) quaternions (rasterizer_autograd.py:61-96)."""
    squeeze = q.dim() == 1
    if squeeze:
        q = q.unsqueeze(0)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    ], dim=-1).reshape(-1, 3, 3)
    return R.squeeze(0) if squeeze else R


def compute_scales_rotations_grad(grad_cov: torch.Tensor, scales: torch.Tensor,
                                  rotations: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Kept for API compatibility with rasterizer_autograd.py:9-58, which the
    reference never calls. Same values: every scale gradient column is
    2 exp(s_k) * sum_ij R[i, j] * M[j, i] evaluated on the first rows of
    R and M = grad_cov @ R^T (as the reference indexes them), and the rotation
    gradient is zero."""
    exp_scales = torch.exp(scales)
    R = quaternion_to_rotation_matrix(rotations)
    M = torch.matmul(grad_cov, R.transpose(-1, -2))
    s = sum(R[j, i] * M[i, j] for i in range(3) for j in range(3))
    grad_scales = torch.zeros_like(scales)
    for k in range(3):
        grad_scales[:, k] = 2 * exp_scales[:, k] * s
    return grad_scales, torch.zeros_like(rotations)


_TRIU6 = ((0, 0), (1, 1), (2, 2), (0, 1), (0, 2), (1, 2))


def cov_3x3_to_6(cov: torch.Tensor) -> torch.Tensor:
    """[N,3,3] -> [N,6] upper triangle in the order xx, yy, zz, xy, xz, yz
    (rasterizer_autograd.py:99-113)."""
    rows = torch.tensor([a for a, _ in _TRIU6], device=cov.device)
    cols = torch.tensor([b for _, b in _TRIU6], device=cov.device)
    return cov[:, rows, cols].contiguous()


def cov_6_to_3x3(cov_flat: torch.Tensor) -> torch.Tensor:
    """[N,6] -> symmetric [N,3,3] (rasterizer_autograd.py:116-131)."""
    idx = torch.tensor([0, 3, 4, 3, 1, 5, 4, 5, 2], device=cov_flat.device)
    return cov_flat[:, idx].reshape(-1, 3, 3)


class SARRasterizerFunction(torch.autograd.Function):
    """Forward renders one view; backward returns the gradients of
    means_world, cov_world, transmittance and sh_coeffs
    (rasterizer_autograd.py:134-274)."""

    @staticmethod
    def forward(ctx, means_world, cov_world, transmittance, sh_coeffs, radar_x, radar_y, radar_z,
                track_angle, incidence_angle, azimuth_angle, range_resolution, azimuth_resolution,
                range_samples, azimuth_samples):
        means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
            means_world, cov_world, transmittance, sh_coeffs)
        view = _native.make_view(radar_x, radar_y, radar_z, track_angle, incidence_angle,
                                 azimuth_angle, range_resolution, azimuth_resolution,
                                 range_samples, azimuth_samples)
        n = means.shape[0]
        dev = means.device
        state = torch.empty(_native.state_bytes(n, view.range_samples, view.azimuth_samples),
                            dtype=torch.uint8, device=dev)
        image = torch.empty((int(range_samples), int(azimuth_samples)), dtype=torch.float32,
                            device=dev)
        _native.forward([view], means, cov, layout, sigma, sh, sh_stride, sh_k, image,
                        states=state)
        ctx.save_for_backward(means_world, cov_world, transmittance, sh_coeffs)
        ctx.view = view
        ctx.state = state
        return image

    @staticmethod
    def backward(ctx, grad_output):
        means_world, cov_world, transmittance, sh_coeffs = ctx.saved_tensors
        means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
            means_world, cov_world, transmittance, sh_coeffs)
        n = means.shape[0]
        dev = means.device
        g = grad_output.to(torch.float32).contiguous()
        grad_means = torch.empty((n, 3), dtype=torch.float32, device=dev)
        if layout == _native.SARR_COV33:
            grad_cov = torch.empty((n, 3, 3), dtype=torch.float32, device=dev)
        else:
            grad_cov = torch.empty((n, 6), dtype=torch.float32, device=dev)
        grad_sigma = torch.empty((n,), dtype=torch.float32, device=dev)
        grad_sh = torch.empty((n, sh_k), dtype=torch.float32, device=dev)
        _native.backward([ctx.view], means, cov, layout, sigma, sh, sh_stride, sh_k, g, grad_means,
                         grad_cov, layout, grad_sigma, grad_sh, states=ctx.state)
        if grad_sigma.numel() == transmittance.numel():
            grad_sigma = grad_sigma.reshape_as(transmittance)
        grad_cov = grad_cov.reshape_as(cov_world) if grad_cov.numel() == cov_world.numel() else grad_cov
        grad_sh = grad_sh.reshape_as(sh_coeffs) if grad_sh.numel() == sh_coeffs.numel() else grad_sh
        return (grad_means, grad_cov, grad_sigma, grad_sh) + (None,) * 10


class SARRasterizer(nn.Module):
    """SAR renderer module holding one radar view (rasterizer_autograd.py:277-340)."""

    def __init__(self, radar_x: float = 0.0, radar_y: float = 0.0, radar_z: float = 10000.0,
                 track_angle: float = 0.0, incidence_angle: float = 30.0,
                 azimuth_angle: float = 0.0, range_resolution: float = 0.3,
                 azimuth_resolution: float = 0.3, range_samples: int = 128,
                 azimuth_samples: int = 128):
        super().__init__()
        self.radar_x = radar_x
        self.radar_y = radar_y
        self.radar_z = radar_z
        self.track_angle = track_angle
        self.incidence_angle = incidence_angle
        self.azimuth_angle = azimuth_angle
        self.range_resolution = range_resolution
        self.azimuth_resolution = azimuth_resolution
        self.range_samples = range_samples
        self.azimuth_samples = azimuth_samples
        self.last_omega: Optional[torch.Tensor] = None

    def forward(self, means_world, cov_world, transmittance, sh_coeffs):
        result = SARRasterizerFunction.apply(
            means_world, cov_world, transmittance, sh_coeffs, self.radar_x, self.radar_y,
            self.radar_z, self.track_angle, self.incidence_angle, self.azimuth_angle,
            self.range_resolution, self.azimuth_resolution, self.range_samples,
            self.azimuth_samples)
        if isinstance(result, (list, tuple)):
            self.last_omega = result[1].detach()
            return result[0]
        return result

    def get_last_omega(self) -> Optional[torch.Tensor]:
        return self.last_omega
