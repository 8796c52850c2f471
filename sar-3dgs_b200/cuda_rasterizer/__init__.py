"""SAR-3DGS CUDA rasterizer package, B200 build.

Drop-in for the `cuda_rasterizer` package of SAR-3DGS
(cuda_rasterizer/__init__.py): same module-level names (CUDA_AVAILABLE,
CUDASARRasterizer, render_sar_func, render_sar_backward, render_sar,
GaussianDataCPU, GaussianDataGPU) and submodules (cuda_rasterizer_sar,
rasterizer_autograd). The native code is libsarr.so, built in place by
sar-3dgs_b200/build.py; importing the package never compiles anything and
never changes the working directory (the reference's loader calls os.chdir,
:50). Put the `sar-3dgs_b200` directory on sys.path to use it.

Rendering model (the reference's, rasterizer_impl_v2.cu:721-839):
    I(c, r) = sum_i T_i * sigma_i * gamma_i,ipp(c, r) * max(0, S_i),
    T_i = prod_{j before i in Z_r order} (1 - sigma_j * gamma_j,ipp(c, r)),
over the first 64 valid Gaussians (index order) whose bbox overlaps the pixel's
16x16 tile. The shadow term Omega is a separate per-Gaussian output of
render_sar and does not enter the image.
"""
from typing import Dict, Tuple

import torch

from . import _native
from . import cuda_rasterizer_sar
from .cuda_rasterizer_sar import SARRasterizationSettings

CUDASARRasterizer = None
render_sar_func = cuda_rasterizer_sar.render_sar
render_sar_backward = cuda_rasterizer_sar.render_sar_backward


class GaussianDataCPU:
    """Host-side Gaussian bundle (cuda_rasterizer/__init__.py:67-112)."""

    def __init__(self, means, covs, transmittance, scattering, radar_position, track_angle,
                 incidence_angle, azimuth_angle=0.0, range_resolution=1.0, azimuth_resolution=1.0,
                 range_samples=64, azimuth_samples=64):
        self.means = means
        self.covs = covs
        self.transmittance = transmittance
        self.scattering = scattering
        self.radar_position = radar_position
        self.track_angle = track_angle
        self.incidence_angle = incidence_angle
        self.azimuth_angle = azimuth_angle
        self.range_resolution = range_resolution
        self.azimuth_resolution = azimuth_resolution
        self.range_samples = range_samples
        self.azimuth_samples = azimuth_samples

    def to_device(self, device: torch.device) -> "GaussianDataGPU":
        return GaussianDataGPU(self.means.to(device), self.covs.to(device),
                               self.transmittance.to(device), self.scattering.to(device),
                               self.radar_position, self.track_angle, self.incidence_angle,
                               self.azimuth_angle, self.range_resolution, self.azimuth_resolution,
                               self.range_samples, self.azimuth_samples)


class GaussianDataGPU(GaussianDataCPU):
    """Device-side Gaussian bundle (cuda_rasterizer/__init__.py:115-144)."""


def render_sar(gaussian_data: GaussianDataGPU, output_height: int = 512,
               output_width: int = 512) -> Tuple[list, Dict]:
    """(cuda_rasterizer/__init__.py:147-186): renders with the bundle's own
    sample counts (output_height / output_width are unused, as in the
    reference) and returns ([image, omega], {})."""
    if not _native.available():
        raise RuntimeError("CUDA SAR rasterizer unavailable (no CUDA device or libsarr.so missing)")
    d = gaussian_data
    out = render_sar_func(d.means, d.covs, d.transmittance, d.scattering, d.radar_position[0],
                          d.radar_position[1], d.radar_position[2], d.track_angle,
                          d.incidence_angle, d.azimuth_angle, d.range_resolution,
                          d.azimuth_resolution, d.range_samples, d.azimuth_samples)
    return out, {}


def __getattr__(name):
    """CUDA_AVAILABLE (cuda_rasterizer/__init__.py:20-64 of the reference) is
    evaluated on first access rather than at import, so that importing the
    package (for its synthetic scenes, say) never loads libsarr.so."""
    if name == "CUDA_AVAILABLE":
        return _native.available()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = ["CUDA_AVAILABLE", "CUDASARRasterizer", "render_sar", "GaussianDataCPU",
           "GaussianDataGPU", "SARRasterizationSettings"]
