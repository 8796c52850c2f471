"""Host-side behaviour of the drop-in Python modules (no GPU): surface,
argument handling, loud failure without CUDA, and the covariance packing
helpers against the reference definitions (rasterizer_autograd.py:99-131)."""
import inspect

import pytest
import torch

import cuda_rasterizer
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import rasterizer_autograd as RA


def test_module_surface_matches_reference():
    for name in ("render_sar", "render_sar_backward", "render_sar_with_settings"):
        assert callable(getattr(M, name))
    for name in ("SARRasterizerFunction", "SARRasterizer", "cov_3x3_to_6", "cov_6_to_3x3",
                 "quaternion_to_rotation_matrix", "compute_scales_rotations_grad"):
        assert hasattr(RA, name)
    for name in ("CUDA_AVAILABLE", "CUDASARRasterizer", "render_sar", "GaussianDataCPU",
                 "GaussianDataGPU", "render_sar_func", "render_sar_backward"):
        assert hasattr(cuda_rasterizer, name)


def test_render_sar_accepts_14_and_16_arguments():
    sig = inspect.signature(M.render_sar)
    args14 = [None] * 4 + [0.0] * 8 + [64, 64]
    sig.bind(*args14)
    sig.bind(*(args14 + [False, False]))
    with pytest.raises(TypeError):
        sig.bind(*args14[:13])
    assert len(inspect.signature(M.render_sar_backward).parameters) == 15


def test_cpu_tensors_fail_loudly():
    n = 4
    args = (torch.zeros(n, 3), torch.zeros(n, 6), torch.ones(n), torch.zeros(n, 16),
            0.0, 0.0, 5000.0, 0.0, 30.0, 0.0, 0.3, 0.3, 32, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.render_sar(*args)
    with pytest.raises(RuntimeError, match="CUDA"):
        RA.SARRasterizer(range_samples=32, azimuth_samples=32)(args[0], torch.zeros(n, 3, 3), args[2], args[3])
    if not torch.cuda.is_available():
        assert cuda_rasterizer.CUDA_AVAILABLE is False
        with pytest.raises(RuntimeError):
            cuda_rasterizer.render_sar(cuda_rasterizer.GaussianDataGPU(
                args[0], args[1], args[2], args[3], (0, 0, 5000), 0.0, 30.0))


def _ref_cov_3x3_to_6(cov):
    n = cov.shape[0]
    out = torch.zeros(n, 6, dtype=cov.dtype)
    out[:, 0] = cov[:, 0, 0]
    out[:, 1] = cov[:, 1, 1]
    out[:, 2] = cov[:, 2, 2]
    out[:, 3] = cov[:, 0, 1]
    out[:, 4] = cov[:, 0, 2]
    out[:, 5] = cov[:, 1, 2]
    return out


def _ref_cov_6_to_3x3(f):
    n = f.shape[0]
    c = torch.zeros(n, 3, 3, dtype=f.dtype)
    c[:, 0, 0] = f[:, 0]
    c[:, 1, 1] = f[:, 1]
    c[:, 2, 2] = f[:, 2]
    c[:, 0, 1] = f[:, 3]
    c[:, 0, 2] = f[:, 4]
    c[:, 1, 2] = f[:, 5]
    c[:, 1, 0] = f[:, 3]
    c[:, 2, 0] = f[:, 4]
    c[:, 2, 1] = f[:, 5]
    return c


def test_cov_packing_matches_reference_definition():
    g = torch.Generator().manual_seed(0)
    cov = torch.randn(17, 3, 3, generator=g)  # deliberately non-symmetric: only the upper triangle is read
    assert torch.equal(RA.cov_3x3_to_6(cov), _ref_cov_3x3_to_6(cov))
    f = torch.randn(17, 6, generator=g)
    assert torch.equal(RA.cov_6_to_3x3(f), _ref_cov_6_to_3x3(f))


def test_quaternion_to_rotation_matrix():
    q = torch.tensor([[1.0, 0.0, 0.0, 0.0], [0.0, 0.0, 0.0, 1.0]])
    R = RA.quaternion_to_rotation_matrix(q)
    assert torch.allclose(R[0], torch.eye(3))
    assert torch.allclose(R[1], torch.diag(torch.tensor([-1.0, -1.0, 1.0])))
    assert RA.quaternion_to_rotation_matrix(q[0]).shape == (3, 3)


def test_sar_rasterizer_defaults_and_omega():
    r = RA.SARRasterizer()
    assert (r.radar_z, r.incidence_angle, r.range_resolution, r.range_samples) == (10000.0, 30.0, 0.3, 128)
    assert r.get_last_omega() is None


def test_settings_object_fields():
    s = M.SARRasterizationSettings(range_samples=64, azimuth_samples=32)
    for f in ("n_gaussians", "radar_x", "radar_y", "radar_z", "track_angle", "incidence_angle",
              "azimuth_angle", "range_resolution", "azimuth_resolution", "range_samples",
              "azimuth_samples", "prefiltered", "debug"):
        assert hasattr(s, f)
