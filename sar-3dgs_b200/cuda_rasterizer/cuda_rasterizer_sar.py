"""Drop-in for the pybind11 module `cuda_rasterizer_sar` of SAR-3DGS.

The reference module (cuda_rasterizer/rasterizer_impl_v2.cu:1701-1705) exports
render_sar, render_sar_with_settings and render_sar_backward. This module
exports the same three functions with the same argument order, shapes and
return values, backed by libsarr.so on PyTorch's current CUDA stream, plus
batched multi-view variants.

Differences that only remove reference failure modes:
  - render_sar accepts 14 or 16 positional arguments (the reference binding has
    no py::arg defaults, so its own 14-argument callers raise TypeError);
  - inputs are made contiguous instead of being read through data_ptr() as if
    they were, and an SH column slice [N, K] of a wider tensor is read through
    its row stride with the K active columns only;
  - errors raise RuntimeError instead of being ignored.
"""
import torch

from . import _native

__all__ = ["render_sar", "render_sar_backward", "render_sar_with_settings",
           "SARRasterizationSettings", "render_sar_batched", "render_sar_backward_batched"]


class SARRasterizationSettings:
    """Python counterpart of the C++ struct SARRasterizationSettings
    (rasterizer_impl_v2.cu:476-488), which the reference never exposed to
    Python (so its render_sar_with_settings could not be called)."""

    def __init__(self, n_gaussians=0, radar_x=0.0, radar_y=0.0, radar_z=10000.0, track_angle=0.0,
                 incidence_angle=30.0, azimuth_angle=0.0, range_resolution=0.3,
                 azimuth_resolution=0.3, range_samples=128, azimuth_samples=128,
                 prefiltered=False, debug=False):
        self.n_gaussians = n_gaussians
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
        self.prefiltered = prefiltered
        self.debug = debug


def _view(radar_x, radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
          range_resolution, azimuth_resolution, range_samples, azimuth_samples):
    return _native.make_view(radar_x, radar_y, radar_z, track_angle, incidence_angle,
                             azimuth_angle, range_resolution, azimuth_resolution,
                             range_samples, azimuth_samples)


def render_sar(means_world, cov_world, transmittance, sh_coeffs, radar_x, radar_y, radar_z,
               track_angle, incidence_angle, azimuth_angle, range_resolution,
               azimuth_resolution, range_samples, azimuth_samples, prefiltered=False,
               debug=False):
    """Forward render of one view (rasterizer_impl_v2.cu:1618-1662).

    cov_world is the packed [N,6] upper triangle (cov_3x3_to_6 order); a full
    [N,3,3] matrix is accepted too. Returns [image, omega]: image has shape
    [range_samples, azimuth_samples] with the reference's azimuth-major memory
    (element (r, c) of the picture at flat index c * range_samples + r);
    omega [N] is the per-Gaussian mean shadow occlusion. `prefiltered` is
    ignored, as in the reference; `debug=True` synchronises and raises on
    device-side errors."""
    means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
        means_world, cov_world, transmittance, sh_coeffs)
    view = _view(radar_x, radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
                 range_resolution, azimuth_resolution, range_samples, azimuth_samples)
    n = means.shape[0]
    image = torch.empty((int(range_samples), int(azimuth_samples)), dtype=torch.float32,
                        device=means.device)
    omega = torch.empty((n,), dtype=torch.float32, device=means.device)
    _native.forward([view], means, cov, layout, sigma, sh, sh_stride, sh_k, image, omega=omega,
                    check_device=bool(debug))
    return [image, omega]


def render_sar_with_settings(means_world, cov_world, transmittance, sh_coeffs, settings):
    """render_sar with a SARRasterizationSettings object (:1664-1699)."""
    s = settings
    return render_sar(means_world, cov_world, transmittance, sh_coeffs, s.radar_x, s.radar_y,
                      s.radar_z, s.track_angle, s.incidence_angle, s.azimuth_angle,
                      s.range_resolution, s.azimuth_resolution, s.range_samples,
                      s.azimuth_samples, s.prefiltered, s.debug)


def render_sar_backward(means_world, cov_world, transmittance, sh_coeffs, grad_output, radar_x,
                        radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
                        range_resolution, azimuth_resolution, range_samples, azimuth_samples):
    """Backward of one view (rasterizer_impl_v2.cu:1380-1616).

    grad_output has the image's shape and layout. Returns
    [grad_means [N,3], grad_cov [N,6], grad_transmittance [N], grad_sh [N,16]]
    with grad_cov slots 0, 1, 3 holding the image-plane rr, cc, rc terms and
    slots 2, 4, 5 zero, as the reference computes them."""
    means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
        means_world, cov_world, transmittance, sh_coeffs)
    view = _view(radar_x, radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
                 range_resolution, azimuth_resolution, range_samples, azimuth_samples)
    n = means.shape[0]
    g = _native._as_cuda_f32(grad_output, "grad_output").contiguous()
    if g.numel() != int(range_samples) * int(azimuth_samples):
        raise RuntimeError("grad_output must have range_samples * azimuth_samples elements")
    dev = means.device
    grad_means = torch.empty((n, 3), dtype=torch.float32, device=dev)
    grad_cov = torch.empty((n, 6), dtype=torch.float32, device=dev)
    grad_sigma = torch.empty((n,), dtype=torch.float32, device=dev)
    grad_sh = torch.empty((n, 16), dtype=torch.float32, device=dev)
    _native.backward([view], means, cov, layout, sigma, sh, sh_stride, sh_k, g, grad_means,
                     grad_cov, _native.SARR_COV6, grad_sigma, grad_sh)
    return [grad_means, grad_cov, grad_sigma, grad_sh]


def _views_from(views):
    out = []
    for v in views:
        if isinstance(v, _native.SarrView):
            out.append(v)
        elif isinstance(v, SARRasterizationSettings):
            out.append(_view(v.radar_x, v.radar_y, v.radar_z, v.track_angle, v.incidence_angle,
                             v.azimuth_angle, v.range_resolution, v.azimuth_resolution,
                             v.range_samples, v.azimuth_samples))
        elif isinstance(v, dict):
            out.append(_view(v.get("radar_x", 0.0), v.get("radar_y", 0.0), v["radar_z"],
                             v["track_angle"], v["incidence_angle"], v.get("azimuth_angle", 0.0),
                             v["range_resolution"], v["azimuth_resolution"], v["range_samples"],
                             v["azimuth_samples"]))
        else:
            out.append(_view(*v))
    if not out:
        raise RuntimeError("at least one view is required")
    return out


def render_sar_batched(means_world, cov_world, transmittance, sh_coeffs, views, want_omega=False,
                       out=None, states=None):
    """Renders many views of one scene in a few launches (views are processed
    up to 256 per kernel launch). `views`: SarrView, SARRasterizationSettings,
    dicts or 10-tuples sharing range/azimuth samples. Returns images
    [V, range_samples, azimuth_samples] (each in the reference layout) and,
    with want_omega, omega [V, N]."""
    means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
        means_world, cov_world, transmittance, sh_coeffs)
    vs = _views_from(views)
    nr, na = vs[0].range_samples, vs[0].azimuth_samples
    dev = means.device
    if out is None:
        out = torch.empty((len(vs), nr, na), dtype=torch.float32, device=dev)
    omega = torch.empty((len(vs), means.shape[0]), dtype=torch.float32, device=dev) if want_omega else None
    _native.forward(vs, means, cov, layout, sigma, sh, sh_stride, sh_k, out, omega=omega,
                    states=states)
    return (out, omega) if want_omega else out


def render_sar_backward_batched(means_world, cov_world, transmittance, sh_coeffs, grad_images,
                                views, states=None, grad_sh_cols=16, grad_norm=False):
    """Summed backward of many views: returns grad_means [N,3], grad_cov [N,6],
    grad_transmittance [N], grad_sh [N, grad_sh_cols] (and the per-Gaussian
    ||grad_means|| when grad_norm=True)."""
    means, cov, layout, sigma, sh, sh_stride, sh_k = _native.prepare_inputs(
        means_world, cov_world, transmittance, sh_coeffs)
    vs = _views_from(views)
    n = means.shape[0]
    dev = means.device
    g = _native._as_cuda_f32(grad_images, "grad_images").contiguous()
    gm = torch.empty((n, 3), dtype=torch.float32, device=dev)
    gc = torch.empty((n, 6), dtype=torch.float32, device=dev)
    gs = torch.empty((n,), dtype=torch.float32, device=dev)
    gsh = torch.empty((n, grad_sh_cols), dtype=torch.float32, device=dev)
    gn = torch.empty((n,), dtype=torch.float32, device=dev) if grad_norm else None
    _native.backward(vs, means, cov, layout, sigma, sh, sh_stride, sh_k, g, gm, gc,
                     _native.SARR_COV6, gs, gsh, grad_norm=gn, states=states)
    return (gm, gc, gs, gsh, gn) if grad_norm else (gm, gc, gs, gsh)
