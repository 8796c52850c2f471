"""Seeded synthetic SAR scenes and radar view sets.

These are the workloads the benchmark and the tests run (no dataset is
shipped with this package; the MSTAR images the reference trains on are not
redistributable):
  - Gaussians: means uniform in a W x L x H box centred at the origin with
    z in [0, H]; covariance R diag(s^2) R^T with per-axis scales s
    log-uniform in [s_min, s_max] and R from a normalised N(0,1)^4 quaternion
    (w, x, y, z); transmittance sigmoid(N(0,1)); 16 SH coefficients
    N(0, 0.1^2) with +0.5 on the DC term.
  - Views: radar altitude 5 km, squint (azimuth_angle) 0, track angle and
    incidence per workload.
Generation runs on the CPU with torch.Generator so that the same seed gives
the same scene on every machine; tensors are then moved to `device`.
"""
import math

import torch

SCENES = {
    # name: (n, box (W, L, H) [m], scale range [m])
    "cpu_1k": (1000, (20.0, 20.0, 6.0), (0.05, 0.5)),
    "train_50k": (50_000, (20.0, 20.0, 6.0), (0.05, 0.5)),
    "target_20k": (20_000, (20.0, 20.0, 6.0), (0.05, 0.5)),
    "hires_500k": (500_000, (60.0, 60.0, 15.0), (0.02, 0.3)),
    "sweep_1m": (1_000_000, (40.0, 40.0, 10.0), (0.05, 0.5)),
}


def quat_to_rot(q):
    w, x, y, z = q.unbind(-1)
    return torch.stack([
        1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
        2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
        2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y),
    ], dim=-1).reshape(*q.shape[:-1], 3, 3)


def cov33_to_cov6(cov):
    return torch.stack([cov[:, 0, 0], cov[:, 1, 1], cov[:, 2, 2], cov[:, 0, 1], cov[:, 0, 2],
                        cov[:, 1, 2]], dim=1).contiguous()


def make_scene(n, box=(20.0, 20.0, 6.0), scale_range=(0.05, 0.5), seed=0, device="cpu"):
    """Returns dict(means [n,3], cov33 [n,3,3], cov6 [n,6], sigma [n], sh [n,16])."""
    g = torch.Generator().manual_seed(int(seed))
    W, L, H = box
    u = torch.rand(n, 3, generator=g, dtype=torch.float64)
    means = torch.stack([(u[:, 0] - 0.5) * W, (u[:, 1] - 0.5) * L, u[:, 2] * H], dim=1)
    lo, hi = math.log(scale_range[0]), math.log(scale_range[1])
    s = torch.exp(torch.rand(n, 3, generator=g, dtype=torch.float64) * (hi - lo) + lo)
    q = torch.randn(n, 4, generator=g, dtype=torch.float64)
    q = q / q.norm(dim=1, keepdim=True)
    R = quat_to_rot(q)
    cov = R @ torch.diag_embed(s * s) @ R.transpose(1, 2)
    cov = 0.5 * (cov + cov.transpose(1, 2))
    sigma = torch.sigmoid(torch.randn(n, generator=g, dtype=torch.float64))
    sh = torch.randn(n, 16, generator=g, dtype=torch.float64) * 0.1
    sh[:, 0] += 0.5
    cov33 = cov.float()
    out = {"means": means.float(), "cov33": cov33, "cov6": cov33_to_cov6(cov33),
           "sigma": sigma.float(), "sh": sh.float()}
    return {k: v.to(device) for k, v in out.items()}


def named_scene(name, seed=0, device="cpu"):
    n, box, sr = SCENES[name]
    return make_scene(n, box, sr, seed=seed, device=device)


def view_tuple(track_angle, incidence_angle, rho, samples, azimuth_angle=0.0, altitude=5000.0):
    """(radar_x, radar_y, radar_z, track, incidence, azimuth, rho_r, rho_a, Nr, Na)."""
    return (0.0, 0.0, float(altitude), float(track_angle), float(incidence_angle),
            float(azimuth_angle), float(rho), float(rho), int(samples), int(samples))


def cpu_view():
    """CPU forward case: 128 x 128 at 0.3 m, incidence 15 deg, squint 0, track 30 deg."""
    return view_tuple(30.0, 15.0, 0.3, 128)


def sweep_views(n_views=1024, step_deg=0.35, incidence=(15.0, 45.0), rho=0.2, samples=256,
                seed=2, offset_deg=0.0):
    """Multi-view inference sweep: track angle stepped by `step_deg`, incidence
    uniform in `incidence`, 256 x 256 at 0.2 m."""
    g = torch.Generator().manual_seed(int(seed))
    inc = torch.rand(n_views, generator=g, dtype=torch.float64) * (incidence[1] - incidence[0]) + incidence[0]
    return [view_tuple(offset_deg + k * step_deg, float(inc[k]), rho, samples) for k in range(n_views)]


def training_views(n_views=64, incidences=(15.0, 17.0), rho=0.3, samples=128, seed=2):
    """Training views: track angle uniform over 0-360 deg, incidence 15 or 17 deg."""
    g = torch.Generator().manual_seed(int(seed))
    az = torch.rand(n_views, generator=g, dtype=torch.float64) * 360.0
    pick = torch.randint(0, len(incidences), (n_views,), generator=g)
    return [view_tuple(float(az[k]), incidences[int(pick[k])], rho, samples) for k in range(n_views)]


def hires_views(n_views=16, incidence=(15.0, 45.0), rho=0.1, samples=512, seed=2):
    """High-resolution views: 512 x 512 at 0.1 m, incidence uniform 15-45 deg."""
    g = torch.Generator().manual_seed(int(seed))
    az = torch.rand(n_views, generator=g, dtype=torch.float64) * 360.0
    inc = torch.rand(n_views, generator=g, dtype=torch.float64) * (incidence[1] - incidence[0]) + incidence[0]
    return [view_tuple(float(az[k]), float(inc[k]), rho, samples) for k in range(n_views)]


def make_param_scene(n, box=(40.0, 40.0, 10.0), scale_range=(0.05, 0.5), seed=0, device="cpu"):
    """The same distributions as make_scene, in the trainable form of
    GaussianModel (gaussian_model.py:112-132): means [n,3], log-scales [n,3],
    unit quaternions (w, x, y, z) [n,4], opacity logits [n] (sigmoid gives
    the transmittance) and SH [n,16]."""
    g = torch.Generator().manual_seed(int(seed))
    W, L, H = box
    u = torch.rand(n, 3, generator=g, dtype=torch.float64)
    means = torch.stack([(u[:, 0] - 0.5) * W, (u[:, 1] - 0.5) * L, u[:, 2] * H], dim=1)
    lo, hi = math.log(scale_range[0]), math.log(scale_range[1])
    scales = torch.rand(n, 3, generator=g, dtype=torch.float64) * (hi - lo) + lo
    q = torch.randn(n, 4, generator=g, dtype=torch.float64)
    q = q / q.norm(dim=1, keepdim=True)
    logits = torch.randn(n, generator=g, dtype=torch.float64)
    sh = torch.randn(n, 16, generator=g, dtype=torch.float64) * 0.1
    sh[:, 0] += 0.5
    return {k: v.float().to(device) for k, v in
            (("means", means), ("scales", scales), ("rotations", q), ("logits", logits), ("sh", sh))}
