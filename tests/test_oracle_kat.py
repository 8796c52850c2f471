"""Known-answer tests of the CPU oracle (no GPU).

The reference ships no tests, so these pin the oracle with values derived by
hand from the reference formulas (cuda_rasterizer/rasterizer_impl_v2.cu):
a single isotropic Gaussian at the scene centre, whose projection, bbox and
pixel values have closed forms; the index-ordered 64 cap; the stable depth
sort; validity rules; and single-Gaussian gradients.
"""
import math

import numpy as np
import pytest

from oracle import oracle as O

C0 = 0.28209479177387814


def iso_scene(n, s=0.3, sigma=0.8, sh0=1.0, spread=0.0, seed=0):
    rng = np.random.default_rng(seed)
    means = np.zeros((n, 3), np.float32)
    if spread:
        means[:, :2] = rng.uniform(-spread, spread, (n, 2))
    cov6 = np.zeros((n, 6), np.float32)
    cov6[:, :3] = s * s
    sig = np.full(n, sigma, np.float32)
    sh = np.zeros((n, 16), np.float32)
    sh[:, 0] = sh0
    return means, cov6, sig, sh


def test_view_setup_matches_formulas():
    v = O.make_view(radar_z=5000.0, track_angle=30.0, incidence_angle=15.0, azimuth_angle=0.0,
                    range_resolution=0.3, azimuth_resolution=0.3, range_samples=128,
                    azimuth_samples=128)
    vc = O.view_consts(v)
    beta = math.asin(math.sin(math.radians(15.0)))
    assert vc.beta == pytest.approx(beta, rel=1e-6)
    assert vc.Rc == pytest.approx(5000.0 / math.cos(beta), rel=1e-6)
    assert vc.radar_x == pytest.approx(5000.0 * math.tan(beta) * math.sin(math.radians(30)), rel=1e-5)
    assert vc.radar_y == pytest.approx(-5000.0 * math.tan(beta) * math.cos(math.radians(30)), rel=1e-5)
    assert vc.sh_basis[0] == pytest.approx(C0)
    # basis term 3 = C1 cos(theta) with theta = beta (compute_sh_basis_host :299)
    assert vc.sh_basis[3] == pytest.approx(0.4886025119029199 * math.cos(beta), rel=1e-6)


def test_single_isotropic_gaussian_closed_form():
    """A Gaussian at the origin projects to the image centre with an isotropic
    image-plane covariance (s/rho)^2; the pixel value is sigma * gamma * S."""
    s, rho, N = 0.45, 0.3, 64
    v = O.make_view(radar_z=5000.0, track_angle=0.0, incidence_angle=30.0, range_resolution=rho,
                    azimuth_resolution=rho, range_samples=N, azimuth_samples=N)
    means, cov6, sig, sh = iso_scene(1, s=s, sigma=0.8, sh0=1.0)
    fw = O.forward(v, means, cov6, sig, sh)
    f, q = fw["f"], fw["q"]
    r, c = f[0, 0], f[1, 0]
    assert c == pytest.approx(N / 2, abs=1e-4)
    assert r == pytest.approx(N / 2, abs=2e-2)      # R_min/rho - R_c/rho cancels to float rounding
    var = (s / rho) ** 2
    assert f[2, 0] == pytest.approx(var, rel=1e-4)  # cov_rr
    assert f[3, 0] == pytest.approx(var, rel=1e-5)  # cov_cc
    assert abs(f[4, 0]) < 1e-4 * var                 # cov_rc
    # bbox: std = sqrt(rr*cc/det) = 1 -> centre +- 3, floored / ceiled
    assert q[0, 0] == 1
    assert (q[1, 0], q[2, 0]) == (math.floor(r - 3), math.ceil(r + 3))
    assert (q[3, 0], q[4, 0]) == (math.floor(c - 3), math.ceil(c + 3))
    S = 1.0 * C0
    img = fw["image"].reshape(N, N)  # [c][r]
    for (pc, pr) in [(32, 32), (33, 32), (30, 35), (36, 29)]:
        d2 = (pc - c) ** 2 + (pr - r) ** 2
        gamma = math.exp(-0.5 * d2 / var) / (2 * math.pi * var)
        assert img[pc, pr] == pytest.approx(0.8 * gamma * S, rel=2e-4)
    # pixels outside the Gaussian's tiles are exactly zero
    assert img[0, 0] == 0.0
    # one Gaussian: Omega_before is 1 at every pixel it reaches -> mean 1
    assert fw["omega"][0] == pytest.approx(1.0)


def test_validity_rules():
    N = 64
    v = O.make_view(radar_z=5000.0, incidence_angle=30.0, range_samples=N, azimuth_samples=N)
    means, cov6, sig, sh = iso_scene(3)
    sig[1] = 0.0099            # transmittance < 0.01 -> invalid (:351)
    means[2, 0] = 1000.0       # projects far outside the image -> invalid (:405)
    fw = O.forward(v, means, cov6, sig, sh)
    assert list(fw["q"][0]) == [1, 0, 0]
    assert list(fw["q"][1:5, 2]) == [0, 0, 0, 0]  # ranges zeroed for invalid (:431-436)
    assert fw["omega"][1] == 1.0 and fw["omega"][2] == 1.0


def test_cap_keeps_first_64_in_index_order():
    N = 32
    v = O.make_view(radar_z=5000.0, incidence_angle=30.0, range_resolution=0.3,
                    azimuth_resolution=0.3, range_samples=N, azimuth_samples=N)
    means, cov6, sig, sh = iso_scene(100, spread=0.3, seed=1)
    fw = O.forward(v, means, cov6, sig, sh)
    tx = (N + 15) // 16
    counts, lists = fw["counts"], fw["lists"]
    assert counts.max() == 64
    for t in range(counts.size):
        ids = lists[t, :counts[t]]
        assert np.all(np.diff(ids) > 0)  # index order
        # every Gaussian passing the hit test with a smaller index is listed
        tc, tr = t % tx, t // tx
        q = fw["q"]
        hit = [i for i in range(100) if q[0, i] and not (
            q[2, i] < tr * 16 or q[1, i] > min(tr * 16 + 16, N) or q[4, i] < tc * 16
            or q[3, i] > min(tc * 16 + 16, N))]
        assert list(ids) == hit[:64]


def test_depth_sort_is_stable():
    counts = np.array([5], np.int32)
    lists = np.full((1, 64), -1, np.int32)
    lists[0, :5] = [0, 1, 2, 3, 4]
    z = np.array([3.0, 1.0, 3.0, 1.0, 2.0], np.float32)
    s = O.sort_lists(counts, lists, z)
    assert list(s[0, :5]) == [1, 3, 4, 0, 2]


def test_one_tile_class_lists_are_identity():
    """16x16 image, N <= 64 valid Gaussians: the tile list is [0..N-1], the
    case in which the reference's global-id shared-memory indexing happens to
    equal slot indexing."""
    v = O.make_view(radar_z=5000.0, incidence_angle=30.0, range_resolution=0.3,
                    azimuth_resolution=0.3, range_samples=16, azimuth_samples=16)
    means, cov6, sig, sh = iso_scene(40, spread=0.8, seed=3)
    fw = O.forward(v, means, cov6, sig, sh)
    assert fw["q"][0].sum() == 40
    assert fw["counts"][0] == 40
    assert list(fw["lists"][0, :40]) == list(range(40))


def test_single_gaussian_gradients():
    """With one Gaussian T = 1 everywhere, so grad_sigma = sum_p g_p S gamma_p
    = sum_p g_p I_p / sigma and grad_sh_k = sum_p g_p sigma gamma_p b_k."""
    N = 48
    v = O.make_view(radar_z=5000.0, track_angle=20.0, incidence_angle=30.0, range_samples=N,
                    azimuth_samples=N)
    means, cov6, sig, sh = iso_scene(1, s=0.5, sigma=0.6, sh0=1.3)
    fw = O.forward(v, means, cov6, sig, sh)
    rng = np.random.default_rng(0)
    g = rng.standard_normal(N * N).astype(np.float32)
    gm, gc, gs, gsh = O.backward(fw["vc"], fw["f"], sig, fw["counts"], fw["sorted"], g)
    img = fw["image"].astype(np.float64)
    assert gs[0] == pytest.approx(float((g * img).sum() / 0.6), rel=1e-4)
    S = 1.3 * C0
    for k in range(16):
        expect = float((g * img).sum() / S) * fw["vc"].sh_basis[k]
        assert gsh[0, k] == pytest.approx(expect, rel=1e-3, abs=1e-6)
    assert gc[0, 2] == 0 and gc[0, 4] == 0 and gc[0, 5] == 0


def test_empty_inputs():
    v = O.make_view(range_samples=32, azimuth_samples=32)
    z = np.zeros((0, 3), np.float32)
    fw = O.forward(v, z, np.zeros((0, 6), np.float32), np.zeros(0, np.float32),
                   np.zeros((0, 16), np.float32))
    assert fw["image"].shape == (32 * 32,) and not fw["image"].any()
    assert fw["omega"].shape == (0,)
