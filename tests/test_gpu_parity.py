"""Parity of the CUDA library (called through its C ABI via the drop-in
modules) with the CPU oracle, on seeded synthetic scenes and edge cases.

The oracle is given the GPU's rotation trig values (CUDA's cosf/sinf), which
makes its per-Gaussian floats, bboxes, tile lists and depth orders
bit-identical to the GPU's: those are compared exactly, both end to end and by
feeding the GPU's own validity/bbox integers into the oracle's list builder.
Images / Omega: 1e-4 relative L-inf; gradients: 1e-3 relative per tensor.
"""
import numpy as np
import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import rasterizer_autograd as RA
from cuda_rasterizer import synthetic as S
from oracle import oracle as O

from _helpers import (GRAD_RTOL, IMAGE_RTOL, device_trig, gpu_forward, gpu_lists, gpu_preprocess,
                      image_flat, np_scene, oracle_backward, oracle_forward, oview, rel_linf, scene)

pytestmark = pytest.mark.gpu

VIEWS = {
    "cpu": S.cpu_view(),
    "train": S.training_views(4)[1],
    "sweep": S.sweep_views(8)[5],
    "odd": S.view_tuple(47.0, 25.0, 0.25, 100)[:8] + (100, 72),
}
CASES = [("cpu_1k", "cpu"), ("cpu_1k", "odd"), (20000, "train"), (50000, "sweep"), (90000, "sweep")]


def _check_lists(sc, view):
    f, q = gpu_preprocess(sc, view)
    cnt, lst, srt, scnt, slst, ssrt = gpu_lists(sc, view)
    nr, na = view[8], view[9]
    oc, ol = O.tile_lists(nr, na, q, shadow=False)
    np.testing.assert_array_equal(cnt, oc)
    np.testing.assert_array_equal(lst, ol)
    np.testing.assert_array_equal(srt, O.sort_lists(oc, ol, f[11]))
    osc, osl = O.tile_lists(nr, na, q, shadow=True)
    np.testing.assert_array_equal(scnt, osc)
    np.testing.assert_array_equal(slst, osl)
    np.testing.assert_array_equal(ssrt, O.sort_lists(osc, osl, f[11]))
    return f, q, (cnt, lst, srt)


@pytest.mark.parametrize("name,vk", CASES)
def test_tile_lists_bit_exact(name, vk):
    sc = scene(name, seed=0)
    view = VIEWS[vk]
    f, q, (cnt, lst, srt) = _check_lists(sc, view)
    fw = oracle_forward(sc, view, want_omega=False)
    np.testing.assert_array_equal(q, fw["q"])
    for row in range(13):  # bit-identical floats on every Gaussian
        assert np.array_equal(f[row].view(np.uint32), fw["f"][row].view(np.uint32)), O.F_ROWS[row]
    # and the end-to-end lists of the oracle are the same
    np.testing.assert_array_equal(cnt, fw["counts"])
    np.testing.assert_array_equal(lst, fw["lists"])
    np.testing.assert_array_equal(srt, fw["sorted"])


@pytest.mark.parametrize("name,vk", CASES)
def test_forward_image_and_omega(name, vk):
    sc = scene(name, seed=1)
    view = VIEWS[vk]
    img, om = gpu_forward(sc, view)
    assert img.shape == (view[8], view[9])
    fw = oracle_forward(sc, view)
    assert rel_linf(image_flat(img), fw["image"]) <= IMAGE_RTOL
    assert rel_linf(om.cpu().numpy(), fw["omega"]) <= IMAGE_RTOL
    assert np.abs(image_flat(img)).max() > 0


@pytest.mark.parametrize("name,vk", CASES)
def test_backward_gradients(name, vk):
    sc = scene(name, seed=2)
    view = VIEWS[vk]
    g = torch.randn(view[8], view[9], generator=torch.Generator().manual_seed(5)).cuda()
    gm, gc, gs, gsh = M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g, *view)
    ref = oracle_backward(sc, view, g.cpu().numpy())
    for got, want in zip((gm, gc, gs, gsh), ref):
        assert rel_linf(got.cpu().numpy(), want) <= GRAD_RTOL
    assert torch.all(gc[:, [2, 4, 5]] == 0)


def test_autograd_matches_functional_api():
    sc = scene("cpu_1k", seed=3)
    view = VIEWS["cpu"]
    means = sc["means"].clone().requires_grad_(True)
    cov = sc["cov33"].clone().requires_grad_(True)
    op = sc["sigma"].clone().requires_grad_(True)
    sh_full = sc["sh"].clone()
    sh = sh_full.requires_grad_(True)
    rast = RA.SARRasterizer(*view)
    img = rast(means, cov, op, sh)
    img_ref, _ = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], *view)
    assert torch.equal(img, img_ref)
    g = torch.randn_like(img)
    img.backward(g)
    gm, gc, gs, gsh = M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g, *view)
    assert torch.equal(means.grad, gm)
    assert torch.equal(op.grad, gs)
    assert torch.equal(sh.grad, gsh)
    assert torch.equal(cov.grad, RA.cov_6_to_3x3(gc))
    # expanded gradients (image.sum()) are read correctly
    means.grad = None
    rast(means, cov, op, sh).sum().backward()
    gm1, *_ = M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"],
                                     torch.ones_like(img), *view)
    assert torch.equal(means.grad, gm1)


def test_sh_column_slice_reads_active_coefficients_only():
    sc = scene("cpu_1k", seed=4)
    view = VIEWS["cpu"]
    wide = sc["sh"].clone()
    wide[:, 4:] = 0.0
    full = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], wide, *view)[0]
    sl = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], wide[:, :4], *view)[0]
    assert torch.equal(full, sl)
    noisy = sc["sh"].clone()  # nonzero inactive columns are ignored by the slice
    sl2 = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], noisy[:, :4], *view)[0]
    ref = oracle_forward(sc, view, want_omega=False, sh_k=4, sh=noisy[:, :4].cpu().numpy())
    assert rel_linf(image_flat(sl2), ref["image"]) <= IMAGE_RTOL


def test_cov33_and_cov6_paths_identical():
    sc = scene(20000, seed=6)
    view = VIEWS["train"]
    a = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], *view)
    b = M.render_sar(sc["means"], sc["cov33"], sc["sigma"], sc["sh"], *view)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_batched_equals_single_and_deterministic():
    sc = scene(20000, seed=7)
    views = S.training_views(5)
    batch, om = M.render_sar_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], views,
                                     want_omega=True)
    for k, v in enumerate(views):
        img, o1 = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], *v)
        assert torch.equal(batch[k], img)
        assert torch.equal(om[k], o1)
    again = M.render_sar_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], views)
    assert torch.equal(again, batch)
    g = torch.randn_like(batch)
    grads = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g, views)
    grads2 = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g, views)
    single = [M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g[k], *v)
              for k, v in enumerate(views)]
    for i in range(4):
        assert torch.equal(grads[i], grads2[i])
        total = sum(s[i] for s in single)
        assert rel_linf(grads[i].cpu().numpy(), total.cpu().numpy()) <= 1e-5


def test_grad_norm_and_accumulate():
    sc = scene(20000, seed=8)
    views = S.training_views(2)
    g = torch.randn(2, 128, 128, device="cuda")
    gm, gc, gs, gsh, gn = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"],
                                                         g, views, grad_norm=True)
    assert torch.allclose(gn, gm.norm(dim=1), rtol=1e-6, atol=0)
    means, cov, layout, sigma, sh, st, k = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    v = [_native.make_view(*views[0])]
    acc = [t.clone() for t in (gm, gc, gs, gsh)]
    _native.backward(v, means, cov, layout, sigma, sh, st, k, g[0].contiguous(), *acc[:2],
                     _native.SARR_COV6, acc[2], acc[3], accumulate=True)
    one = M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g[0], *views[0])
    for a, b, o in zip(acc, (gm, gc, gs, gsh), one):
        assert rel_linf(a.cpu().numpy(), (b + o).cpu().numpy()) <= 1e-6


def test_edge_cases():
    view = VIEWS["cpu"]
    # no Gaussians
    e = {k: torch.zeros((0,) + tuple(s), device="cuda") for k, s in
         (("means", (3,)), ("cov6", (6,)), ("sigma", ()), ("sh", (16,)))}
    img, om = M.render_sar(e["means"], e["cov6"], e["sigma"], e["sh"], *view)
    assert img.shape == (128, 128) and not img.any() and om.shape == (0,)
    sc = scene("cpu_1k", seed=9)
    # every Gaussian below the transmittance threshold
    img, om = M.render_sar(sc["means"], sc["cov6"], torch.full_like(sc["sigma"], 0.005), sc["sh"], *view)
    assert not img.any() and torch.all(om == 1.0)
    # degenerate covariances (det < EPSILON) render nothing but stay listed
    z = torch.zeros_like(sc["cov6"])
    img, om = M.render_sar(sc["means"], z, sc["sigma"], sc["sh"], *view)
    ref = oracle_forward({**sc, "cov6": z}, view)
    assert rel_linf(image_flat(img), ref["image"]) <= IMAGE_RTOL
    assert rel_linf(om.cpu().numpy(), ref["omega"]) <= IMAGE_RTOL
    # a single 16x16 tile with N <= 64: the list is 0..N-1
    small = {k: v[:40] for k, v in sc.items()}
    small["means"] = small["means"] * 0.05
    one = S.view_tuple(30.0, 15.0, 0.3, 16)
    cnt, lst, *_ = gpu_lists(small, one)
    assert cnt[0] == 40 and list(lst[0, :40]) == list(range(40))
    img, om = M.render_sar(small["means"], small["cov6"], small["sigma"], small["sh"], *one)
    ref = oracle_forward(small, one)
    assert rel_linf(image_flat(img), ref["image"]) <= IMAGE_RTOL


def test_saturation_skip_is_exact():
    """After the exactly binned prefix, Gaussians whose conservative bbox only
    reaches tiles already holding 64 hits skip the covariance projection. A
    dense central cluster (saturating its tiles inside the prefix) followed by
    spread-out, strongly anisotropic and near-singular Gaussians around the
    saturation boundary must still give the oracle's lists bit for bit."""
    g = torch.Generator().manual_seed(21)
    n1, n2 = 30000, 60000  # past the exactly binned prefix (64 chunks of 1024)
    core = S.make_scene(n1, (6.0, 6.0, 2.0), (0.05, 0.3), seed=22)
    rest = S.make_scene(n2, (30.0, 30.0, 8.0), (0.05, 0.5), seed=23)
    # anisotropic tail: per-axis scales from 1e-3 to 2 m (condition numbers up to 4e6)
    k = n2 // 3
    s = torch.exp(torch.empty(k, 3).uniform_(-6.9, 0.7, generator=g))
    q = torch.randn(k, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    R = S.quat_to_rot(q.double())
    cov = (R @ torch.diag_embed((s * s).double()) @ R.transpose(1, 2)).float()
    rest["cov33"][:k] = cov
    rest["cov6"][:k] = S.cov33_to_cov6(cov)
    sc = {key: torch.cat([core[key], rest[key]]).cuda() for key in core}
    for view in (S.sweep_views(8, samples=128)[2], S.training_views(3)[1]):
        f, q_, (cnt, lst, srt) = _check_lists(sc, view)
        fw = oracle_forward(sc, view)
        np.testing.assert_array_equal(cnt, fw["counts"])
        np.testing.assert_array_equal(lst, fw["lists"])
        np.testing.assert_array_equal(srt, fw["sorted"])
        img, om = gpu_forward(sc, view)
        assert rel_linf(image_flat(img), fw["image"]) <= IMAGE_RTOL
        assert rel_linf(om.cpu().numpy(), fw["omega"]) <= IMAGE_RTOL


@pytest.mark.parametrize("npx,rho", [(640, 0.08), (1024, 0.05)])
def test_saturation_skip_on_large_tile_grids(npx, rho):
    """The skipping binner keeps per-warp tile counters up to 2048 tiles per
    list and switches to CTA-wide counters beyond. 640 px (1600 tiles): the
    image-only forward (one list) takes the per-warp path and the debug lists
    (image and shadow list) the CTA-wide one; 1024 px (4096 tiles): CTA-wide
    for both. Lists bit-exact, images within tolerance."""
    sc = {k: v.cuda() for k, v in S.make_scene(90000, (40.0, 40.0, 6.0), (0.05, 0.4), seed=31).items()}
    view = S.view_tuple(33.0, 21.0, rho, npx)
    f, q, (cnt, lst, srt) = _check_lists(sc, view)
    assert cnt.max() == 64
    fw = oracle_forward(sc, view, want_omega=False)
    np.testing.assert_array_equal(cnt, fw["counts"])
    np.testing.assert_array_equal(lst, fw["lists"])
    img = RA.SARRasterizer(*view)(sc["means"], sc["cov33"], sc["sigma"], sc["sh"])
    torch.cuda.synchronize()
    assert rel_linf(image_flat(img), fw["image"]) <= IMAGE_RTOL


@pytest.mark.parametrize("view_idx", [3, 700])
def test_full_size_sweep_view(view_idx):
    """N = 1M Gaussians, 256 x 256 at 0.2 m (the sweep workload): lists
    bit-exact and image within tolerance against the oracle."""
    sc = scene("sweep_1m", seed=0)
    view = S.sweep_views(1024)[view_idx]
    f, q, (cnt, lst, srt) = _check_lists(sc, view)
    assert cnt.max() == 64
    img, _ = gpu_forward(sc, view)
    vc = O.view_consts(oview(view), device_trig(view))
    s = np_scene(sc)
    ref_img = O.render(vc, f, s["sigma"], cnt, srt)
    # the oracle's render, fed with the GPU's projections and lists
    assert rel_linf(image_flat(img), ref_img) <= IMAGE_RTOL
    fw = oracle_forward(sc, view, want_omega=False)
    assert rel_linf(image_flat(img), fw["image"]) <= IMAGE_RTOL


def test_device_error_word_clear():
    sc = scene("cpu_1k", seed=10)
    img, om = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], *VIEWS["cpu"], False, True)
    assert img.shape == (128, 128)


def test_package_render_sar_and_settings_surface():
    """cuda_rasterizer.render_sar(GaussianDataGPU, H, W) (the reference's
    cuda_rasterizer/__init__.py:147-186) and render_sar_with_settings
    (rasterizer_impl_v2.cu:1664-1699) against the oracle."""
    import cuda_rasterizer as CR
    sc = scene("cpu_1k", seed=11)
    view = VIEWS["odd"]
    assert CR.CUDA_AVAILABLE is True
    host = CR.GaussianDataCPU(sc["means"].cpu(), sc["cov6"].cpu(), sc["sigma"].cpu(), sc["sh"].cpu(),
                              (view[0], view[1], view[2]), view[3], view[4], view[5], view[6],
                              view[7], view[8], view[9])
    data = host.to_device(torch.device("cuda"))
    (img, om), aux = CR.render_sar(data, 512, 512)
    assert aux == {} and img.shape == (view[8], view[9]) and om.shape == (1000,)
    fw = oracle_forward(sc, view)
    assert rel_linf(image_flat(img), fw["image"]) <= IMAGE_RTOL
    assert rel_linf(om.cpu().numpy(), fw["omega"]) <= IMAGE_RTOL
    settings = M.SARRasterizationSettings(
        n_gaussians=1000, radar_x=view[0], radar_y=view[1], radar_z=view[2], track_angle=view[3],
        incidence_angle=view[4], azimuth_angle=view[5], range_resolution=view[6],
        azimuth_resolution=view[7], range_samples=view[8], azimuth_samples=view[9])
    img2, om2 = M.render_sar_with_settings(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], settings)
    assert torch.equal(img2, img) and torch.equal(om2, om)
