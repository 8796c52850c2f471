"""Parity at full size, on the configurations the benchmark runs.

The sweep (N = 1M Gaussians in 40 x 40 x 10 m, 1024 views of 256 x 256 at
0.2 m, incidence 15-45 deg) is rendered exactly as the benchmark calls it: one
sarr_forward call over the 1024 views, processed in launch groups of 256 views
(cell culling, the tile scan, the fused selection and four-pixel
compositing for the image-only call, the separate kernels for the call with
states). Views
spread over the groups are checked against the CPU oracle: tile lists and
depth orders bit-exact, images and Omega within 1e-4 relative L-inf. The
backward is checked against the oracle's gradients at 1M Gaussians (1e-3
relative per tensor), for one view and for a 16-view batch (cell path).

The high-resolution scene (N = 500k in 60 x 60 x 15 m, scales 0.02-0.3 m,
512 x 512 at 0.1 m, 1024 tiles, 16 views with incidence 15-45 deg) is checked
the same way.

The oracle is given the device's rotation trig (CUDA's cosf/sinf), which
makes its per-Gaussian floats bit-identical to the device's.
"""
import numpy as np
import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import synthetic as S
from oracle import oracle as O

from _helpers import (GRAD_RTOL, IMAGE_RTOL, device_trig, np_scene, oracle_backward,
                      oracle_forward, oview, rel_linf)

pytestmark = pytest.mark.gpu

CAP = 64


def _a256(x):
    return (x + 255) // 256 * 256


def state_tables(states, k, n, T, sbytes):
    """(count [T], list [T,64], sorted [T,64]) of view k from a batch of
    per-view forward states: the index-ordered lists and, through each
    record's list slot, the compositing (Z_r, index) order."""
    base = k * sbytes
    o_count = _a256(4 * n)
    o_list = o_count + _a256(4 * T)
    o_yz = o_list + _a256(4 * T * CAP)
    o_recs = o_yz + _a256(8 * T * CAP)
    count = states[base + o_count: base + o_count + 4 * T].view(torch.int32).cpu().numpy()
    lst = states[base + o_list: base + o_list + 4 * T * CAP].view(torch.int32).view(T, CAP).cpu().numpy()
    recs = states[base + o_recs: base + o_recs + 48 * T * CAP].view(torch.int32).view(T, CAP, 12)
    pos = recs[:, :, 11].cpu().numpy()
    srt = np.full((T, CAP), -1, np.int32)
    for t in range(T):
        c = int(count[t])
        srt[t, :c] = lst[t, pos[t, :c]]
    lst = np.where(np.arange(CAP)[None, :] < count[:, None], lst, -1)
    return count, lst, srt


def _check_view_against_oracle(sc_np, view, count, lst, srt, image, omega=None):
    fw = O.forward(oview(view), sc_np["means"], sc_np["cov6"], sc_np["sigma"], sc_np["sh"],
                   want_omega=omega is not None, trig=device_trig(view))
    np.testing.assert_array_equal(count, fw["counts"])
    np.testing.assert_array_equal(lst, fw["lists"])
    np.testing.assert_array_equal(srt, fw["sorted"])
    assert rel_linf(image, fw["image"]) <= IMAGE_RTOL
    if omega is not None:
        assert rel_linf(omega, fw["omega"]) <= IMAGE_RTOL
    return fw


@pytest.fixture(scope="module")
def sweep():
    sc = S.named_scene("sweep_1m", seed=0, device="cuda")
    return sc, np_scene(sc)


def test_sweep_benchmark_call_matches_oracle(sweep):
    """1024 views in one call, as the benchmark makes it (no states, no
    Omega); then the same call with per-view states, whose lists and depth
    orders are compared bit for bit with the oracle's."""
    sc, s = sweep
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    n = inputs[0].shape[0]
    views_t = S.sweep_views(1024)
    views = [_native.make_view(*v) for v in views_t]
    V, nr = len(views), 256
    T = (nr // 16) ** 2
    ws = torch.empty(_native.workspace_bytes(n, nr, nr, V), dtype=torch.uint8, device="cuda")
    images = torch.empty((V, nr, nr), dtype=torch.float32, device="cuda")
    _native.forward(views, *inputs, images, ws=ws, check_device=True)

    sbytes = _native.state_bytes(n, nr, nr)
    states = torch.empty(V * sbytes, dtype=torch.uint8, device="cuda")
    images2 = torch.empty_like(images)
    _native.forward(views, *inputs, images2, states=states, ws=ws, check_device=True)
    assert torch.equal(images2, images)

    for k in (0, 97, 255, 256 + 131, 767, 1023):
        count, lst, srt = state_tables(states, k, n, T, sbytes)
        assert count.max() == CAP
        img = images[k].contiguous().view(-1).cpu().numpy()
        _check_view_against_oracle(s, views_t[k], count, lst, srt, img)


def test_sweep_group_omega_matches_oracle(sweep):
    """One 256-view launch group with Omega: its images equal those of the
    image-only call bit for bit, and Omega of views in the group matches the
    oracle."""
    sc, s = sweep
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    n = inputs[0].shape[0]
    views_t = S.sweep_views(1024)[:256]
    views = [_native.make_view(*v) for v in views_t]
    V, nr = len(views), 256
    images = torch.empty((V, nr, nr), dtype=torch.float32, device="cuda")
    _native.forward(views, *inputs, images, check_device=True)
    images_om = torch.empty_like(images)
    omega = torch.empty((V, n), dtype=torch.float32, device="cuda")
    _native.forward(views, *inputs, images_om, omega=omega, check_device=True)
    assert torch.equal(images_om, images)
    for k in (5, 200):
        fw = oracle_forward(sc, views_t[k], want_omega=True)
        assert rel_linf(images[k].contiguous().view(-1).cpu().numpy(), fw["image"]) <= IMAGE_RTOL
        assert rel_linf(omega[k].cpu().numpy(), fw["omega"]) <= IMAGE_RTOL


def test_full_size_backward_matches_oracle(sweep):
    """One 1M-Gaussian view: the four dense gradients against the oracle's."""
    sc, s = sweep
    view = S.sweep_views(1024)[11]
    g = torch.randn(256, 256, generator=torch.Generator().manual_seed(3)).cuda()
    got = M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], g, *view)
    ref = oracle_backward(sc, view, g.cpu().numpy())
    for a, b in zip(got, ref):
        assert rel_linf(a.cpu().numpy(), b) <= GRAD_RTOL
    assert int((got[2] != 0).sum()) > 1000


def test_full_size_batched_backward_matches_oracle(sweep):
    """16 views in one backward call (cell culling, views summed; states from
    the forward reused): the summed gradients against the sum of the oracle's
    per-view gradients."""
    sc, s = sweep
    views = S.sweep_views(1024)[::64]
    n = sc["means"].shape[0]
    sbytes = _native.state_bytes(n, 256, 256)
    states = torch.empty(len(views) * sbytes, dtype=torch.uint8, device="cuda")
    M.render_sar_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], views, states=states)
    gimg = torch.randn((len(views), 256, 256), generator=torch.Generator().manual_seed(4)).cuda()
    got = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg, views,
                                        states=states)
    total = None
    for k, v in enumerate(views):
        r = oracle_backward(sc, v, gimg[k].cpu().numpy())
        total = list(r) if total is None else [a + b for a, b in zip(total, r)]
    for a, b in zip(got, total):
        assert rel_linf(a.cpu().numpy(), b) <= GRAD_RTOL


def test_hires_500k_512px_lists_images_gradients():
    """The high-resolution scene: 16 views in one call (cell path, 1024 tiles
    per view): lists and depth orders bit-exact and images within tolerance
    for every view, the summed backward within tolerance."""
    sc = S.named_scene("hires_500k", seed=0, device="cuda")
    s = np_scene(sc)
    views_t = S.hires_views(16)
    views = [_native.make_view(*v) for v in views_t]
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    n = inputs[0].shape[0]
    V, nr = len(views), 512
    T = (nr // 16) ** 2
    sbytes = _native.state_bytes(n, nr, nr)
    states = torch.empty(V * sbytes, dtype=torch.uint8, device="cuda")
    images = torch.empty((V, nr, nr), dtype=torch.float32, device="cuda")
    _native.forward(views, *inputs, images, states=states, check_device=True)
    saturated = 0
    for k in range(V):
        count, lst, srt = state_tables(states, k, n, T, sbytes)
        saturated += int((count == CAP).sum())
        _check_view_against_oracle(s, views_t[k], count, lst, srt,
                                   images[k].contiguous().view(-1).cpu().numpy())
    assert saturated > 0
    gimg = torch.randn((V, nr, nr), generator=torch.Generator().manual_seed(6)).cuda()
    got = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg,
                                        views_t, states=states)
    total = None
    for k, v in enumerate(views_t[:4]):
        r = oracle_backward(sc, v, gimg[k].cpu().numpy())
        total = list(r) if total is None else [a + b for a, b in zip(total, r)]
    part = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg[:4],
                                         views_t[:4])
    for a, b in zip(part, total):
        assert rel_linf(a.cpu().numpy(), b) <= GRAD_RTOL
    # the 16-view sum equals the sum of four 4-view calls
    acc = [torch.zeros_like(t) for t in got]
    for j in range(0, V, 4):
        r = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"],
                                          gimg[j:j + 4], views_t[j:j + 4])
        acc = [a + b for a, b in zip(acc, r)]
    for a, b in zip(got, acc):
        assert rel_linf(a.cpu().numpy(), b.cpu().numpy()) <= 1e-5
