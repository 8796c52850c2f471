"""Cell culling of multi-view calls (8 views or more, N past the exactly
binned prefix): the tile lists, images, Omega and gradients must equal those of
single-view calls, which bin without cells and match the oracle bit for bit
(test_gpu_parity). Lists and images are compared bitwise."""
import numpy as np
import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import synthetic as S

from _helpers import rel_linf

pytestmark = pytest.mark.gpu


def _a256(x):
    return (x + 255) // 256 * 256


def _state_lists(states, k, n, T, sbytes):
    """(count [T], list [T,64]) of view k from a batch of per-view states."""
    base = k * sbytes
    o_count = _a256(4 * n)
    o_list = o_count + _a256(4 * T)
    count = states[base + o_count: base + o_count + 4 * T].view(torch.int32)
    lst = states[base + o_list: base + o_list + 4 * T * 64].view(torch.int32).view(T, 64)
    return count.cpu().numpy(), lst.cpu().numpy()


def _check_batch_vs_single(sc, views, want_omega):
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    means = inputs[0]
    n = means.shape[0]
    vs = [_native.make_view(*v) for v in views]
    nr, na = views[0][8], views[0][9]
    T = ((nr + 15) // 16) * ((na + 15) // 16)
    sbytes = _native.state_bytes(n, nr, na)
    V = len(vs)
    states = torch.empty(V * sbytes, dtype=torch.uint8, device="cuda")
    images = torch.empty((V, nr, na), dtype=torch.float32, device="cuda")
    omega = torch.empty((V, n), dtype=torch.float32, device="cuda") if want_omega else None
    _native.forward(vs, *inputs, images, omega=omega, states=states, check_device=True)
    one_state = torch.empty(sbytes, dtype=torch.uint8, device="cuda")
    one_img = torch.empty((1, nr, na), dtype=torch.float32, device="cuda")
    one_om = torch.empty((1, n), dtype=torch.float32, device="cuda") if want_omega else None
    for k, v in enumerate(vs):
        _native.forward([v], *inputs, one_img, omega=one_om, states=one_state, check_device=True)
        c1, l1 = _state_lists(one_state, 0, n, T, sbytes)
        cb, lb = _state_lists(states, k, n, T, sbytes)
        np.testing.assert_array_equal(cb, c1)
        used = np.arange(64)[None, :] < c1[:, None]  # slots past the count are unspecified
        np.testing.assert_array_equal(lb[used], l1[used])
        assert torch.equal(images[k], one_img[0])
        if want_omega:
            assert torch.equal(omega[k], one_om[0])
    return images


@pytest.mark.parametrize("want_omega", [False, True])
def test_cell_culling_lists_images_omega(want_omega):
    sc = {k: v.cuda() for k, v in S.make_scene(200000, (40.0, 40.0, 10.0), (0.05, 0.5), seed=51).items()}
    views = S.sweep_views(96)[::8]  # 12 views, incidence 15-45 deg
    _check_batch_vs_single(sc, views, want_omega)


def test_many_view_launch_matches_single_views():
    """20 views in one launch group: the tile scan, the four-pixel render
    layout and the cell path give each view the lists, image and Omega of a
    single-view call."""
    sc = {k: v.cuda() for k, v in S.make_scene(150000, (40.0, 40.0, 10.0), (0.05, 0.5), seed=57).items()}
    views = S.sweep_views(160)[::8]  # 20 views
    _check_batch_vs_single(sc, views, want_omega=True)


def _edge_scene():
    """Non-finite centres, near-singular and very elongated covariances (no
    cell), transmittances below 0.01, in a flat scene (zero z extent)."""
    g = torch.Generator().manual_seed(52)
    sc = S.make_scene(120000, (30.0, 30.0, 0.0), (0.02, 0.6), seed=53)
    n = sc["means"].shape[0]
    idx = torch.randperm(n, generator=g)
    sc["means"][idx[:50]] = float("nan")
    sc["means"][idx[50:60], 0] = float("inf")
    k = 3000
    s = torch.exp(torch.empty(k, 3).uniform_(-7.0, 1.0, generator=g))
    q = torch.randn(k, 4, generator=g)
    q = q / q.norm(dim=1, keepdim=True)
    R = S.quat_to_rot(q.double())
    cov = (R @ torch.diag_embed((s * s).double()) @ R.transpose(1, 2)).float()
    sc["cov33"][idx[100:100 + k]] = cov
    sc["cov6"][idx[100:100 + k]] = S.cov33_to_cov6(cov)
    sc["sigma"][idx[5000:9000]] = 0.005
    return {key: v.cuda() for key, v in sc.items()}


def test_cell_culling_edge_cases():
    """Non-finite centres, near-singular and very elongated covariances (no
    cell), transmittances below 0.01, and a flat scene (zero z extent)."""
    sc = _edge_scene()
    views = S.sweep_views(64, rho=0.15)[::7]  # 10 views
    _check_batch_vs_single(sc, views, want_omega=True)


@pytest.mark.parametrize("scene", ["sweep", "edge"])
def test_fused_select_render_matches_separate_kernels(scene):
    """Image-only calls of 16 views or more select and composite each tile in
    one kernel (the tile's list and records stay in shared memory); the same
    call with per-view states runs the separate selection and compositing
    kernels. The images agree bit for bit whatever the workspace holds, and
    equal those of single-view calls."""
    if scene == "sweep":
        sc = {k: v.cuda() for k, v in
              S.make_scene(150000, (40.0, 40.0, 10.0), (0.05, 0.5), seed=58).items()}
        views = S.sweep_views(160)[::8]  # 20 views
    else:
        sc = _edge_scene()
        views = S.sweep_views(66, rho=0.15)[::3]  # 22 views
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    n = inputs[0].shape[0]
    vs = [_native.make_view(*v) for v in views]
    V, nr, na = len(vs), views[0][8], views[0][9]
    sbytes = _native.state_bytes(n, nr, na)
    states = torch.empty(V * sbytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty((V, nr, na), dtype=torch.float32, device="cuda")
    _native.forward(vs, *inputs, ref, states=states, check_device=True)
    wsb = _native.workspace_bytes(n, nr, na, V)
    for fill in ("zero", "ff", "random"):
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        if fill == "ff":
            ws.fill_(255)
        elif fill == "random":
            ws.random_(0, 256, generator=torch.Generator(device="cuda").manual_seed(13))
        imgs = torch.full((V, nr, na), float("nan"), device="cuda")
        _native.forward(vs, *inputs, imgs, ws=ws, check_device=True)
        assert torch.equal(imgs, ref)
    one = torch.empty((1, nr, na), dtype=torch.float32, device="cuda")
    for k in (0, V // 2, V - 1):
        _native.forward([vs[k]], *inputs, one, check_device=True)
        assert torch.equal(one[0], ref[k])


@pytest.mark.parametrize("nviews", [10, 20, 40])
def test_cell_culling_backward_equals_sum_of_single_views(nviews):
    """10 views: the per-tile pass with one pixel per lane; 20 views: four
    pixels per lane (launches of 16 views or more), the tile's records in
    four parts; 40 views: four pixels per lane, one part (launches of 32
    views or more). Single views use the first."""
    sc = {k: v.cuda() for k, v in S.make_scene(100000, (40.0, 40.0, 10.0), (0.05, 0.5), seed=54).items()}
    views = S.sweep_views(8 * nviews)[::8]
    batch = M.render_sar_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], views)
    for k, v in enumerate(views):
        img, _ = M.render_sar(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], *v)
        assert torch.equal(batch[k], img)
    gimg = torch.randn_like(batch)
    grads = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg, views)
    single = [M.render_sar_backward(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg[k], *v)
              for k, v in enumerate(views)]
    for i in range(4):
        total = sum(s[i] for s in single)
        assert rel_linf(grads[i].cpu().numpy(), total.cpu().numpy()) <= 1e-5
    # the backward reusing the forward's states (sparse rectangles) agrees
    n = sc["means"].shape[0]
    sbytes = _native.state_bytes(n, views[0][8], views[0][9])
    states = torch.empty(len(views) * sbytes, dtype=torch.uint8, device="cuda")
    batch2 = M.render_sar_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], views, states=states)
    assert torch.equal(batch2, batch)
    grads3 = M.render_sar_backward_batched(sc["means"], sc["cov6"], sc["sigma"], sc["sh"], gimg, views,
                                           states=states)
    for i in range(4):
        assert torch.equal(grads3[i], grads[i])


@pytest.mark.parametrize("nviews", [1, 10])
def test_results_do_not_depend_on_workspace_contents(nviews):
    """The workspace and the state buffers are caller memory of any content:
    zero-filled, 0xFF-filled and random-filled buffers give identical images,
    Omega and lists (the cell path for 10 views, the per-view path for 1)."""
    n = 100000
    sc = {k: v.cuda() for k, v in S.make_scene(n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=55).items()}
    views = S.sweep_views(80)[::8][:nviews]
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    vs = [_native.make_view(*v) for v in views]
    wsb = _native.workspace_bytes(n, 256, 256, nviews, _native.SARR_FLAG_OMEGA)
    sbytes = _native.state_bytes(n, 256, 256)
    out = {}
    for fill in ("zero", "ff", "random"):
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        st = torch.zeros(nviews * sbytes, dtype=torch.uint8, device="cuda")
        if fill == "ff":
            ws.fill_(255)
            st.fill_(255)
        elif fill == "random":
            g = torch.Generator(device="cuda").manual_seed(9)
            ws.random_(0, 256, generator=g)
            st.random_(0, 256, generator=g)
        imgs = torch.empty((nviews, 256, 256), device="cuda")
        om = torch.empty((nviews, n), device="cuda")
        _native.forward(vs, *inputs, imgs, omega=om, states=st, ws=ws, check_device=True)
        lists = [_state_lists(st, k, n, 256, sbytes) for k in range(nviews)]
        out[fill] = (imgs, om, lists)
    for fill in ("ff", "random"):
        assert torch.equal(out[fill][0], out["zero"][0])
        assert torch.equal(out[fill][1], out["zero"][1])
        for (c0, l0), (c1, l1) in zip(out["zero"][2], out[fill][2]):
            np.testing.assert_array_equal(c1, c0)
            used = np.arange(64)[None, :] < c0[:, None]
            np.testing.assert_array_equal(l1[used], l0[used])


@pytest.mark.parametrize("nviews,with_states", [(1, False), (1, True), (10, False), (10, True)])
def test_backward_does_not_depend_on_workspace_contents(nviews, with_states):
    """The backward reads nothing of the caller's workspace (and, without the
    forward's states, of its own selection scratch) that it did not write:
    zero-filled, 0xFF-filled and random-filled workspaces give bitwise equal
    gradients, single view (per-view path) and 10 views (cell path)."""
    n = 100000
    sc = {k: v.cuda() for k, v in S.make_scene(n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=56).items()}
    views = S.sweep_views(80)[::8][:nviews]
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    vs = [_native.make_view(*v) for v in views]
    wsb = _native.workspace_bytes(n, 256, 256, nviews, 0)
    sbytes = _native.state_bytes(n, 256, 256)
    g = torch.Generator(device="cuda").manual_seed(11)
    gimg = torch.randn((nviews, 256, 256), device="cuda", generator=g)
    states = None
    if with_states:
        states = torch.empty(nviews * sbytes, dtype=torch.uint8, device="cuda")
        imgs = torch.empty((nviews, 256, 256), device="cuda")
        _native.forward(vs, *inputs, imgs, states=states, check_device=True)
    out = {}
    for fill in ("zero", "ff", "random"):
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        if fill == "ff":
            ws.fill_(255)
        elif fill == "random":
            ws.random_(0, 256, generator=torch.Generator(device="cuda").manual_seed(12))
        grads = [torch.full((n, c), float("nan"), device="cuda") for c in (3, 6, 1, 16, 1)]
        _native.backward(vs, *inputs, gimg, grads[0], grads[1], _native.SARR_COV6, grads[2].view(n),
                         grads[3], grad_norm=grads[4].view(n), states=states, ws=ws, check_device=True)
        out[fill] = grads
    for fill in ("ff", "random"):
        for a, b in zip(out[fill], out["zero"]):
            assert torch.equal(a, b)
