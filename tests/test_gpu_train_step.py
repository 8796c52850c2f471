"""The native Adam step and the view-parallel training step on one GPU.

sarr_adam_step is compared with torch.optim.Adam (parameter groups with their
own learning rates, three steps); bucketed calls over sub-ranges must give the
same bits as one call. ViewParallelTrainer's step is compared with the same
step composed from the drop-in modules and torch.optim.Adam: producer,
batched forward, CombinedLoss gradient, batched backward, sigmoid chain, Adam.
"""
import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import multiview
from cuda_rasterizer import synthetic as S

from _helpers import rel_linf

pytestmark = pytest.mark.gpu


def test_adam_step_matches_torch_adam():
    g = torch.Generator(device="cuda").manual_seed(81)
    sizes = (3000, 1000, 16000)
    lrs = (1e-3, 5e-3, 1e-5)
    params = [torch.randn(s, device="cuda", generator=g) for s in sizes]
    ref = [p.clone().requires_grad_(True) for p in params]
    opt = torch.optim.Adam([{"params": [r], "lr": lr} for r, lr in zip(ref, lrs)])
    flat = torch.cat(params)
    m = torch.zeros_like(flat)
    v = torch.zeros_like(flat)
    ends = [sum(sizes[:i + 1]) for i in range(3)]
    segs = list(zip(ends, lrs))
    for step in range(1, 4):
        grads = [torch.randn(s, device="cuda", generator=g) for s in sizes]
        for r, gr in zip(ref, grads):
            r.grad = gr.clone()
        opt.step()
        _native.adam_step(flat, torch.cat(grads), m, v, segs, step)
    want = torch.cat([r.detach() for r in ref])
    assert torch.allclose(flat, want, rtol=1e-6, atol=1e-7)
    exp_avg = torch.cat([opt.state[r]["exp_avg"] for r in ref])
    assert torch.allclose(m, exp_avg, rtol=1e-5, atol=1e-7)


def test_adam_step_buckets_equal_one_call():
    g = torch.Generator(device="cuda").manual_seed(82)
    total = 10_003
    p0 = torch.randn(total, device="cuda", generator=g)
    grad = torch.randn(total, device="cuda", generator=g)
    segs = [(4000, 1e-2), (total, 1e-4)]
    a, ma, va = p0.clone(), torch.zeros(total, device="cuda"), torch.zeros(total, device="cuda")
    _native.adam_step(a, grad, ma, va, segs, 1)
    b, mb, vb = p0.clone(), torch.zeros(total, device="cuda"), torch.zeros(total, device="cuda")
    for lo, hi in ((0, 2048), (2048, 6144), (6144, total)):
        sub = [(max(0, min(e, hi) - lo), lr) for e, lr in segs if e > lo]
        _native.adam_step(b[lo:hi], grad[lo:hi], mb[lo:hi], vb[lo:hi], sub, 1)
    assert torch.equal(a, b) and torch.equal(ma, mb) and torch.equal(va, vb)


def _scene_params(n, seed):
    g = torch.Generator().manual_seed(seed)
    means = (torch.rand((n, 3), generator=g) - 0.5) * torch.tensor([20.0, 20.0, 0.0]) \
        + torch.tensor([0.0, 0.0, 3.0]) * torch.rand((n, 1), generator=g)
    scales = torch.rand((n, 3), generator=g) * 2.3 - 3.0  # log-scales, 0.05-0.5 m
    rot = torch.randn((n, 4), generator=g)
    rot = rot / rot.norm(dim=1, keepdim=True)
    logits = torch.randn((n,), generator=g)
    sh = torch.randn((n, 16), generator=g) * 0.1
    sh[:, 0] += 0.5
    return [t.cuda() for t in (means, scales, rot, logits, sh)]


def test_trainer_step_matches_composed_step():
    n = 20000
    means, scales, rot, logits, sh = _scene_params(n, 83)
    views_t = S.training_views(8)
    views = [_native.make_view(*v) for v in views_t]
    tgt = S.named_scene("target_20k", seed=1, device="cuda")
    targets = M.render_sar_batched(tgt["means"], tgt["cov6"], tgt["sigma"], tgt["sh"], views_t)
    lr = 1e-3
    tr = multiview.ViewParallelTrainer(means, scales, rot, logits, sh, lr=lr, buckets=3)

    p_means = means.clone().requires_grad_(True)
    p_logits = logits.clone().requires_grad_(True)
    p_sh = sh.clone().requires_grad_(True)
    opt = torch.optim.Adam([{"params": [p_means], "lr": lr}, {"params": [p_logits], "lr": lr},
                            {"params": [p_sh], "lr": lr * 0.01}])
    for _ in range(2):
        losses = tr.step(views, targets)
        cov6, sigma = _native.gaussian_params(scales, rot, p_logits.detach(), _native.SARR_COV6)
        imgs = M.render_sar_batched(p_means.detach(), cov6, sigma, p_sh.detach(), views_t)
        ref_losses, gimg = _native.combined_loss(imgs, targets, 1.0, 0.2, 5, "plain")
        gm, _, gs, gsh = M.render_sar_backward_batched(p_means.detach(), cov6, sigma,
                                                       p_sh.detach(), gimg, views_t)
        p_means.grad = gm
        p_logits.grad = gs * sigma * (1.0 - sigma)
        p_sh.grad = gsh
        opt.step()
        assert torch.allclose(losses, ref_losses, rtol=1e-6, atol=0)
    torch.cuda.synchronize()
    for got, want in ((tr.means, p_means), (tr.logits, p_logits), (tr.sh, p_sh)):
        assert rel_linf(got.cpu().numpy(), want.detach().cpu().numpy()) <= 1e-6
    moved = (tr.means - means).abs().max().item()
    assert moved > 1e-4  # the step moved the means (lr 1e-3)


@pytest.mark.parametrize("nviews", [1, 10])
def test_split_backward_equals_single_call(nviews):
    """sarr_backward with SARR_FLAG_TILES_ONLY followed by sarr_backward_scatter
    over disjoint Gaussian ranges (boundaries not on warp multiples) writes the
    same gradient bits as one sarr_backward call."""
    n = 150_000
    sc = {k: v.cuda() for k, v in S.make_scene(n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=84).items()}
    views_t = S.sweep_views(80)[::8][:nviews]
    views = [_native.make_view(*v) for v in views_t]
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    g = torch.randn((nviews, 256, 256), generator=torch.Generator().manual_seed(85)).cuda()
    ws = torch.empty(_native.workspace_bytes(n, 256, 256, nviews), dtype=torch.uint8, device="cuda")

    def grads():
        return [torch.full((n, 3), float("nan"), device="cuda"), torch.full((n, 6), float("nan"), device="cuda"),
                torch.full((n,), float("nan"), device="cuda"), torch.full((n, 16), float("nan"), device="cuda"),
                torch.full((n,), float("nan"), device="cuda")]

    a = grads()
    _native.backward(views, *inputs, g, a[0], a[1], _native.SARR_COV6, a[2], a[3], grad_norm=a[4], ws=ws)
    b = grads()
    _native.backward(views, *inputs, g, b[0], b[1], _native.SARR_COV6, b[2], b[3], ws=ws,
                     tiles_only=True)
    assert torch.isnan(b[0]).all()  # the per-tile pass writes no rows
    for lo, hi in ((0, 1000), (1000, 77_777), (77_777, n)):
        _native.backward_scatter(views, n, lo, hi, b[0], b[1], _native.SARR_COV6, b[2], b[3], ws,
                                 grad_norm=b[4])
    torch.cuda.synchronize()
    for x, y in zip(a, b):
        assert torch.equal(x, y)
    # the same rows into arrays that hold only the range (SARR_FLAG_RANGE_ROWS)
    lo, hi = 1000, 77_777
    r = [t[:hi - lo].clone().fill_(float("nan")) for t in grads()]
    _native.backward_scatter(views, n, lo, hi, r[0], r[1], _native.SARR_COV6, r[2], r[3], ws,
                             grad_norm=r[4], range_rows=True)
    torch.cuda.synchronize()
    for x, y in zip(a, r):
        assert torch.equal(x[lo:hi], y)


def test_adam_ranges_equal_per_range_calls():
    g = torch.Generator(device="cuda").manual_seed(86)
    total = 20_000
    p0 = torch.randn(total, device="cuda", generator=g)
    grad = torch.randn(total, device="cuda", generator=g)
    ranges = [(0, 3000, 1e-3), (12_000, 13_000, 5e-3), (16_000, 19_997, 1e-5)]
    a, ma, va = p0.clone(), torch.zeros(total, device="cuda"), torch.zeros(total, device="cuda")
    for lo, hi, lr in ranges:
        _native.adam_step(a[lo:hi], grad[lo:hi], ma[lo:hi], va[lo:hi], [(hi - lo, lr)], 2)
    b, mb, vb = p0.clone(), torch.zeros(total, device="cuda"), torch.zeros(total, device="cuda")
    import ctypes
    k = len(ranges)
    # the gradients of the ranges packed back to back in another array
    packed = torch.cat([grad[lo:hi] for lo, hi, _ in ranges])
    gb = [0, 3000, 4000]
    st = _native.lib().sarr_adam_step_ranges(
        k, (ctypes.c_int64 * k)(*[r[0] for r in ranges]), (ctypes.c_int64 * k)(*[r[1] for r in ranges]),
        (ctypes.c_int64 * k)(*gb), (ctypes.c_float * k)(*[r[2] for r in ranges]),
        ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(packed.data_ptr()), ctypes.c_void_p(mb.data_ptr()),
        ctypes.c_void_p(vb.data_ptr()), 0.9, 0.999, 1e-8, 2,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(ma, mb) and torch.equal(va, vb)


def test_densifying_trainer_sh_ramp_and_densification():
    """DensifyingTrainer: (1) at SH degree d only the first (d + 1)^2
    coefficients are rendered and trained, the others keep their values;
    (2) densification runs on the due iterations from the step's summed means
    gradient, the new set is densify_and_prune_tensors' output, and that step
    updates nothing; (3) a densification that changes nothing restarts Adam:
    one update from zero moments."""
    from cuda_rasterizer import densify
    n = 20000
    means, scales, rot, logits, sh = _scene_params(n, 84)
    views_t = S.training_views(8)
    views = [_native.make_view(*v) for v in views_t]
    tgt = S.named_scene("target_20k", seed=1, device="cuda")
    targets = M.render_sar_batched(tgt["means"], tgt["cov6"], tgt["sigma"], tgt["sh"], views_t)
    # clone every Gaussian of norm(scale) < 1 m with a nonzero gradient
    dt = multiview.DensifyingTrainer(means, scales, rot, logits, sh, buckets=1, densify_interval=3,
                                     grad_threshold=0.0, size_threshold=1.0, sh_interval=2)
    dt.step(views, targets)
    dt.step(views, targets)  # iterations 0 and 1: degree 0
    torch.cuda.synchronize()
    assert torch.equal(dt.tr.sh[:, 1:], sh[:, 1:])
    assert not torch.equal(dt.tr.sh[:, 0], sh[:, 0])
    dt.step(views, targets)  # iteration 2: degree 1
    torch.cuda.synchronize()
    assert torch.equal(dt.tr.sh[:, 4:], sh[:, 4:])
    assert not torch.equal(dt.tr.sh[:, 1:4], sh[:, 1:4])
    assert dt.history == []

    old = dt.tr
    before = [t.clone() for t in (old.means, old.scales, old.rotations, old.logits, old.sh)]
    dt.step(views, targets)  # iteration 3: densification
    torch.cuda.synchronize()
    out, counts = densify.densify_and_prune_tensors(*before, old.gradients()[0], 0.0, 1.0, 2.0,
                                                    0.005, 2_000_000)
    assert counts[3] > 0
    assert dt.history == [(3, n) + tuple(counts[:3]) + (out[0].shape[0],)]
    assert dt.n == out[0].shape[0] != n
    for got, want in zip((dt.tr.means, dt.tr.scales, dt.tr.rotations, dt.tr.logits, dt.tr.sh), out):
        assert torch.equal(got, want.reshape(got.shape))
    assert dt.tr.steps_done == 0
    dt.step(views, targets)  # the new set trains
    torch.cuda.synchronize()
    assert dt.tr.steps_done == 1 and not torch.equal(dt.tr.means, out[0])

    dt2 = multiview.DensifyingTrainer(means, scales, rot, logits, sh, buckets=1, densify_interval=1,
                                      grad_threshold=1e30, large_scale_threshold=1e30,
                                      opacity_threshold=0.0)
    dt2.step(views, targets)  # iteration 0: not due
    dt2.step(views, targets)  # iteration 1: due, nothing changes
    torch.cuda.synchronize()
    assert dt2.history == [(1, n, 0, 0, 0, n)]
    assert dt2.tr.steps_done == 1
    g = torch.cat([x.reshape(-1) for x in dt2.tr.gradients()])
    assert torch.allclose(dt2.tr.exp_avg, 0.1 * g, rtol=1e-5, atol=0)
