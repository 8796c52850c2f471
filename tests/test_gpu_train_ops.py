"""Training-step kernels: the Gaussian parameter producer against the
reference's formula (gaussian_model.py:33-55, :261-330) in float64, and the
fused combined loss against golden vectors of the reference's CombinedLoss
(losses.py) and the oracle restatement."""
import os

import numpy as np
import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import gaussian_params as GP
from cuda_rasterizer import losses as LS
from oracle import loss_oracle as LO

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "loss_cases.npz")
CASES = ["plain_64x80", "linear_3x48x40", "square_2x40x56", "sqrt_2x40x56", "window11_2x33x37"]


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _ref_cov64(scales, rot):
    """gaussian_model.py:261-283 / :285-328 in float64."""
    s = torch.exp(scales.double())
    w, x, y, z = rot.double().unbind(1)
    R = torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y),
                     2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x),
                     2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], 1).view(-1, 3, 3)
    S = torch.diag_embed(s)
    return R @ S @ S.transpose(-1, -2) @ R.transpose(-1, -2)


def test_producer_matches_reference_formula():
    g = torch.Generator().manual_seed(61)
    n = 200_000
    scales = torch.empty(n, 3).uniform_(-4.0, 0.5, generator=g)
    rot = torch.randn(n, 4, generator=g)
    rot[: n // 2] = rot[: n // 2] / rot[: n // 2].norm(dim=1, keepdim=True)  # half unnormalised
    logits = torch.randn(n, generator=g) * 3
    cov33 = GP.compute_covariance_full(scales.cuda(), rot.cuda()).cpu()
    ref = _ref_cov64(scales, rot)
    scale = ref.abs().flatten(1).max(dim=1).values
    assert float(((cov33.double() - ref).abs().flatten(1).max(dim=1).values / scale).max()) <= 2e-6
    cov6 = GP.compute_covariance_rasterizer(scales.cuda(), rot.cuda()).cpu()
    idx = [(0, 0), (1, 1), (2, 2), (0, 1), (0, 2), (1, 2)]
    assert torch.equal(cov6, torch.stack([cov33[:, a, b] for a, b in idx], 1))
    ref6 = GP.compute_covariance(scales.cuda(), rot.cuda()).cpu()
    assert torch.equal(ref6, torch.stack([cov33[:, a, b] for a, b in
                                          [(0, 0), (0, 1), (0, 2), (1, 1), (1, 2), (2, 2)]], 1))
    lg = logits.cuda().requires_grad_(True)
    sig = GP.get_opacity(lg)
    assert _rel(sig.detach().cpu(), torch.sigmoid(logits.double())) <= 1e-6
    sig.sum().backward()
    s64 = torch.sigmoid(logits.double())
    assert _rel(lg.grad.cpu(), s64 * (1 - s64)) <= 1e-5


@pytest.mark.parametrize("name", CASES)
def test_combined_loss_matches_reference_golden(name):
    z = np.load(GOLDEN)
    l1w, sw, window, weighted = z[f"{name}/params"]
    mode = str(z[f"{name}/mode"])
    pred = torch.from_numpy(z[f"{name}/pred"]).cuda().requires_grad_(True)
    target = torch.from_numpy(z[f"{name}/target"]).cuda()
    fn = LS.CombinedLoss(float(l1w), float(sw), int(window), bool(weighted), mode)
    total, info = fn(pred, target)
    ref = z[f"{name}/losses"]
    assert abs(info["total"] - ref[0]) <= 1e-5 * abs(ref[0])
    assert abs(info["l1"] - ref[1]) <= 1e-5 * abs(ref[1])
    assert abs(info["dssim"] - ref[2]) <= 1e-5 * abs(ref[2])
    assert abs(total.item() - ref[0]) <= 1e-5 * abs(ref[0])
    total.backward()
    assert _rel(pred.grad.cpu(), z[f"{name}/grad"]) <= 1e-4


def test_combined_loss_full_size_batch_and_transposed_layout():
    """8 images of 256 x 256 against the oracle; the rasterizer's transposed
    image views give the same loss and gradient as contiguous copies."""
    g = torch.Generator().manual_seed(62)
    p = torch.rand(8, 256, 256, generator=g) ** 2
    t = torch.rand(8, 256, 256, generator=g) ** 2
    losses, grad = _native.combined_loss(p.cuda(), t.cuda(), 0.9, 0.1, 5, "plain")
    total, l1, dssim, ograd = LO.combined_loss(p.numpy(), t.numpy(), 0.9, 0.1, 5, "plain")
    lv = losses.cpu().numpy()
    assert abs(lv[0] - total) <= 1e-5 * total and abs(lv[2] - dssim) <= 1e-5 * dssim
    assert _rel(grad.cpu(), ograd) <= 1e-4
    pt = p.cuda().transpose(1, 2).contiguous().transpose(1, 2).requires_grad_(True)  # strided view
    tt = t.cuda().transpose(1, 2).contiguous().transpose(1, 2)
    tot2, _ = LS.CombinedLoss(0.9, 0.1)(pt, tt)
    tot2.backward()
    assert abs(tot2.item() - lv[0]) <= 1e-6 * lv[0]
    assert _rel(pt.grad.cpu(), grad.cpu()) <= 1e-5


DGOLDEN = os.path.join(os.path.dirname(__file__), "golden", "densify_cases.npz")
DKEYS = ("_means", "_scales", "_rotations", "_opacities", "_sh_coeffs")


@pytest.mark.parametrize("name", ["n3000", "n2000_capped"])
def test_densify_matches_reference_golden(name):
    from cuda_rasterizer import densify as DZ
    z = np.load(DGOLDEN)

    class Model:
        pass

    m = Model()
    for k in DKEYS:
        setattr(m, k, torch.nn.Parameter(torch.from_numpy(z[f"{name}/in{k}"]).cuda()))
    grad = torch.from_numpy(z[f"{name}/grad"]).cuda()
    counts = DZ.densify_and_prune(m, grad, None, None, 1e-4, 0.01, 2.0, 0.05, int(z[f"{name}/max"]))
    assert tuple(counts) == tuple(int(c) for c in z[f"{name}/counts"])
    for k in DKEYS:
        got = getattr(m, k).detach().cpu().numpy()
        ref = z[f"{name}/out{k}"]
        assert got.shape == ref.shape
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_densify_large_set_matches_oracle_and_is_deterministic():
    from cuda_rasterizer import densify as DZ
    from oracle import densify_oracle as DO
    g = torch.Generator().manual_seed(63)
    n = 300_000
    means = (torch.rand(n, 3, generator=g) - 0.5) * 40
    scales = torch.empty(n, 3).uniform_(-6.5, 1.5, generator=g)
    rot = torch.randn(n, 4, generator=g)
    op = torch.randn(n, 1, generator=g) * 2.5
    sh = torch.randn(n, 16, generator=g) * 0.1
    grad = torch.randn(n, 3, generator=g) * 1e-4
    args = (1e-4, 0.01, 2.0, 0.05, 10_000_000)
    out1, c1 = DZ.densify_and_prune_tensors(means.cuda(), scales.cuda(), rot.cuda(), op.cuda(), sh.cuda(),
                                            grad.cuda(), *args)
    out2, c2 = DZ.densify_and_prune_tensors(means.cuda(), scales.cuda(), rot.cuda(), op.cuda(), sh.cuda(),
                                            grad.cuda(), *args)
    assert c1 == c2 and all(torch.equal(a, b) for a, b in zip(out1, out2))
    ref, rc = DO.densify_and_prune(means.numpy(), scales.numpy(), rot.numpy(), op.numpy(), sh.numpy(),
                                   grad.numpy(), *args)
    assert tuple(c1) == tuple(rc)
    for a, b in zip(out1, ref):
        np.testing.assert_allclose(a.cpu().numpy(), b, rtol=1e-6, atol=1e-6)
