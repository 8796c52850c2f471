"""The loss restatement (oracle/loss_oracle.py) against golden vectors made by
the reference's own CombinedLoss (losses.py, torch autograd float32):
values within 1e-5 relative, gradients within 1e-4 relative L-inf."""
import os

import numpy as np
import pytest

from oracle import loss_oracle as LO

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "loss_cases.npz")
CASES = ["plain_64x80", "linear_3x48x40", "square_2x40x56", "sqrt_2x40x56", "window11_2x33x37"]


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("name", CASES)
def test_loss_restatement_matches_reference(name):
    z = np.load(GOLDEN)
    l1w, sw, window, weighted = z[f"{name}/params"]
    mode = str(z[f"{name}/mode"]) if weighted else "plain"
    total, l1, dssim, grad = LO.combined_loss(z[f"{name}/pred"], z[f"{name}/target"], l1w, sw,
                                              int(window), mode)
    ref = z[f"{name}/losses"]
    assert abs(total - ref[0]) <= 1e-5 * abs(ref[0])
    assert abs(l1 - ref[1]) <= 1e-5 * abs(ref[1])
    assert abs(dssim - ref[2]) <= 1e-5 * abs(ref[2])
    assert _rel(grad, z[f"{name}/grad"]) <= 1e-4
