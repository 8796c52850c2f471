"""The densify/prune restatement (oracle/densify_oracle.py) against golden
vectors of the reference's own GaussianModel.densify_and_prune: counts and
order exact, values within float32 rounding of exp/log."""
import os

import numpy as np
import pytest

from oracle import densify_oracle as DO

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "densify_cases.npz")
KEYS = ("_means", "_scales", "_rotations", "_opacities", "_sh_coeffs")


@pytest.mark.parametrize("name", ["n3000", "n2000_capped"])
def test_densify_restatement_matches_reference(name):
    z = np.load(GOLDEN)
    ins = [z[f"{name}/in{k}"] for k in KEYS]
    out, counts = DO.densify_and_prune(*ins, z[f"{name}/grad"], 1e-4, 0.01, 2.0, 0.05, int(z[f"{name}/max"]))
    assert tuple(counts) == tuple(z[f"{name}/counts"])
    for k, o in zip(KEYS, out):
        ref = z[f"{name}/out{k}"]
        assert o.shape == ref.shape
        np.testing.assert_allclose(o, ref, rtol=1e-6, atol=1e-6)
