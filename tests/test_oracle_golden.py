"""Pins the CPU oracle against golden vectors produced by the reference
rasterizer itself on a B200 (tests/golden/make_golden.py): preprocess floats
within float rounding, the index-ordered capped tile lists bit for bit (both
from the reference's own validity/range integers and end to end), the image
and Omega within 1e-4 relative L-inf and the gradients within 1e-3 relative.
No GPU needed."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
# rasterizer fixtures (loss_ and densify_ files belong to the training-op tests)
FILES = sorted(f for f in glob.glob(os.path.join(HERE, "golden", "*.npz"))
               if not os.path.basename(f).startswith(("loss_", "densify_")))


def rel(a, b):
    b = np.asarray(b, np.float64)
    s = np.abs(b).max()
    return np.abs(np.asarray(a, np.float64) - b).max() / s if s > 0 else np.abs(a).max()


def test_golden_vectors_present():
    assert len(FILES) >= 3, "golden vectors missing: run tests/golden/make_golden.py on a GPU"


@pytest.mark.parametrize("path", FILES, ids=[os.path.basename(f)[:-4] for f in FILES])
def test_oracle_matches_reference(path):
    z = np.load(path)
    view = O.make_view(*[float(x) for x in z["view"][:8]], int(z["view"][8]), int(z["view"][9]))
    nr, na = int(z["view"][8]), int(z["view"][9])
    # the rotation trig as CUDA's cosf/sinf evaluated it on the B200
    fw = O.forward(view, z["means"], z["cov6"], z["sigma"], z["sh"], trig=z["trig"])
    valid = z["valid"].astype(bool)
    # SH basis (host math) is bit-identical
    assert np.array_equal(np.array(fw["vc"].sh_basis[:], np.float32), z["sh_basis"])
    # preprocess floats: bit-identical on every Gaussian the reference processed
    for row in range(13):
        a, b = fw["f"][row][valid], z["f"][row][valid]
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), O.F_ROWS[row]
    np.testing.assert_array_equal(fw["q"][0].astype(bool), valid)
    np.testing.assert_array_equal(fw["q"][1:5], z["ranges"])
    # integer stage fed with the reference's own validity / ranges
    q = fw["q"].copy()
    q[0] = z["valid"]
    q[1:5] = z["ranges"]
    c, l = O.tile_lists(nr, na, q, shadow=False)
    np.testing.assert_array_equal(c, z["counts"])
    np.testing.assert_array_equal(l, z["lists"])
    # end to end
    np.testing.assert_array_equal(fw["counts"], z["counts"])
    np.testing.assert_array_equal(fw["lists"], z["lists"])
    np.testing.assert_array_equal(fw["shadow_counts"], z["shadow_counts"])
    np.testing.assert_array_equal(fw["shadow_lists"], z["shadow_lists"])
    assert rel(fw["image"], z["image"]) <= 1e-4
    assert rel(fw["omega"], z["omega"]) <= 1e-4
    grads = O.backward(fw["vc"], fw["f"], z["sigma"], fw["counts"], fw["sorted"], z["grad_output"])
    for got, name in zip(grads, ("grad_means", "grad_cov6", "grad_sigma", "grad_sh")):
        assert rel(got, z[name]) <= 1e-3, name
