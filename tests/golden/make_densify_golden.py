"""Generates tests/golden/densify_cases.npz with the reference's own
GaussianModel.densify_and_prune (gaussian_model.py of SAR-3DGS, imported from
its checkout, run on the CPU) on seeded Gaussian sets and mean gradients.

    python tests/golden/make_densify_golden.py [path/to/SAR-3DGS]
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SARR_REFERENCE_DIR")
if not REF:
    sys.exit("usage: pass the SAR-3DGS checkout as the first argument (or set SARR_REFERENCE_DIR)")
sys.path.insert(0, REF)
from gaussian_model import GaussianModel  # noqa: E402


def case(name, n, seed, max_gaussians):
    g = torch.Generator().manual_seed(seed)
    m = GaussianModel(sh_degree=3)
    m._initialize_params(n, torch.device("cpu"))
    with torch.no_grad():
        m._means.copy_((torch.rand(n, 3, generator=g) - 0.5) * 20)
        # scale norms spread across the small (< 0.01) and large (> 2) thresholds
        m._scales.copy_(torch.empty(n, 3).uniform_(-6.5, 1.5, generator=g))
        q = torch.randn(n, 4, generator=g)
        m._rotations.copy_(q / q.norm(dim=1, keepdim=True))
        m._opacities.copy_(torch.randn(n, 1, generator=g) * 2.5)
        m._sh_coeffs.copy_(torch.randn(n, 16, generator=g) * 0.1)
    grad = torch.randn(n, 3, generator=g) * 1e-4
    inputs = {k: getattr(m, k).detach().clone().numpy() for k in
              ("_means", "_scales", "_rotations", "_opacities", "_sh_coeffs")}
    res = m.densify_and_prune(grad, torch.zeros(n, 3), torch.zeros(n, 1), grad_threshold=1e-4,
                              size_threshold=0.01, large_scale_threshold=2.0, opacity_threshold=0.05,
                              max_gaussians=max_gaussians)
    out = {f"{name}/in{k}": v for k, v in inputs.items()}
    out[f"{name}/grad"] = grad.numpy()
    out[f"{name}/max"] = np.array(max_gaussians)
    out[f"{name}/counts"] = np.array(res)
    for k in ("_means", "_scales", "_rotations", "_opacities", "_sh_coeffs"):
        out[f"{name}/out{k}"] = getattr(m, k).detach().numpy()
    return out


def main():
    out = {}
    out.update(case("n3000", 3000, 11, 500000))
    out.update(case("n2000_capped", 2000, 12, 1600))
    np.savez_compressed(os.path.join(HERE, "densify_cases.npz"), **out)
    print({k: v for k, v in out.items() if k.endswith("counts")})


if __name__ == "__main__":
    main()
