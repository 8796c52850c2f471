"""Generates tests/golden/loss_cases.npz with the reference's own loss module
(losses.py of SAR-3DGS, imported from its checkout): CombinedLoss forward
values and the gradient of the total loss with respect to pred (torch
autograd, float32 on the CPU) for seeded image pairs.

    python tests/golden/make_loss_golden.py [path/to/SAR-3DGS]
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
from losses import CombinedLoss  # noqa: E402


def case(name, shape, l1w, sw, window, weighted, mode, seed):
    g = torch.Generator().manual_seed(seed)
    # SAR-like amplitudes: non-negative, heavy-tailed
    pred = (torch.rand(shape, generator=g) ** 2 * 2.0).requires_grad_(True)
    target = torch.rand(shape, generator=g) ** 2 * 2.0
    fn = CombinedLoss(l1_weight=l1w, ssim_weight=sw, window_size=window, use_weighted_l1=weighted,
                      l1_weight_mode=mode)
    total, info = fn(pred, target)
    total.backward()
    return {f"{name}/pred": pred.detach().numpy(), f"{name}/target": target.numpy(),
            f"{name}/params": np.array([l1w, sw, window, float(weighted)], np.float64),
            f"{name}/mode": np.array(mode),
            f"{name}/losses": np.array([info["total"], info["l1"], info["dssim"]], np.float64),
            f"{name}/grad": pred.grad.numpy()}


def main():
    out = {}
    out.update(case("plain_64x80", (64, 80), 0.9, 0.1, 5, False, "linear", 1))
    out.update(case("linear_3x48x40", (3, 48, 40), 0.9, 0.1, 5, True, "linear", 2))
    out.update(case("square_2x40x56", (2, 40, 56), 0.7, 0.3, 5, True, "square", 3))
    out.update(case("sqrt_2x40x56", (2, 40, 56), 0.7, 0.3, 5, True, "sqrt", 4))
    out.update(case("window11_2x33x37", (2, 33, 37), 0.5, 0.5, 11, False, "linear", 5))
    np.savez_compressed(os.path.join(HERE, "loss_cases.npz"), **out)
    print("wrote", len(out), "arrays")


if __name__ == "__main__":
    main()
