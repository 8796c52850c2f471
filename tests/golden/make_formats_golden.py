"""Generates tests/golden/formats_checkpoint.pt (a checkpoint written by the
reference's GaussianModel.save_checkpoint) and tests/golden/formats_names.json
(the reference's parse_sar_filename on a set of file names).

    python tests/golden/make_formats_golden.py [path/to/SAR-3DGS]
"""
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SARR_REFERENCE_DIR")
if not REF:
    sys.exit("usage: pass the SAR-3DGS checkout as the first argument (or set SARR_REFERENCE_DIR)")
sys.path.insert(0, REF)
from gaussian_model import GaussianModel  # noqa: E402
from scene.dataset_readers import parse_sar_filename  # noqa: E402

NAMES = ["inc_30.0-track_45.5-height_5000-squint_0.0-rr_0.3-ar_0.3.png",
         "inc_17-track_n120.25-height_10000-squint_n2.5-rr_0.2-ar_0.25.png",
         "elev-15-azim-30.5-A.png", "elev-17.0-azim--45-A.png", "image_001.png",
         "inc_30-track_45-height_5000-squint_0-rr_0.3-ar_0.3.jpg"]


def main():
    g = torch.Generator().manual_seed(71)
    m = GaussianModel(sh_degree=3)
    m._initialize_params(50, torch.device("cpu"))
    with torch.no_grad():
        for p in (m._means, m._scales, m._rotations, m._opacities, m._sh_coeffs):
            p.copy_(torch.randn(p.shape, generator=g))
    m._active_sh_degree = 2
    m.save_checkpoint(os.path.join(HERE, "formats_checkpoint.pt"), iteration=1234)
    with open(os.path.join(HERE, "formats_names.json"), "w") as fh:
        json.dump({n: parse_sar_filename(n) for n in NAMES}, fh, indent=1)
    print("ok")


if __name__ == "__main__":
    main()
