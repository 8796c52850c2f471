"""Generates the golden vectors in tests/golden/*.npz by running the reference
rasterizer's own CUDA kernels (cuda_rasterizer/rasterizer_impl_v2.cu with the
slot-indexing fix, built by oracle/ref/build_ref.py) on a GPU.

    python tests/golden/make_golden.py        # on a CUDA machine

Each file holds the seeded inputs, the view, the reference's intermediate
arrays (preprocess floats, valid mask, ranges, image-plane and shadow tile
lists), its render_sar outputs (image in its azimuth-major memory, omega) and
its render_sar_backward gradients for a seeded grad_output. All image sizes
are multiples of 16: the reference's render and Omega kernels return early
for out-of-image threads before __syncthreads, which is undefined for
partial tiles, so partial tiles are only compared against the oracle.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(REPO, "sar-3dgs_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

from cuda_rasterizer import _native  # noqa: E402
from cuda_rasterizer import synthetic as S  # noqa: E402
from oracle.ref import build_ref  # noqa: E402


def cases():
    out = []
    sc = S.named_scene("cpu_1k", seed=0)
    out.append(("config1_n1000_128", sc, S.cpu_view()))
    one = S.make_scene(40, (2.0, 2.0, 0.6), (0.05, 0.4), seed=4)
    out.append(("onetile_n40_16", one, S.view_tuple(30.0, 15.0, 0.3, 16)))
    rect = S.make_scene(3000, (20.0, 20.0, 6.0), (0.05, 0.5), seed=5)
    out.append(("rect_n3000_48x80", rect, S.view_tuple(120.0, 40.0, 0.3, 48)[:8] + (48, 80)))
    return out


def main():
    R = build_ref.load_module()
    dev = torch.device("cuda", 0)
    for name, sc, view in cases():
        t = {k: sc[k].to(dev).contiguous() for k in ("means", "cov6", "sigma", "sh")}
        f, valid, ranges, cnt, lst, scnt, slst, basis = R.intermediates(
            t["means"], t["cov6"], t["sigma"], t["sh"], view[2], view[3], view[4], view[5], view[6],
            view[7], view[8], view[9])
        img, om = R.render_sar(t["means"], t["cov6"], t["sigma"], t["sh"], *view, False, False)
        g = torch.randn(view[8] * view[9], generator=torch.Generator().manual_seed(7)).reshape(
            view[8], view[9]).to(dev)
        gm, gc, gs, gsh = R.render_sar_backward(t["means"], t["cov6"], t["sigma"], t["sh"], g, *view)
        # CUDA's cosf/sinf of the view angles (what the reference kernels use;
        # the C library's may differ in the last bit)
        trig = _native.debug_view_constants(_native.make_view(*view), dev)[10:14]
        torch.cuda.synchronize()
        c = lambda x: x.detach().cpu().numpy()  # noqa: E731
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            view=np.array(view, dtype=np.float64), means=c(t["means"]), cov6=c(t["cov6"]),
            sigma=c(t["sigma"]), sh=c(t["sh"]), f=c(f), valid=c(valid).astype(np.int32),
            ranges=c(ranges), counts=c(cnt), lists=c(lst), shadow_counts=c(scnt),
            shadow_lists=c(slst), sh_basis=c(basis), image=c(img).reshape(-1), omega=c(om),
            grad_output=c(g).reshape(-1), grad_means=c(gm), grad_cov6=c(gc), grad_sigma=c(gs),
            grad_sh=c(gsh), trig=c(trig))
        print(name, "valid", int(c(valid).sum()), "max count", int(c(cnt).max()),
              "image max", float(c(img).max()))


if __name__ == "__main__":
    main()
