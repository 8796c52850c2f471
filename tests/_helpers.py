"""Shared helpers of the GPU tests: scenes, calls into the CUDA library and
into the oracle, and the tolerance checks.

Tolerances (from the parity target): tile lists and depth orders bit-exact;
images and Omega within 1e-4 relative L-infinity, i.e.
max|got - ref| <= 1e-4 * max|ref|; parameter gradients within 1e-3 relative
per tensor, max|got - ref| <= 1e-3 * max|ref|.
"""
import numpy as np
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import cuda_rasterizer_sar as M
from cuda_rasterizer import synthetic as S
from oracle import oracle as O

IMAGE_RTOL = 1e-4
GRAD_RTOL = 1e-3


def rel_linf(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.abs(ref).max() if ref.size else 0.0
    err = np.abs(got - ref).max() if ref.size else 0.0
    return err / scale if scale > 0 else err


def scene(name_or_n, seed=0, device="cuda", box=(20.0, 20.0, 6.0), scales=(0.05, 0.5)):
    if isinstance(name_or_n, str):
        return S.named_scene(name_or_n, seed=seed, device=device)
    return S.make_scene(int(name_or_n), box, scales, seed=seed, device=device)


def oview(t):
    return O.make_view(*t)


def gpu_forward(sc, view, cov="cov6", omega=True):
    img, om = M.render_sar(sc["means"], sc[cov], sc["sigma"], sc["sh"], *view)
    torch.cuda.synchronize()
    return img, om


def gpu_lists(sc, view, cov="cov6"):
    means, c, layout, sigma, sh, st, k = _native.prepare_inputs(sc["means"], sc[cov], sc["sigma"], sc["sh"])
    v = _native.make_view(*view)
    out = _native.debug_tile_lists(v, means, c, layout, sigma)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in out]


def gpu_preprocess(sc, view, cov="cov6"):
    means, c, layout, sigma, sh, st, k = _native.prepare_inputs(sc["means"], sc[cov], sc["sigma"], sc["sh"])
    f, q = _native.debug_preprocess(_native.make_view(*view), means, c, layout, sigma, sh, st, k)
    torch.cuda.synchronize()
    return f.cpu().numpy(), q.cpu().numpy()


def np_scene(sc):
    return {k: v.detach().cpu().numpy() for k, v in sc.items()}


def device_trig(view):
    """cos/sin of the view's track and beta angles as the GPU evaluates them
    (CUDA's cosf/sinf, which the C library's may differ from in the last bit)."""
    vc = _native.debug_view_constants(_native.make_view(*view), torch.device("cuda"))
    return vc[10:14].cpu().numpy()


def oracle_forward(sc, view, want_omega=True, sh_k=None, sh=None):
    s = np_scene(sc)
    return O.forward(oview(view), s["means"], s["cov6"], s["sigma"], s["sh"] if sh is None else sh,
                     want_omega=want_omega, trig=device_trig(view), sh_k=sh_k)


def oracle_backward(sc, view, grad_image):
    s = np_scene(sc)
    return O.backward_full(oview(view), s["means"], s["cov6"], s["sigma"], s["sh"], grad_image,
                           trig=device_trig(view))


def image_flat(img):
    """The image's memory as the reference lays it out (flat c * Nr + r)."""
    return img.detach().contiguous().view(-1).cpu().numpy()
