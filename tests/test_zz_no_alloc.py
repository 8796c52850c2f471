"""sarr_forward_static (the forward whose scratch is a static device array of
the library) against sarr_forward, called through the C ABI with ctypes.

Kept in its own file, collected last, so that it runs both alone and after
every other test of the session.
"""
import ctypes

import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import synthetic as S

from _helpers import IMAGE_RTOL, rel_linf

pytestmark = pytest.mark.gpu

SARR_ERR_CAPACITY = 6


def _static_fn():
    fn = _native.lib().sarr_forward_static
    P = ctypes.c_void_p
    fn.argtypes = [ctypes.POINTER(_native.SarrView), ctypes.c_int64, P, P, ctypes.c_int, P, P,
                   ctypes.c_int, ctypes.c_int, P, P]
    fn.restype = ctypes.c_int
    return fn


def _call_static(fn, view, inputs, image):
    means, cov, layout, sigma, sh, sh_stride, sh_k = inputs
    stream = torch.cuda.current_stream(means.device).cuda_stream
    return fn(ctypes.byref(view), means.shape[0], means.data_ptr(), cov.data_ptr(), layout,
              sigma.data_ptr(), sh.data_ptr(), sh_stride, sh_k, image.data_ptr(), stream)


@pytest.mark.parametrize("n,vk", [(1000, "cpu"), (131072, "sweep")])
def test_static_scratch_forward_matches_workspace_forward(n, vk):
    sc = {k: v.cuda() for k, v in S.make_scene(n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=41).items()}
    view_t = S.cpu_view() if vk == "cpu" else S.sweep_views(8)[3]
    view = _native.make_view(*view_t)
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    nr, na = view_t[8], view_t[9]

    ref = torch.empty((1, nr, na), dtype=torch.float32, device="cuda")
    _native.forward([view], *inputs, ref)

    fn = _static_fn()
    for _ in range(2):  # two consecutive calls on the same scratch
        img = torch.full((nr, na), float("nan"), dtype=torch.float32, device="cuda")
        status = _call_static(fn, view, inputs, img)
        torch.cuda.synchronize()
        assert status == 0, _native.lib().sarr_status_string(status).decode()
        assert torch.isfinite(img).all()
        assert rel_linf(img.cpu().numpy().ravel(), ref[0].cpu().numpy().ravel()) <= IMAGE_RTOL


def test_static_scratch_rejects_requests_beyond_its_size():
    fn = _static_fn()
    sc = {k: v.cuda() for k, v in S.make_scene(1000, (20.0, 20.0, 6.0), (0.05, 0.5), seed=42).items()}
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    big = _native.make_view(*S.view_tuple(30.0, 15.0, 0.3, 257))
    img = torch.zeros((257, 257), dtype=torch.float32, device="cuda")
    assert _call_static(fn, big, inputs, img) == SARR_ERR_CAPACITY
    msg = _native.lib().sarr_status_string(SARR_ERR_CAPACITY).decode()
    assert "static scratch" in msg
