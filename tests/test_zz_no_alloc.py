"""sarr_forward_static (the forward whose scratch is a static device array of
the library) against sarr_forward, called through the C ABI with ctypes.

This entry point is for callers that cannot allocate device memory: a host
whose device memory is all owned by another allocator, or a C caller with no
device allocator of its own. The tests check that its images equal the
workspace forward's bit for bit on two calls in a row (the scratch keeps the
previous call's contents), that those calls change the device's free memory
by nothing, that its device error word reads clear, and that requests beyond
the scratch's limits are refused.

Kept in its own file, collected last, so that it runs both alone and after
every other test of the session.
"""
import ctypes

import pytest
import torch

from cuda_rasterizer import _native
from cuda_rasterizer import synthetic as S

pytestmark = pytest.mark.gpu

SARR_ERR_CAPACITY = 6
MAX_GAUSSIANS = 131072


def _static_fns():
    L = _native.lib()
    fn = L.sarr_forward_static
    P = ctypes.c_void_p
    fn.argtypes = [ctypes.POINTER(_native.SarrView), ctypes.c_int64, P, P, ctypes.c_int, P, P,
                   ctypes.c_int, ctypes.c_int, P, P]
    fn.restype = ctypes.c_int
    chk = L.sarr_check_static_errors
    chk.argtypes = [P]
    chk.restype = ctypes.c_int
    return fn, chk


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _call_static(fn, view, inputs, image, n=None):
    means, cov, layout, sigma, sh, sh_stride, sh_k = inputs
    return fn(ctypes.byref(view), means.shape[0] if n is None else n, means.data_ptr(),
              cov.data_ptr(), layout, sigma.data_ptr(), sh.data_ptr(), sh_stride, sh_k,
              image.data_ptr(), _stream())


def _status_text(status):
    return _native.lib().sarr_status_string(status).decode()


@pytest.mark.parametrize("n,vk", [(1000, "cpu"), (MAX_GAUSSIANS, "sweep")])
def test_static_scratch_forward_matches_workspace_forward(n, vk):
    sc = {k: v.cuda() for k, v in S.make_scene(n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=41).items()}
    view_t = S.cpu_view() if vk == "cpu" else S.sweep_views(8)[3]
    view = _native.make_view(*view_t)
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    nr, na = view_t[8], view_t[9]

    ref = torch.empty((1, nr, na), dtype=torch.float32, device="cuda")
    _native.forward([view], *inputs, ref)

    fn, chk = _static_fns()
    imgs = [torch.full((nr, na), float("nan"), dtype=torch.float32, device="cuda") for _ in range(3)]
    # warm-up: the first call in a context looks up the scratch's address
    assert _call_static(fn, view, inputs, imgs[0]) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for img in imgs[1:]:  # two consecutive calls on the same scratch
        status = _call_static(fn, view, inputs, img)
        assert status == 0, _status_text(status)
        assert chk(_stream()) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0  # no device allocation by the calls
    for img in imgs:
        assert torch.equal(img, ref[0])  # the same kernels: identical bits


def test_static_scratch_rejects_requests_beyond_its_size():
    fn, chk = _static_fns()
    sc = {k: v.cuda() for k, v in S.make_scene(1000, (20.0, 20.0, 6.0), (0.05, 0.5), seed=42).items()}
    inputs = _native.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    big = _native.make_view(*S.view_tuple(30.0, 15.0, 0.3, 257))
    img = torch.zeros((257, 257), dtype=torch.float32, device="cuda")
    assert _call_static(fn, big, inputs, img) == SARR_ERR_CAPACITY
    assert "static scratch" in _status_text(SARR_ERR_CAPACITY)
    # one Gaussian more than the limit is refused before any pointer is read
    ok_view = _native.make_view(*S.view_tuple(30.0, 15.0, 0.3, 128))
    small = torch.zeros((128, 128), dtype=torch.float32, device="cuda")
    assert _call_static(fn, ok_view, inputs, small, n=MAX_GAUSSIANS + 1) == SARR_ERR_CAPACITY
    assert chk(_stream()) == 0
