"""C ABI checks that need no GPU: the library loads, exports every function
declared in include/sarr.h, sizes workspaces, rejects bad arguments before
touching the device, and maps pixel bboxes to tile rectangles exactly like
the reference's per-tile hit test."""
import ctypes
import os
import re

import numpy as np
import pytest

from cuda_rasterizer import _native

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(REPO, "include", "sarr.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sarr_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols():
    L = _native.lib()
    syms = declared_symbols()
    assert "sarr_forward" in syms and "sarr_backward" in syms
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/sarr.h but not exported"
    assert L.sarr_version().decode().startswith("sarr")


def test_status_strings():
    L = _native.lib()
    for code in range(0, 6):
        assert L.sarr_status_string(code)
    assert L.sarr_status_string(0).decode() == "ok"


def test_workspace_and_state_sizes():
    ws1 = _native.workspace_bytes(1000, 128, 128, 1)
    ws4 = _native.workspace_bytes(1000, 128, 128, 4)
    assert ws4 > ws1 > 0
    # views beyond one launch group (256) need no more workspace
    assert _native.workspace_bytes(1000, 128, 128, 512) == _native.workspace_bytes(1000, 128, 128, 256)
    assert _native.workspace_bytes(1000, 128, 128, 256) > _native.workspace_bytes(1000, 128, 128, 128)
    st_small = _native.state_bytes(1000, 128, 128)
    st_big = _native.state_bytes(1_000_000, 256, 256)
    assert st_big > st_small
    # state: per-Gaussian tile rectangle (4 B) + per-tile lists and records
    assert st_big >= 4 * 1_000_000 + 256 * 64 * 48


def _view(nr=64, na=64):
    return _native.make_view(0, 0, 5000, 0, 30, 0, 0.3, 0.3, nr, na)


def test_arguments_rejected_before_device_use():
    L = _native.lib()
    v = (_native.SarrView * 2)(_view(), _view(32, 64))
    dummy = ctypes.c_void_p(256)
    # views with different image sizes in one call
    assert L.sarr_forward(v, 2, 10, dummy, dummy, 6, dummy, dummy, 16, 16, dummy, None, None,
                          dummy, 1 << 20, None) == 1
    one = (_native.SarrView * 1)(_view())
    # bad covariance layout
    assert L.sarr_forward(one, 1, 10, dummy, dummy, 7, dummy, dummy, 16, 16, dummy, None, None,
                          dummy, 1 << 20, None) == 1
    # sh_k out of range
    assert L.sarr_forward(one, 1, 10, dummy, dummy, 6, dummy, dummy, 16, 17, dummy, None, None,
                          dummy, 1 << 20, None) == 1
    # null inputs with n > 0
    assert L.sarr_forward(one, 1, 10, None, dummy, 6, dummy, dummy, 16, 16, dummy, None, None,
                          dummy, 1 << 20, None) == 1
    # workspace too small / misaligned
    assert L.sarr_forward(one, 1, 10, dummy, dummy, 6, dummy, dummy, 16, 16, dummy, None, None,
                          dummy, 64, None) == 2
    assert L.sarr_forward(one, 1, 10, dummy, dummy, 6, dummy, dummy, 16, 16, dummy, None, None,
                          ctypes.c_void_p(260), 1 << 30, None) == 2
    # image over 2048 pixels per axis
    big = (_native.SarrView * 1)(_view(4096, 64))
    assert L.sarr_forward(big, 1, 10, dummy, dummy, 6, dummy, dummy, 16, 16, dummy, None, None,
                          dummy, 1 << 30, None) == 3
    # backward: bad grad_sh_cols
    assert L.sarr_backward(one, 1, 10, dummy, dummy, 6, dummy, dummy, 16, 16, dummy, None, dummy,
                           dummy, 6, dummy, dummy, 0, None, 0, dummy, 1 << 20, None) == 1


def _reference_hits(r0, r1, c0, c1, nr, na):
    """build_tile_gaussian_list_kernel's hit test (rasterizer_impl_v2.cu:511-529)."""
    tx, ty = (na + 15) // 16, (nr + 15) // 16
    hits = set()
    for tr in range(ty):
        for tc in range(tx):
            pmin_c, pmin_r = tc * 16, tr * 16
            pmax_c, pmax_r = min(pmin_c + 16, na), min(pmin_r + 16, nr)
            if not (r1 < pmin_r or r0 > pmax_r or c1 < pmin_c or c0 > pmax_c):
                hits.add((tr, tc))
    return hits


@pytest.mark.parametrize("nr,na", [(64, 64), (50, 37), (16, 16), (33, 80)])
def test_tile_rect_equals_reference_hit_test(nr, na):
    rng = np.random.default_rng(nr * 1000 + na)
    cases = []
    # exhaustive over small clamped ranges, plus random out-of-image cases
    for r0 in range(0, nr + 2, 3):
        for r1 in range(-2, nr, 5):
            cases.append((r0, r1, int(rng.integers(0, na)), int(rng.integers(-3, na))))
    for _ in range(300):
        a, b = sorted(rng.integers(-20, max(nr, na) + 20, 2))
        c, d = sorted(rng.integers(-20, max(nr, na) + 20, 2))
        cases.append((max(0, int(a)), min(nr - 1, int(b)), max(0, int(c)), min(na - 1, int(d))))
    for r0, r1, c0, c1 in cases:
        tc0, tc1, tr0, tr1 = _native.tile_rect(r0, r1, c0, c1, nr, na)
        got = {(tr, tc) for tr in range(tr0, tr1 + 1) for tc in range(tc0, tc1 + 1)} if tc0 <= tc1 else set()
        assert got == _reference_hits(r0, r1, c0, c1, nr, na), (r0, r1, c0, c1)
