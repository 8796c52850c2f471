"""Test infrastructure: ctypes wrapper of the CPU oracle (oracle/sarr_oracle.c).

Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py use
this module, as the oracle of the CUDA library. The product never imports it.

Arrays are numpy float32 / int32. Images use the reference's azimuth-major
memory layout: a flat array indexed c * Nr + r.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
TILE = 16
CAP = 64

F_ROWS = ["ipp_r", "ipp_c", "cov_ipp_rr", "cov_ipp_cc", "cov_ipp_rc", "shadow_x", "shadow_y",
          "cov_shadow_xx", "cov_shadow_yy", "cov_shadow_xy", "gaussian_yr", "gaussian_z",
          "scattering"]
I_ROWS = ["valid", "range_min", "range_max", "azi_min", "azi_max", "shadow_ok", "shadow_c_min",
          "shadow_c_max", "shadow_r_min", "shadow_r_max"]


class View(ctypes.Structure):
    """Same layout as sarr_view / SARRenderParams' scalar fields."""
    _fields_ = [("radar_x", ctypes.c_float), ("radar_y", ctypes.c_float),
                ("radar_z", ctypes.c_float), ("track_angle", ctypes.c_float),
                ("incidence_angle", ctypes.c_float), ("azimuth_angle", ctypes.c_float),
                ("range_resolution", ctypes.c_float), ("azimuth_resolution", ctypes.c_float),
                ("range_samples", ctypes.c_int32), ("azimuth_samples", ctypes.c_int32)]


class ViewC(ctypes.Structure):
    _fields_ = [("radar_x", ctypes.c_float), ("radar_y", ctypes.c_float),
                ("radar_z", ctypes.c_float), ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
                ("Rc", ctypes.c_float), ("rho_r", ctypes.c_float), ("rho_a", ctypes.c_float),
                ("Nr", ctypes.c_int32), ("Na", ctypes.c_int32),
                ("sh_basis", ctypes.c_float * 16), ("cos_a", ctypes.c_float),
                ("sin_a", ctypes.c_float), ("cos_b", ctypes.c_float), ("sin_b", ctypes.c_float)]


_lib = None


def set_threads(n=None):
    """Sets the oracle's OpenMP thread count (default: every core this
    process may run on) and returns the count in effect."""
    if n is None:
        n = len(os.sched_getaffinity(0))
    return lib().oracle_set_threads(int(n))


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "sarr_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            subprocess.check_call(["make", "-s", "-C", HERE])
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        L.oracle_set_threads.argtypes = [I]
        L.oracle_set_threads.restype = I
        L.oracle_view_setup.argtypes = [ctypes.POINTER(View), P, ctypes.POINTER(ViewC)]
        L.oracle_preprocess.argtypes = [ctypes.POINTER(ViewC), I, P, P, I, P, P, I, I, P, P]
        L.oracle_tile_lists.argtypes = [I, I, I, P, I, P, P]
        L.oracle_sort_lists.argtypes = [I, P, P, P, P]
        L.oracle_render.argtypes = [ctypes.POINTER(ViewC), I, P, P, P, P, P]
        L.oracle_omega.argtypes = [ctypes.POINTER(ViewC), I, P, P, P, P, P]
        L.oracle_backward.argtypes = [ctypes.POINTER(ViewC), I, P, P, P, P, P, P, P, P, P]
        for f in ("oracle_view_setup", "oracle_preprocess", "oracle_tile_lists",
                  "oracle_sort_lists", "oracle_render", "oracle_omega", "oracle_backward"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def make_view(radar_x=0.0, radar_y=0.0, radar_z=10000.0, track_angle=0.0, incidence_angle=30.0,
              azimuth_angle=0.0, range_resolution=0.3, azimuth_resolution=0.3, range_samples=128,
              azimuth_samples=128):
    return View(radar_x, radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
                range_resolution, azimuth_resolution, range_samples, azimuth_samples)


def view_consts(view, trig=None):
    vc = ViewC()
    t = None
    if trig is not None:
        t = np.ascontiguousarray(trig, dtype=np.float32)
    lib().oracle_view_setup(ctypes.byref(view), _p(t) if t is not None else None, ctypes.byref(vc))
    return vc


def preprocess(vc, means, cov, sigma, sh, cov_layout=6, sh_k=None):
    means, cov, sigma, sh = _f32(means), _f32(cov), _f32(sigma), _f32(sh)
    n = means.shape[0]
    sh2 = sh.reshape(n, -1) if n else sh.reshape(0, 16)
    if sh_k is None:
        sh_k = min(16, sh2.shape[1])
    f = np.zeros((13, n), np.float32)
    q = np.zeros((10, n), np.int32)
    if n:
        lib().oracle_preprocess(ctypes.byref(vc), n, _p(means), _p(cov), cov_layout, _p(sigma),
                                _p(sh2), sh2.shape[1], sh_k, _p(f), _p(q))
    return f, q


def tiles(Nr, Na):
    tx, ty = (Na + TILE - 1) // TILE, (Nr + TILE - 1) // TILE
    return tx, ty, tx * ty


def tile_lists(Nr, Na, q, shadow=False):
    q = np.ascontiguousarray(q, dtype=np.int32)
    n = q.shape[1]
    T = tiles(Nr, Na)[2]
    counts = np.zeros(T, np.int32)
    lists = np.full((T, CAP), -1, np.int32)
    if T:
        lib().oracle_tile_lists(Nr, Na, n, _p(q), 1 if shadow else 0, _p(counts), _p(lists))
    return counts, lists


def sort_lists(counts, lists, z):
    z = _f32(z)
    T = counts.shape[0]
    sorted_ = np.full((T, CAP), -1, np.int32)
    if T:
        lib().oracle_sort_lists(T, _p(counts), _p(lists), _p(z), _p(sorted_))
    return sorted_


def render(vc, f, sigma, counts, sorted_):
    f, sigma = _f32(f), _f32(sigma)
    img = np.zeros(vc.Nr * vc.Na, np.float32)
    if img.size:
        lib().oracle_render(ctypes.byref(vc), f.shape[1], _p(f), _p(sigma), _p(counts),
                            _p(sorted_), _p(img))
    return img


def omega(vc, f, sigma, counts, sorted_):
    f, sigma = _f32(f), _f32(sigma)
    n = f.shape[1]
    om = np.ones(n, np.float32)
    if n and counts.size:
        lib().oracle_omega(ctypes.byref(vc), n, _p(f), _p(sigma), _p(counts), _p(sorted_), _p(om))
    return om


def backward(vc, f, sigma, counts, sorted_, grad_image):
    f, sigma, g = _f32(f), _f32(sigma), _f32(grad_image).reshape(-1)
    n = f.shape[1]
    gm = np.zeros((n, 3), np.float32)
    gc = np.zeros((n, 6), np.float32)
    gs = np.zeros(n, np.float32)
    gsh = np.zeros((n, 16), np.float32)
    if n and counts.size:
        lib().oracle_backward(ctypes.byref(vc), n, _p(f), _p(sigma), _p(counts), _p(sorted_),
                              _p(g), _p(gm), _p(gc), _p(gs), _p(gsh))
    return gm, gc, gs, gsh


def forward(view, means, cov, sigma, sh, cov_layout=6, trig=None, want_omega=True, sh_k=None):
    """The reference forward (render_sar) restated: returns a dict with the
    preprocess arrays, the capped lists, their depth order, the image (flat,
    azimuth-major) and omega."""
    vc = view_consts(view, trig)
    f, q = preprocess(vc, means, cov, sigma, sh, cov_layout, sh_k)
    counts, lists = tile_lists(view.range_samples, view.azimuth_samples, q, shadow=False)
    sorted_ = sort_lists(counts, lists, f[11])
    out = {"vc": vc, "f": f, "q": q, "counts": counts, "lists": lists, "sorted": sorted_,
           "image": render(vc, f, sigma, counts, sorted_)}
    if want_omega:
        sc, sl = tile_lists(view.range_samples, view.azimuth_samples, q, shadow=True)
        ss = sort_lists(sc, sl, f[11])
        out.update(shadow_counts=sc, shadow_lists=sl, shadow_sorted=ss,
                   omega=omega(vc, f, sigma, sc, ss))
    return out


def backward_full(view, means, cov, sigma, sh, grad_image, cov_layout=6, trig=None, sh_k=None):
    """render_sar_backward restated: (grad_means, grad_cov6, grad_sigma, grad_sh[n,16])."""
    fw = forward(view, means, cov, sigma, sh, cov_layout, trig, want_omega=False, sh_k=sh_k)
    return backward(fw["vc"], fw["f"], sigma, fw["counts"], fw["sorted"], grad_image)
