"""ctypes binding of libsarr.so (the sm_100a kernels behind include/sarr.h).

Tensors stay PyTorch tensors: this module only passes their device pointers,
the current CUDA stream and caching-allocator workspaces to the C ABI. It has
no CPU path: a missing library, a CPU tensor or a non-float32 tensor raises.
ctypes releases the GIL for the duration of each C call.
"""
import ctypes
import os
import threading

import torch

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("SARR_LIBRARY", os.path.join(_PKG_ROOT, "libsarr.so"))

SARR_OK = 0
SARR_COV6 = 6
SARR_COV33 = 9
SARR_FLAG_OMEGA = 1
SARR_FLAG_ACCUMULATE = 2
SARR_FLAG_TILES_ONLY = 4
SARR_FLAG_RANGE_ROWS = 8
SARR_L1_MODES = {"plain": 0, "linear": 1, "square": 2, "sqrt": 3}
MAX_SH = 16


class SarrView(ctypes.Structure):
    """sarr_view (include/sarr.h)."""
    _fields_ = [("radar_x", ctypes.c_float), ("radar_y", ctypes.c_float),
                ("radar_z", ctypes.c_float), ("track_angle", ctypes.c_float),
                ("incidence_angle", ctypes.c_float), ("azimuth_angle", ctypes.c_float),
                ("range_resolution", ctypes.c_float), ("azimuth_resolution", ctypes.c_float),
                ("range_samples", ctypes.c_int32), ("azimuth_samples", ctypes.c_int32)]


def make_view(radar_x, radar_y, radar_z, track_angle, incidence_angle, azimuth_angle,
              range_resolution, azimuth_resolution, range_samples, azimuth_samples):
    # Python floats are narrowed to float32 exactly as pybind11 does for the
    # reference's float parameters.
    return SarrView(float(radar_x), float(radar_y), float(radar_z), float(track_angle),
                    float(incidence_angle), float(azimuth_angle), float(range_resolution),
                    float(azimuth_resolution), int(range_samples), int(azimuth_samples))


_lib = None
_lock = threading.Lock()


def _declare(L):
    P = ctypes.c_void_p
    I = ctypes.c_int
    I64 = ctypes.c_int64
    SZ = ctypes.c_size_t
    VP = ctypes.POINTER(SarrView)
    L.sarr_status_string.argtypes = [I]
    L.sarr_status_string.restype = ctypes.c_char_p
    L.sarr_version.argtypes = []
    L.sarr_version.restype = ctypes.c_char_p
    L.sarr_workspace_size.argtypes = [I64, I, I, I, I, ctypes.POINTER(SZ)]
    L.sarr_state_size.argtypes = [I64, I, I, ctypes.POINTER(SZ)]
    L.sarr_forward.argtypes = [VP, I, I64, P, P, I, P, P, I, I, P, P, P, P, SZ, P]
    L.sarr_backward.argtypes = [VP, I, I64, P, P, I, P, P, I, I, P, P, P, P, I, P, P, I, P, I, P,
                                SZ, P]
    L.sarr_backward_scatter.argtypes = [VP, I, I64, P, I64, I64, P, P, I, P, P, I, P, I, P, SZ, P]
    L.sarr_debug_preprocess.argtypes = [VP, I64, P, P, I, P, P, I, I, P, P, P]
    L.sarr_debug_tile_lists.argtypes = [VP, I64, P, P, I, P, P, P, P, P, P, P, P, SZ, P]
    L.sarr_check_device_errors.argtypes = [P, SZ, P]
    L.sarr_debug_view_constants.argtypes = [VP, P, P]
    L.sarr_debug_view_constants.restype = I
    IP = ctypes.POINTER(ctypes.c_int32)
    L.sarr_debug_tile_rect.argtypes = [I, I, I, I, I, I, IP, IP, IP, IP]
    L.sarr_launch_count.argtypes = []
    L.sarr_launch_count.restype = ctypes.c_int64
    L.sarr_profile_enable.argtypes = [I]
    L.sarr_profile_enable.restype = I
    L.sarr_profile_read.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int64), I]
    L.sarr_profile_read.restype = I
    L.sarr_kernel_name.argtypes = [I]
    L.sarr_kernel_name.restype = ctypes.c_char_p
    L.sarr_gaussian_params.argtypes = [I64, P, P, P, I, P, P, P]
    L.sarr_loss_workspace_size.argtypes = [I, I, I, ctypes.POINTER(SZ)]
    F = ctypes.c_float
    L.sarr_combined_loss.argtypes = [I, I, I, P, P, F, F, I, I, P, P, P, SZ, P]
    L.sarr_adam_step.argtypes = [I64, P, P, P, P, I, ctypes.POINTER(I64), ctypes.POINTER(F), F, F,
                                 F, I64, P]
    L.sarr_adam_step_ranges.argtypes = [I, ctypes.POINTER(I64), ctypes.POINTER(I64),
                                        ctypes.POINTER(I64), ctypes.POINTER(F), P, P, P, P, F, F,
                                        F, I64, P]
    L.sarr_densify_workspace_size.argtypes = [I64, ctypes.POINTER(SZ)]
    L.sarr_densify_flags.argtypes = [I64, P, P, P, F, F, F, F, P, P, SZ, P]
    L.sarr_densify_apply.argtypes = [I64, P, P, P, P, P, I, P, P, I, I, P, P, P, P, P, P, SZ, P]
    for name in ("sarr_workspace_size", "sarr_state_size", "sarr_forward", "sarr_backward",
                 "sarr_backward_scatter",
                 "sarr_debug_preprocess", "sarr_debug_tile_lists", "sarr_check_device_errors",
                 "sarr_debug_tile_rect", "sarr_gaussian_params", "sarr_loss_workspace_size",
                 "sarr_combined_loss", "sarr_adam_step", "sarr_adam_step_ranges", "sarr_densify_workspace_size", "sarr_densify_flags",
                 "sarr_densify_apply"):
        getattr(L, name).restype = I
    return L


def lib():
    """Loads libsarr.so (raises RuntimeError if it is missing)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libsarr.so not found at {LIB_PATH}; build it with "
                        "`python sar-3dgs_b200/build.py` (there is no CPU fallback)")
                _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def available():
    try:
        lib()
    except (OSError, RuntimeError):
        return False
    return torch.cuda.is_available()


def _check(status, what):
    if status != SARR_OK:
        msg = lib().sarr_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _as_cuda_f32(t, name):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the SAR rasterizer has no CPU path)")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32, got {t.dtype}")
    return t


def _sh_rows(sh, n):
    """(tensor, row stride, active coefficients) for an SH tensor [n, K].

    A column slice of a wider parameter (GaussianModel.get_active_sh_coeffs,
    gaussian_model.py:334-337) is used in place through its row stride; only
    its K active columns are read and the others count as zero."""
    if sh.dim() == 1:
        sh = sh.reshape(n, -1) if n else sh.reshape(0, 1)
    if sh.dim() != 2 or sh.shape[0] != n:
        raise RuntimeError(f"sh_coeffs must have shape [N, K], got {tuple(sh.shape)}")
    k = sh.shape[1]
    if k < 1 or k > MAX_SH:
        raise RuntimeError(f"sh_coeffs must have 1..16 columns, got {k}")
    if sh.stride(1) != 1 or sh.stride(0) < k:
        sh = sh.contiguous()
    return sh, max(sh.stride(0), k), k


def _cov(cov, n):
    if cov.dim() == 3 and cov.shape[1:] == (3, 3):
        return cov.contiguous(), SARR_COV33
    if cov.dim() == 2 and cov.shape[1] == 6:
        return cov.contiguous(), SARR_COV6
    if cov.numel() == 6 * n:
        return cov.reshape(n, 6).contiguous(), SARR_COV6
    raise RuntimeError(f"covariance must be [N,6] or [N,3,3], got {tuple(cov.shape)}")


def prepare_inputs(means, cov, transmittance, sh):
    """Validates and normalises the four Gaussian tensors."""
    means = _as_cuda_f32(means, "means_world")
    n = means.shape[0]
    if means.dim() != 2 or means.shape[1] != 3:
        raise RuntimeError(f"means_world must be [N,3], got {tuple(means.shape)}")
    cov, layout = _cov(_as_cuda_f32(cov, "cov_world"), n)
    sigma = _as_cuda_f32(transmittance, "transmittance")
    if sigma.numel() != n:
        raise RuntimeError(f"transmittance must have N={n} elements, got {sigma.numel()}")
    sigma = sigma.reshape(n).contiguous()
    sh, sh_stride, sh_k = _sh_rows(_as_cuda_f32(sh, "sh_coeffs"), n)
    dev = means.device
    for name, t in (("cov_world", cov), ("transmittance", sigma), ("sh_coeffs", sh)):
        if t.device != dev:
            raise RuntimeError(f"{name} is on {t.device}, means_world on {dev}")
    return means.contiguous(), cov, layout, sigma, sh, sh_stride, sh_k


def workspace_bytes(n, nr, na, n_views=1, flags=0):
    out = ctypes.c_size_t()
    _check(lib().sarr_workspace_size(n, nr, na, n_views, flags, ctypes.byref(out)),
           "sarr_workspace_size")
    return out.value


def state_bytes(n, nr, na):
    out = ctypes.c_size_t()
    _check(lib().sarr_state_size(n, nr, na, ctypes.byref(out)), "sarr_state_size")
    return out.value


def _views_array(views):
    arr = (SarrView * len(views))()
    for i, v in enumerate(views):
        arr[i] = v
    return arr


def forward(views, means, cov, layout, sigma, sh, sh_stride, sh_k, images, omega=None,
            states=None, ws=None, check_device=False):
    """sarr_forward on the current stream of the inputs' device."""
    n = means.shape[0]
    nv = len(views)
    nr, na = views[0].range_samples, views[0].azimuth_samples
    dev = means.device
    with torch.cuda.device(dev):
        if ws is None:
            ws = torch.empty(workspace_bytes(n, nr, na, nv, SARR_FLAG_OMEGA if omega is not None else 0),
                             dtype=torch.uint8, device=dev)
        st = _stream(dev)
        status = lib().sarr_forward(_views_array(views), nv, n, _ptr(means), _ptr(cov), layout,
                                    _ptr(sigma), _ptr(sh), sh_stride, sh_k, _ptr(images),
                                    _ptr(omega), _ptr(states), _ptr(ws), ws.numel(), st)
        _check(status, "sarr_forward")
        if check_device:
            _check(lib().sarr_check_device_errors(_ptr(ws), ws.numel(), st), "sarr_forward (device)")
    return images


def backward(views, means, cov, layout, sigma, sh, sh_stride, sh_k, grad_images, grad_means,
             grad_cov, grad_cov_layout, grad_sigma, grad_sh, grad_norm=None, states=None,
             accumulate=False, ws=None, check_device=False, tiles_only=False):
    """sarr_backward on the current stream of the inputs' device (tiles_only:
    the per-tile pass only, rows then written by backward_scatter)."""
    n = means.shape[0]
    nv = len(views)
    nr, na = views[0].range_samples, views[0].azimuth_samples
    dev = means.device
    with torch.cuda.device(dev):
        if ws is None:
            ws = torch.empty(workspace_bytes(n, nr, na, nv, 0), dtype=torch.uint8, device=dev)
        st = _stream(dev)
        status = lib().sarr_backward(
            _views_array(views), nv, n, _ptr(means), _ptr(cov), layout, _ptr(sigma), _ptr(sh),
            sh_stride, sh_k, _ptr(grad_images), _ptr(states), _ptr(grad_means), _ptr(grad_cov),
            grad_cov_layout, _ptr(grad_sigma), _ptr(grad_sh), grad_sh.shape[1] if grad_sh.dim() == 2 else 16,
            _ptr(grad_norm), (SARR_FLAG_ACCUMULATE if accumulate else 0) |
            (SARR_FLAG_TILES_ONLY if tiles_only else 0), _ptr(ws), ws.numel(), st)
        _check(status, "sarr_backward")
        if check_device:
            _check(lib().sarr_check_device_errors(_ptr(ws), ws.numel(), st), "sarr_backward (device)")


def backward_scatter(views, n, begin, end, grad_means, grad_cov, grad_cov_layout, grad_sigma,
                     grad_sh, ws, states=None, grad_norm=None, accumulate=False, range_rows=False):
    """sarr_backward_scatter: gradient rows [begin, end) after a tiles_only
    backward of the same views on `ws` (range_rows: the arrays hold only those
    rows)."""
    dev = grad_means.device
    with torch.cuda.device(dev):
        _check(lib().sarr_backward_scatter(
            _views_array(views), len(views), n, _ptr(states), int(begin), int(end), _ptr(grad_means),
            _ptr(grad_cov), grad_cov_layout, _ptr(grad_sigma), _ptr(grad_sh),
            grad_sh.shape[1] if grad_sh.dim() == 2 else 16, _ptr(grad_norm),
            (SARR_FLAG_ACCUMULATE if accumulate else 0) | (SARR_FLAG_RANGE_ROWS if range_rows else 0),
            _ptr(ws), ws.numel(), _stream(dev)), "sarr_backward_scatter")


def debug_preprocess(view, means, cov, layout, sigma, sh, sh_stride, sh_k):
    n = means.shape[0]
    dev = means.device
    f = torch.empty((13, n), dtype=torch.float32, device=dev)
    q = torch.empty((10, n), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _check(lib().sarr_debug_preprocess(ctypes.byref(view), n, _ptr(means), _ptr(cov), layout,
                                           _ptr(sigma), _ptr(sh), sh_stride, sh_k, _ptr(f), _ptr(q),
                                           _stream(dev)), "sarr_debug_preprocess")
    return f, q


def debug_tile_lists(view, means, cov, layout, sigma):
    n = means.shape[0]
    dev = means.device
    nr, na = view.range_samples, view.azimuth_samples
    T = ((na + 15) // 16) * ((nr + 15) // 16)
    out = [torch.empty(T, dtype=torch.int32, device=dev), torch.empty((T, 64), dtype=torch.int32, device=dev),
           torch.empty((T, 64), dtype=torch.int32, device=dev), torch.empty(T, dtype=torch.int32, device=dev),
           torch.empty((T, 64), dtype=torch.int32, device=dev), torch.empty((T, 64), dtype=torch.int32, device=dev)]
    with torch.cuda.device(dev):
        ws = torch.empty(workspace_bytes(n, nr, na, 1, SARR_FLAG_OMEGA), dtype=torch.uint8, device=dev)
        _check(lib().sarr_debug_tile_lists(ctypes.byref(view), n, _ptr(means), _ptr(cov), layout,
                                           _ptr(sigma), *[_ptr(t) for t in out], _ptr(ws), ws.numel(),
                                           _stream(dev)), "sarr_debug_tile_lists")
    return out


def debug_view_constants(view, device):
    """The 30 per-view floats the kernels use (device trig included)."""
    out = torch.empty(30, dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _check(lib().sarr_debug_view_constants(ctypes.byref(view), _ptr(out), _stream(device)),
               "sarr_debug_view_constants")
    return out


def tile_rect(r_min, r_max, c_min, c_max, nr, na):
    """(tc0, tc1, tr0, tr1) of a pixel bbox (host-only test hook)."""
    out = [ctypes.c_int32() for _ in range(4)]
    _check(lib().sarr_debug_tile_rect(r_min, r_max, c_min, c_max, nr, na,
                                      *[ctypes.byref(o) for o in out]), "sarr_debug_tile_rect")
    return tuple(o.value for o in out)


def launch_count():
    return int(lib().sarr_launch_count())


KERNEL_KINDS = 15


def profile_enable(on=True):
    _check(lib().sarr_profile_enable(1 if on else 0), "sarr_profile_enable")


def profile_read():
    """{kernel name: (total device ms, launches)} since the last read."""
    ms = (ctypes.c_double * KERNEL_KINDS)()
    cnt = (ctypes.c_int64 * KERNEL_KINDS)()
    _check(lib().sarr_profile_read(ms, cnt, KERNEL_KINDS), "sarr_profile_read")
    return {lib().sarr_kernel_name(k).decode(): (ms[k], cnt[k]) for k in range(KERNEL_KINDS)}


def gaussian_params(scales_log, rotations, opacity_logits=None, layout=SARR_COV33):
    """sarr_gaussian_params: (cov [n,3,3] or [n,6] or None, sigmoid(opacity_logits)
    or None); scales_log/rotations may be None to compute the transmittance only."""
    cov = sigma = None
    if scales_log is not None:
        scales_log = _as_cuda_f32(scales_log, "scales").contiguous()
        rotations = _as_cuda_f32(rotations, "rotations").contiguous()
        n = scales_log.shape[0]
        if scales_log.shape != (n, 3) or rotations.shape != (n, 4):
            raise RuntimeError("scales must be [N,3] and rotations [N,4]")
        dev = scales_log.device
        cov = torch.empty((n, 3, 3) if layout == SARR_COV33 else (n, 6), dtype=torch.float32, device=dev)
    if opacity_logits is not None:
        opacity_logits = _as_cuda_f32(opacity_logits, "opacity").contiguous().reshape(-1)
        if cov is not None and opacity_logits.numel() != n:
            raise RuntimeError("opacity must have N elements")
        n = opacity_logits.numel()
        dev = opacity_logits.device
        sigma = torch.empty_like(opacity_logits)
    if cov is None and sigma is None:
        return None, None
    with torch.cuda.device(dev):
        _check(lib().sarr_gaussian_params(n, _ptr(scales_log), _ptr(rotations), _ptr(cov), layout,
                                          _ptr(opacity_logits), _ptr(sigma), _stream(dev)),
               "sarr_gaussian_params")
    return cov, sigma


def combined_loss(pred, target, l1_weight, ssim_weight, window_size=5, l1_mode="plain",
                  want_grad=True):
    """sarr_combined_loss on [V,H,W] images: (losses [3] device tensor = total,
    L1, D-SSIM; d total / d pred or None)."""
    pred = _as_cuda_f32(pred, "pred").contiguous()
    target = _as_cuda_f32(target, "target").contiguous()
    if pred.shape != target.shape or pred.dim() != 3:
        raise RuntimeError("pred and target must both be [V,H,W]")
    v, h, w = pred.shape
    dev = pred.device
    sz = ctypes.c_size_t()
    _check(lib().sarr_loss_workspace_size(v, h, w, ctypes.byref(sz)), "sarr_loss_workspace_size")
    ws = torch.empty(sz.value, dtype=torch.uint8, device=dev)
    losses = torch.empty(3, dtype=torch.float32, device=dev)
    grad = torch.empty_like(pred) if want_grad else None
    with torch.cuda.device(dev):
        _check(lib().sarr_combined_loss(v, h, w, _ptr(pred), _ptr(target), float(l1_weight),
                                        float(ssim_weight), int(window_size), SARR_L1_MODES[l1_mode],
                                        _ptr(losses), _ptr(grad), _ptr(ws), ws.numel(), _stream(dev)),
               "sarr_combined_loss")
    return losses, grad


def adam_step(param, grad, exp_avg, exp_avg_sq, segments, step, beta1=0.9, beta2=0.999, eps=1e-8):
    """sarr_adam_step over flat (1-D view) fp32 device tensors of equal length;
    `segments` = [(end, lr), ...] with ascending ends covering the tensors."""
    t = [_as_cuda_f32(x, nm) for x, nm in ((param, "param"), (grad, "grad"), (exp_avg, "exp_avg"),
                                           (exp_avg_sq, "exp_avg_sq"))]
    count = t[0].numel()
    for x in t:
        if x.numel() != count or not x.is_contiguous():
            raise RuntimeError("Adam buffers must be contiguous and of equal length")
    k = len(segments)
    ends = (ctypes.c_int64 * k)(*[int(e) for e, _ in segments])
    lrs = (ctypes.c_float * k)(*[float(lr) for _, lr in segments])
    dev = t[0].device
    with torch.cuda.device(dev):
        _check(lib().sarr_adam_step(count, *[_ptr(x) for x in t], k, ends, lrs, float(beta1),
                                    float(beta2), float(eps), int(step), _stream(dev)),
               "sarr_adam_step")


def densify_and_prune(means, scales, rotations, opacities, sh, grad_means, grad_threshold,
                      size_threshold, large_scale_threshold, opacity_threshold, max_gaussians):
    """sarr_densify_flags + sarr_densify_apply with the reference's
    max_gaussians decisions in between: (new means, scales, rotations,
    opacities (same trailing shape as the input), sh, (clones, splits, prunes,
    new))."""
    dev = means.device
    n = means.shape[0]
    t = [_as_cuda_f32(x, nm).contiguous() for x, nm in
         ((means, "means"), (scales, "scales"), (rotations, "rotations"), (opacities, "opacities"),
          (sh, "sh"), (grad_means, "grad_means"))]
    means, scales, rotations, op, sh, grad_means = t
    sh_cols = sh.shape[1] if sh.dim() == 2 else 0
    sz = ctypes.c_size_t()
    _check(lib().sarr_densify_workspace_size(n, ctypes.byref(sz)), "sarr_densify_workspace_size")
    ws = torch.empty(max(sz.value, 256), dtype=torch.uint8, device=dev)
    counts = torch.zeros(3, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        st = _stream(dev)
        _check(lib().sarr_densify_flags(n, _ptr(scales), _ptr(op), _ptr(grad_means), float(grad_threshold),
                                        float(size_threshold), float(large_scale_threshold),
                                        float(opacity_threshold), _ptr(counts), _ptr(ws), ws.numel(), st),
               "sarr_densify_flags")
        kept, clones, splits = (int(x) for x in counts.tolist())
        prunes = n - kept
        # gaussian_model.py:504 and :523: the tests against max_gaussians use
        # the count after pruning
        do_c = clones > 0 and kept + clones < max_gaussians
        added = clones if do_c else 0
        do_s = splits > 0 and kept + added + splits < max_gaussians
        m = kept + added + (2 * splits if do_s else 0)
        out = (torch.empty((m, 3), device=dev), torch.empty((m, 3), device=dev),
               torch.empty((m, 4), device=dev), torch.empty((m,) + tuple(opacities.shape[1:]), device=dev),
               torch.empty((m, sh_cols), device=dev))
        _check(lib().sarr_densify_apply(n, _ptr(means), _ptr(scales), _ptr(rotations), _ptr(op), _ptr(sh),
                                        sh_cols, _ptr(grad_means), _ptr(counts), int(do_c), int(do_s),
                                        _ptr(out[0]), _ptr(out[1]), _ptr(out[2]), _ptr(out[3]),
                                        _ptr(out[4]), _ptr(ws), ws.numel(), st), "sarr_densify_apply")
    new = (clones if do_c else 0) + (2 * splits if do_s else 0)
    return out, (clones, splits, prunes, new)
