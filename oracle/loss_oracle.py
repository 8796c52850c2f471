"""CPU restatement (numpy, float64) of the reference's training loss,
CombinedLoss of losses.py (SAR-3DGS), and of its gradient with respect to the
predicted image. Test infrastructure: the oracle of sarr_combined_loss in the tests.

Forward (losses.py:160-219): L1 = mean |p - t| (weighted by
1 + f(t / max t) for the weighted modes, losses.py:29-62); SSIM map from the
windowed means of p, t, p^2, t^2, p t with a Gaussian window (sigma 1.5,
losses.py:65-78) and zero padding (F.conv2d, padding = window // 2), C1 =
0.01^2, C2 = 0.03^2; total = l1_weight * L1 + ssim_weight * (1 - mean SSIM).

Gradient: with m = K*p, e2 = K*(p^2), ept = K*(p t), the SSIM map depends on
p only through (m, e2, ept), so d mean(SSIM) / d p_j = (1/N) sum_i
k(i - j) [dS/dm_i + 2 p_j dS/de2_i + t_j dS/dept_i] (K symmetric).
"""
import numpy as np

C1 = 0.01 ** 2
C2 = 0.03 ** 2


def gaussian_window(size, sigma=1.5):
    """losses.py:65-78 (in float32, as the reference computes it)."""
    coords = np.arange(size, dtype=np.float32) - size // 2
    g = np.exp(-(coords ** 2) / np.float32(2 * sigma ** 2)).astype(np.float32)
    g = g / g.sum()
    return np.outer(g, g).astype(np.float64)


def conv2d_same(x, k):
    """Correlation of each image of x [V,H,W] with k (zero padding)."""
    v, h, w = x.shape
    r = k.shape[0] // 2
    xp = np.zeros((v, h + 2 * r, w + 2 * r))
    xp[:, r:r + h, r:r + w] = x
    out = np.zeros((v, h, w))
    for a in range(k.shape[0]):
        for b in range(k.shape[1]):
            out += k[a, b] * xp[:, a:a + h, b:b + w]
    return out


def l1_weights(t, mode):
    tmax = t.max()
    if mode == "plain" or not tmax > 0:
        return np.ones_like(t)
    tn = t / tmax
    if mode == "square":
        return 1.0 + tn ** 2
    if mode == "sqrt":
        return 1.0 + np.sqrt(tn + 1e-8)
    return 1.0 + tn


def combined_loss(pred, target, l1_weight, ssim_weight, window, mode="plain"):
    """Returns (total, l1, dssim, d total / d pred) for images [V,H,W]."""
    p = np.asarray(pred, np.float64)
    t = np.asarray(target, np.float64)
    if p.ndim == 2:
        p, t = p[None], t[None]
    n = p.size
    k = gaussian_window(window)
    wgt = l1_weights(t, mode)
    l1 = float((np.abs(p - t) * wgt).mean())
    mp, mt = conv2d_same(p, k), conv2d_same(t, k)
    e2p, e2t, ept = conv2d_same(p * p, k), conv2d_same(t * t, k), conv2d_same(p * t, k)
    sp, st, spt = e2p - mp ** 2, e2t - mt ** 2, ept - mp * mt
    a1, a2 = 2 * mp * mt + C1, 2 * spt + C2
    b1, b2 = mp ** 2 + mt ** 2 + C1, sp + st + C2
    ssim = a1 * a2 / (b1 * b2)
    dssim = float(1.0 - ssim.mean())
    total = l1_weight * l1 + ssim_weight * dssim
    d_mp = 2 * mt * a2 / (b1 * b2) - ssim * 2 * mp / b1
    d_sp = -ssim / b2
    d_spt = 2 * a1 / (b1 * b2)
    dm = d_mp - 2 * mp * d_sp - mt * d_spt
    grad = l1_weight * wgt * np.sign(p - t) / n
    grad -= ssim_weight / n * (conv2d_same(dm, k) + 2 * p * conv2d_same(d_sp, k) + t * conv2d_same(d_spt, k))
    return total, l1, dssim, grad.reshape(np.shape(pred))
