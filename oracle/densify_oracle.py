"""CPU restatement (numpy) of GaussianModel.densify_and_prune
(gaussian_model.py:433-566 of SAR-3DGS), vectorised. Test infrastructure: the
oracle of sarr_densify_flags / sarr_densify_apply in the tests.

Flags (:464-475): clone = |exp(s)| < size and |grad| > g; split = |exp(s)| >
large and |grad| > g; prune = sigmoid(o) < opacity or |exp(s)| > large. New
set: kept Gaussians in order (:491-497), then clones with mean + 0.01 grad
(:504-521), then per split two Gaussians with scale log(0.8 exp(s)) and mean
offset (0.8 exp(s_x) * 0.5 cos a, 0.8 exp(s_y) * 0.5 sin a, 0), a = 0, pi
(:523-548); the max_gaussians tests use the count after pruning.
"""
import numpy as np


def densify_and_prune(means, scales, rotations, opacities, sh, grad, grad_threshold, size_threshold,
                      large_scale_threshold, opacity_threshold, max_gaussians):
    f = np.float32
    s = np.exp(scales.astype(f))
    snorm = np.sqrt((s * s).sum(axis=1))
    gnorm = np.sqrt((grad.astype(f) ** 2).sum(axis=1))
    small, large, high = snorm < f(size_threshold), snorm > f(large_scale_threshold), gnorm > f(grad_threshold)
    low_op = (1.0 / (1.0 + np.exp(-opacities.astype(f)))).reshape(-1) < f(opacity_threshold)
    clone, split, prune = small & high, large & high, low_op | large
    keep = ~prune
    out = [means[keep], scales[keep], rotations[keep], opacities[keep], sh[keep]]
    kept = int(keep.sum())
    nc, ns = int(clone.sum()), int(split.sum())
    added = 0
    if nc > 0 and kept + nc < max_gaussians:
        ci = np.nonzero(clone)[0]
        parts = [(means[ci] + grad[ci] * f(0.01)).astype(f), scales[ci], rotations[ci], opacities[ci], sh[ci]]
        out = [np.concatenate([a, b]) for a, b in zip(out, parts)]
        added = nc
    new = added
    if ns > 0 and kept + added + ns < max_gaussians:
        si = np.nonzero(split)[0]
        v = (s[si] * f(0.8)).astype(f)
        rows = []
        for cos_a, sin_a in ((1.0, 0.0), (-1.0, 1.2246467991473532e-16)):
            off = np.stack([(v[:, 0] * f(0.5)) * f(cos_a), (v[:, 1] * f(0.5)) * f(sin_a),
                            np.zeros(len(si), f)], axis=1)
            rows.append([(means[si] + off).astype(f), np.log(v).astype(f), rotations[si], opacities[si], sh[si]])
        # interleave: (split 0 at 0, split 0 at pi, split 1 at 0, ...)
        parts = [np.stack([rows[0][k], rows[1][k]], axis=1).reshape((-1,) + rows[0][k].shape[1:])
                 for k in range(5)]
        out = [np.concatenate([a, b]) for a, b in zip(out, parts)]
        new += 2 * ns
    return out, (nc, ns, int(prune.sum()), new)
