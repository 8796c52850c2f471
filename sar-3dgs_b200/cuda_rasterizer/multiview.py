"""View data-parallelism for the SAR rasterizer (one process per GPU).

Gaussians are replicated on every rank; radar views are sharded. A forward
sweep needs no communication. A training step renders and back-propagates
this rank's views (their gradients summed by one batched backward), then sums
the trainable gradients over ranks with one all-reduce. Only means, opacity
and SH gradients reach trainable parameters in SAR-3DGS (the covariance is
detached, gaussian_model.py:306-315), so those are the tensors reduced:
3 + 1 + K floats per Gaussian.
"""
from typing import List, Sequence

import torch
import torch.distributed as dist

from . import cuda_rasterizer_sar as M


def shard_range(n_items: int, rank: int, world: int):
    """Contiguous [start, stop) of rank `rank` among `world` ranks; sizes differ
    by at most one and the shards cover 0..n_items-1 exactly once."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_views(views: Sequence, rank: int, world: int) -> List:
    a, b = shard_range(len(views), rank, world)
    return list(views[a:b])


def allreduce_gradients(grads: Sequence[torch.Tensor], group=None, bucket_bytes: int = 64 << 20):
    """Sums `grads` over the ranks of `group` in place, packing them into
    flat buckets of at most `bucket_bytes` so that a few large collectives
    replace many small ones. Works with any torch.distributed backend (NCCL
    on GPUs, gloo on CPU)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return grads
    bucket: List[torch.Tensor] = []
    size = 0

    def flush():
        nonlocal bucket, size
        if not bucket:
            return
        flat = torch.cat([g.reshape(-1) for g in bucket])
        dist.all_reduce(flat, group=group)
        off = 0
        for g in bucket:
            g.copy_(flat[off:off + g.numel()].view_as(g))
            off += g.numel()
        bucket, size = [], 0

    for g in grads:
        nbytes = g.numel() * g.element_size()
        if size + nbytes > bucket_bytes and bucket:
            flush()
        bucket.append(g)
        size += nbytes
    flush()
    return grads


def render_views(means, cov, transmittance, sh, views, want_omega=False):
    """Forward of this rank's views (no communication)."""
    return M.render_sar_batched(means, cov, transmittance, sh, views, want_omega=want_omega)


def backward_views(means, cov, transmittance, sh, grad_images, views, group=None, sh_cols=16):
    """Summed backward of this rank's views followed by the all-reduce of the
    trainable gradients (means, transmittance, SH). Returns
    (grad_means, grad_cov, grad_transmittance, grad_sh, grad_norm); grad_cov is
    local (it reaches no trainable parameter) and grad_norm is recomputed from
    the reduced means gradient."""
    gm, gc, gs, gsh, gn = M.render_sar_backward_batched(
        means, cov, transmittance, sh, grad_images, views, grad_sh_cols=sh_cols, grad_norm=True)
    allreduce_gradients([gm, gs, gsh], group=group)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        gn = gm.norm(dim=1)
    return gm, gc, gs, gsh, gn
