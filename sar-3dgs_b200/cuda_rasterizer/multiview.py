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


def bucket_bounds(total: int, buckets: int, align: int = 64):
    """[a, b) ranges splitting `total` elements into at most `buckets`
    consecutive buckets whose starts are multiples of `align` elements."""
    if total <= 0:
        return []
    step = -(-total // max(1, buckets) // align) * align
    return [(a, min(total, a + step)) for a in range(0, total, step)]


def flat_segments(n: int, k: int, g0: int, g1: int):
    """The parts of Gaussians [g0, g1) in a flat buffer laid out as
    means [n,3] | opacity logits [n] | SH [n,k]: [(start, stop, group)] with
    group 0 = means, 1 = logits, 2 = SH."""
    return [(3 * g0, 3 * g1, 0), (3 * n + g0, 3 * n + g1, 1), (4 * n + k * g0, 4 * n + k * g1, 2)]


class ViewParallelTrainer:
    """Data-parallel training step over radar views, one process per GPU.

    The step of the reference's TrainingPipeline.train_step
    (training/training_pipeline.py:148-212: render -> CombinedLoss ->
    backward -> optimizer.step()) widened to a batch of views per step and
    sharded by view over the ranks of `group`:

      1. Gaussian parameters: covariance from log-scales and quaternions
         (detached, as GaussianModel.compute_covariance_full caches it) and
         the sigmoid transmittance (sarr_gaussian_params);
      2. forward of this rank's views keeping their tile states (sarr_forward);
      3. CombinedLoss (L1 + D-SSIM) against the targets and its image gradient
         (sarr_combined_loss), weighted by 1 / world so that the summed
         gradients are those of the mean loss over all ranks' views;
      4. backward of the views reusing the states: the per-tile pass
         (sarr_backward with SARR_FLAG_TILES_ONLY), then, bucket by bucket
         of `buckets` Gaussian ranges, the dense gradient rows of the range
         written straight into the bucket's part of the gradient buffer
         (sarr_backward_scatter with SARR_FLAG_RANGE_ROWS), the
         transmittance gradient chained through the sigmoid, and the
         bucket's NCCL all-reduce issued (async), so that the all-reduce of
         bucket b overlaps the rows of bucket b + 1;
      5. each bucket's Adam update (sarr_adam_step) queued behind its own
         all-reduce.

    Trainable parameters (the ones that receive gradients in SAR-3DGS: means,
    opacity logits, SH) live in one flat fp32 buffer laid out as
    means [n,3] | logits [n] | SH [n,K], with the Adam moments in the same
    layout and the gradients bucket by bucket (each bucket's means, logits
    and SH rows contiguous; `gradients()` gives them in the parameter
    layout); log-scales and quaternions are held but get no gradient
    (the covariance is detached, gaussian_model.py:306-315), so Adam leaves
    them alone as torch.optim.Adam does for parameters without gradients.
    Learning rates per group follow train.py:429-435 (lr for means and
    opacity, lr / 100 for SH). Every rank must call step() the same number of
    times with the same number of views (the all-reduces are collective).
    """

    def __init__(self, means, scales_log, rotations, opacity_logits, sh, lr=1e-3, group=None,
                 buckets=4, l1_weight=1.0, ssim_weight=0.2, window_size=5, betas=(0.9, 0.999),
                 eps=1e-8, distributed=True):
        from . import _native
        self._N = _native
        dev = means.device
        n, k = means.shape[0], sh.shape[1]
        self.n, self.k, self.device = n, k, dev
        self.group = group
        # distributed=False: a single-process trainer even inside a process group
        self.world = (dist.get_world_size(group) if distributed and dist.is_available()
                      and dist.is_initialized() else 1)
        total = n * (4 + k)
        self.param = torch.empty(total, dtype=torch.float32, device=dev)
        self.means = self.param[:3 * n].view(n, 3)
        self.logits = self.param[3 * n:4 * n]
        self.sh = self.param[4 * n:].view(n, k)
        self.means.copy_(means)
        self.logits.copy_(opacity_logits.reshape(n))
        self.sh.copy_(sh)
        self.scales = scales_log.detach().contiguous().clone()
        self.rotations = rotations.detach().contiguous().clone()
        self.exp_avg = torch.zeros_like(self.param)
        self.exp_avg_sq = torch.zeros_like(self.param)
        self.g_cov = torch.empty((n, 6), dtype=torch.float32, device=dev)  # reaches no parameter
        self.cov6 = torch.empty((n, 6), dtype=torch.float32, device=dev)
        self.sigma = torch.empty((n,), dtype=torch.float32, device=dev)
        self.group_lr = (lr, lr, lr * 0.01)  # means, opacity, SH (train.py:429-435)
        # Gaussian ranges of the buckets (starts on 256-Gaussian multiples);
        # one rank has no all-reduce to overlap, so one bucket
        self.bounds = bucket_bounds(n, buckets if self.world > 1 else 1, align=256)
        # gradients laid out by bucket: bucket b = its Gaussians' means rows |
        # logits | SH rows, contiguous, so that one all-reduce covers it
        self.grad = torch.zeros_like(self.param)
        self.gparts = []  # per bucket: (offset, means [nb,3], logits [nb], SH [nb,K], whole)
        o = 0
        for g0, g1 in self.bounds:
            nb = g1 - g0
            self.gparts.append((o, self.grad[o:o + 3 * nb].view(nb, 3), self.grad[o + 3 * nb:o + 4 * nb],
                                self.grad[o + 4 * nb:o + (4 + k) * nb].view(nb, k),
                                self.grad[o:o + (4 + k) * nb]))
            o += (4 + k) * nb
        self.loss_w = (l1_weight / self.world, ssim_weight / self.world, window_size)
        self.betas, self.eps = betas, eps
        self.steps_done = 0
        # SH coefficients in use (the active degree's (d + 1)^2): the others
        # are neither rendered nor given gradients, as the reference's
        # get_active_sh_coeffs slice (gaussian_model.py:334-337) leaves them
        self.sh_active = k
        self._buf_key = None
        self._args = None

    def _buffers(self, views):
        """Buffers and C-call arguments for this views list (rebuilt when the
        list object or its size changes)."""
        import ctypes
        N = self._N
        nr, na, V = views[0].range_samples, views[0].azimuth_samples, len(views)
        key = (id(views), nr, na, V)
        if key != self._buf_key:
            dev = self.device
            if self._buf_key is None or self._buf_key[1:] != key[1:]:
                self.ws = torch.empty(N.workspace_bytes(self.n, nr, na, V), dtype=torch.uint8,
                                      device=dev)
                self.sbytes = N.state_bytes(self.n, nr, na)
                self.states = torch.empty(V * self.sbytes, dtype=torch.uint8, device=dev)
                self.images = torch.empty((V, nr, na), dtype=torch.float32, device=dev)
                self.grad_images = torch.empty_like(self.images)
                self.losses = torch.empty(3, dtype=torch.float32, device=dev)
                sz = ctypes.c_size_t()
                N._check(N.lib().sarr_loss_workspace_size(V, nr, na, ctypes.byref(sz)),
                         "sarr_loss_workspace_size")
                self.loss_ws = torch.empty(max(sz.value, 256), dtype=torch.uint8, device=dev)
            self._vs = N._views_array(views)
            self._views_ref = views  # keeps id(views) from being reused while cached
            self._buf_key = key
        return nr, na, V

    def _call_args(self):
        """Device pointers and per-bucket Adam ranges (built once)."""
        import ctypes
        if getattr(self, "_args", None) is None:
            P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
            a = {name: P(getattr(self, name)) for name in (
                "scales", "rotations", "cov6", "logits", "sigma", "means", "sh", "param", "grad",
                "exp_avg", "exp_avg_sq", "g_cov")}
            ranges, gptr = [], []
            for (g0, g1), (o, gm, gl, gsh, _) in zip(self.bounds, self.gparts):
                nb = g1 - g0
                segs = flat_segments(self.n, self.k, g0, g1)
                ranges.append(((ctypes.c_int64 * 3)(*[x[0] for x in segs]),
                               (ctypes.c_int64 * 3)(*[x[1] for x in segs]),
                               (ctypes.c_int64 * 3)(o, o + 3 * nb, o + 4 * nb),
                               (ctypes.c_float * 3)(*[self.group_lr[x[2]] for x in segs])))
                gptr.append((P(gm), P(gl), P(gsh)))
            a["ranges"] = ranges
            a["gptr"] = gptr
            self._args = a
        return self._args

    def step(self, views, targets, update=True):
        """One training step over this rank's `views` (SarrView list) against
        `targets` [V, Nr, Na] (the rasterizer's memory layout). Returns this
        rank's losses [3] (total, L1, D-SSIM; device tensor) of the weighted
        loss (the mean over all ranks' views is their sum). update=False
        stops after the all-reduces: the summed gradients are in place
        (gradients()) and no parameter changes."""
        import ctypes
        N = self._N
        L = N.lib()
        nr, na, V = self._buffers(views)
        A = self._call_args()
        n, k = self.n, self.k
        dev = self.device
        P = N._ptr
        vs, ws, wsb, states = self._vs, P(self.ws), self.ws.numel(), P(self.states)
        with torch.cuda.device(dev):
            st = N._stream(dev)
            N._check(L.sarr_gaussian_params(n, A["scales"], A["rotations"], A["cov6"], N.SARR_COV6,
                                            A["logits"], A["sigma"], st), "sarr_gaussian_params")
            ka = self.sh_active
            N._check(L.sarr_forward(vs, V, n, A["means"], A["cov6"], N.SARR_COV6, A["sigma"], A["sh"],
                                    k, ka, P(self.images), None, states, ws, wsb, st), "sarr_forward")
            l1w, ssw, win = self.loss_w
            N._check(L.sarr_combined_loss(V, nr, na, P(self.images), P(targets), float(l1w),
                                          float(ssw), int(win), 0, P(self.losses),
                                          P(self.grad_images), P(self.loss_ws),
                                          self.loss_ws.numel(), st), "sarr_combined_loss")
            gm0, gl0, gsh0 = A["gptr"][0]
            N._check(L.sarr_backward(vs, V, n, A["means"], A["cov6"], N.SARR_COV6, A["sigma"],
                                     A["sh"], k, ka, P(self.grad_images), states, gm0, A["g_cov"],
                                     N.SARR_COV6, gl0, gsh0, k, None, N.SARR_FLAG_TILES_ONLY, ws, wsb,
                                     st), "sarr_backward")
            # d sigmoid(logit) / d logit = sigma (1 - sigma); the same on every
            # rank, so it may be applied before the sum over ranks
            dsig = self.sigma * (1.0 - self.sigma)
            works = []
            for b, (g0, g1) in enumerate(self.bounds):
                gm, gl, gsh = A["gptr"][b]
                N._check(L.sarr_backward_scatter(vs, V, n, states, g0, g1, gm, A["g_cov"], N.SARR_COV6,
                                                 gl, gsh, k, None, N.SARR_FLAG_RANGE_ROWS, ws, wsb,
                                                 st), "sarr_backward_scatter")
                self.gparts[b][2].mul_(dsig[g0:g1])
                if ka < k:
                    self.gparts[b][3][:, ka:].zero_()
                works.append(self._allreduce_bucket(b))
            if not update:
                for w in (w for ws_ in works for w in ws_):
                    w.wait()
                return self.losses
            self.steps_done += 1
            self._update(works, st)
        return self.losses

    def reset_optimizer(self):
        """Adam from scratch (zero moments, step count 0), as the reference's
        optimizer.state.clear() after densification."""
        self.exp_avg.zero_()
        self.exp_avg_sq.zero_()
        self.steps_done = 0

    def apply_update(self):
        """The Adam update of the gradients in place (after step(update=False))."""
        N = self._N
        with torch.cuda.device(self.device):
            self.steps_done += 1
            self._update([], N._stream(self.device))

    def _allreduce_bucket(self, b):
        if self.world == 1:
            return []
        return [dist.all_reduce(self.gparts[b][4], group=self.group, async_op=True)]

    def gradients(self):
        """The last step's gradients (summed over the ranks) in the parameter
        layout: (means [n,3], opacity logits [n], SH [n,K])."""
        return (torch.cat([p[1] for p in self.gparts]), torch.cat([p[2] for p in self.gparts]),
                torch.cat([p[3] for p in self.gparts]))

    def _update(self, works, st):
        """Each bucket's Adam update (one launch over its means, opacity and
        SH ranges), queued behind its all-reduces."""
        N = self._N
        L = N.lib()
        A = self._call_args()
        b1, b2 = self.betas
        for i, (begin, end, gbegin, lr) in enumerate(A["ranges"]):
            for w in works[i] if works else []:
                w.wait()  # the current stream waits for this bucket's all-reduce
            N._check(L.sarr_adam_step_ranges(3, begin, end, gbegin, lr, A["param"], A["grad"],
                                             A["exp_avg"], A["exp_avg_sq"], float(b1), float(b2),
                                             float(self.eps), self.steps_done, st),
                     "sarr_adam_step_ranges")

    def allreduce_only(self):
        """The step's collectives alone (the same buckets, back to back), for
        measuring their cost; a no-op on one rank."""
        if self.world > 1:
            works = [w for b in range(len(self.bounds)) for w in self._allreduce_bucket(b)]
            for w in works:
                w.wait()


def sh_degree_at(iteration: int, interval: int = 1000, max_degree: int = 3) -> int:
    """Active SH degree at an iteration: one more every `interval` iterations
    up to max_degree (the 0 -> 3 ramp of full training; the reference's
    iteration rule is train_gui.py:951-961, with its own interval)."""
    return min(iteration // interval, max_degree)


def densify_due(iteration: int, n: int, interval: int = 100, start: int = 0,
                max_gaussians: int = 2_000_000) -> bool:
    """DensifyPruneManager.should_densify_or_prune (training/densify_prune.py:
    53-86) without its epoch throttle: past `start`, on a multiple of
    `interval`, and with the set below max_gaussians."""
    return iteration > start and iteration % interval == 0 and n < max_gaussians


class DensifyingTrainer:
    """Full training with densification and pruning, data-parallel over views:
    TrainingPipeline.train_step (training/training_pipeline.py:148-212) with
    DensifyPruneManager (training/densify_prune.py:53-141) and the SH-degree
    ramp, on ViewParallelTrainer.

    Each step sets the active SH degree from the iteration (sh_degree_at),
    computes the step's gradients and all-reduces them. When densification is
    due (densify_due), the Gaussian set is densified and pruned from the
    all-reduced means gradient (GaussianModel.densify_and_prune,
    gaussian_model.py:433-566, through sarr_densify_flags/_apply); every rank
    holds the same parameters and the same summed gradient, and the kernels
    are deterministic, so every rank gets the same new set. Then, as the
    reference's step does (optimizer.state.clear(), then optimizer.step()):
    if the set changed, this step updates nothing (the new parameters have no
    gradient) and training continues on a new ViewParallelTrainer over the new
    set; if it did not, Adam restarts from zero moments with this step's
    gradients. `history` records each densification as (iteration, n before,
    clones, splits, prunes, n after).
    """

    def __init__(self, means, scales_log, rotations, opacity_logits, sh, lr=1e-3, group=None,
                 buckets=4, densify_interval=100, densify_start=0, grad_threshold=2e-4,
                 size_threshold=0.01, large_scale_threshold=2.0, opacity_threshold=0.005,
                 max_gaussians=2_000_000, sh_interval=1000, max_sh_degree=3, **trainer_kw):
        self.lr, self.group, self.buckets, self.trainer_kw = lr, group, buckets, trainer_kw
        self.densify_interval, self.densify_start = densify_interval, densify_start
        self.thresholds = (grad_threshold, size_threshold, large_scale_threshold, opacity_threshold)
        self.max_gaussians = max_gaussians
        self.sh_interval, self.max_sh_degree = sh_interval, max_sh_degree
        self.iteration = 0
        self.history = []
        self.tr = self._trainer(means, scales_log, rotations, opacity_logits, sh)

    def _trainer(self, means, scales_log, rotations, logits, sh):
        return ViewParallelTrainer(means, scales_log, rotations, logits, sh, lr=self.lr,
                                   group=self.group, buckets=self.buckets, **self.trainer_kw)

    @property
    def n(self) -> int:
        return self.tr.n

    def step(self, views, targets):
        """One iteration over this rank's views; returns its losses [3]."""
        tr, it = self.tr, self.iteration
        degree = sh_degree_at(it, self.sh_interval, self.max_sh_degree)
        tr.sh_active = min((degree + 1) ** 2, tr.k)
        due = densify_due(it, tr.n, self.densify_interval, self.densify_start, self.max_gaussians)
        losses = tr.step(views, targets, update=not due)
        if due:
            self._densify()
        self.iteration += 1
        return losses

    def _densify(self):
        from . import densify as DZ
        tr = self.tr
        grad_means = tr.gradients()[0]
        out, counts = DZ.densify_and_prune_tensors(tr.means, tr.scales, tr.rotations, tr.logits, tr.sh,
                                                   grad_means, *self.thresholds, self.max_gaussians)
        clones, splits, prunes, new = counts
        n_before = tr.n
        if prunes == 0 and new == 0:
            tr.reset_optimizer()
            tr.apply_update()
        else:
            self.tr = self._trainer(*out)
        self.history.append((self.iteration, n_before, clones, splits, prunes, self.tr.n))
