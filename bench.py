#!/usr/bin/env python
"""Benchmark of the B200 SAR rasterizer.

Headline workload (the multi-view inference sweep): N = 1,000,000 Gaussians
in a 40 x 40 x 10 m box, 1,024 radar views per step (track angle stepped by
0.35 deg, incidence uniform 15-45 deg), 256 x 256 images at 0.2 m, forward
only. Seeded synthetic data (no dataset). With --gpus N (torchrun), every
rank renders its own 1,024-view sweep (offset track angles): per-GPU work is
fixed, views are independent, no collective on the forward data path.

value       forward views/s over all ranks, inputs resident in HBM, L2 flushed
            (512 MiB write) before every timed step, device time from CUDA
            events, max over ranks.
roofline    the dominant kernel against HBM bandwidth with the algorithmic
            bytes of the forward: 104 B per Gaussian per launch group of 256
            views (means, cov6, transmittance, SH read once per launch) plus
            4 B per pixel per view (the image written); path_roofline gives
            the same model for the whole step. render_issue gives the
            compositing kernel against its instruction-issue bound.
e2e         the same sweep through the public C ABI with host buffers: pinned
            host -> device copy of the scene, the render, and device -> host
            copy of all images every step, pipelined (the next step's upload
            and the image copies overlap the render) and timed as one region;
            host_ceiling is the same copies alone.
omega       the forward with the Omega output of render_sar (256 views per step).
fwd_bwd     forward + backward steps/s of one view at 1M Gaussians, 256 x 256
            (forward state reused by the backward, dense gradients for all N
            Gaussians), L2 flushed before every step, against its HBM bytes
            312 B per Gaussian + 8 B per pixel.
train_step  the data-parallel training step on the full-training shape (1M
            Gaussians, 256 x 256 at 0.2 m, 64 views per rank per step):
            parameter producer, forward, L1 + 0.2 D-SSIM loss and gradient,
            backward, NCCL all-reduce of the trainable gradients (N > 1) and
            Adam; steps/s (max over ranks) and the all-reduce's own cost.
train_full  full training with densification: 100k Gaussians growing by
            densify/prune every 100 iterations (cap 2M), SH degree ramp
            0 -> 3 every 1,000 iterations, 64 views per rank per step,
            --full-iters iterations (3,000); steps/s over the whole run, the
            densification record, the final N.
train_configs  (1 GPU) the training step on the 50k-Gaussian 64-view 128 px
            scene and on the 500k-Gaussian 16-view 512 px scene.

--impl reference runs the CPU restatement of the reference algorithm (the
reference ships no CPU implementation) on the host cores, forward and
forward + backward, and times the reference's own CUDA kernels on a few views
as `gpu_reference`.
"""
import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

REPO = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(REPO, "sar-3dgs_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

# The synthetic scenes only: importing the package loads no native library,
# so the reference arm below runs without libsarr.so in the process.
from cuda_rasterizer import synthetic as S  # noqa: E402

METRIC = "fwd views/s & fwd+bwd steps/s, 1M Gaussians 256², 1/8 B200; % HBM roofline"
HBM_FALLBACK_GBS = 6650.0
GROUP_VIEWS = 256          # views per internal launch group of sarr_forward
TRAIN_VIEWS_PER_RANK = 64  # views per rank per training step
# Issue model of the compositing kernel: B200 issues at most one warp
# instruction per cycle in each of the 4 schedulers of its 148 SMs; the
# reference's per-(pixel, listed record) work (offsets, quadratic form,
# exponent and cut-off test, exponential, alpha, the two compositing updates)
# needs at least 12 thread instructions even with the fastest exponential.
SMS, SCHEDULERS = 148, 4
MIN_INSTR_PER_PAIR = 12
# ncu figures of the compositing kernels on one 256-view launch of this
# workload (dram__bytes_read.sum + dram__bytes_write.sum, smsp__inst_executed
# .sum); they belong to this workload and these kernels only. render_kernel
# runs in calls with states or Omega; image-only calls run
# select_render_kernel (selection and compositing in one kernel).
NCU = {"render_kernel": {"dram_bytes": 118_546_432 + 38_688_768, "warp_instructions": 299_738_669},
       "select_render_kernel": {"dram_bytes": 103_740_416 + 41_093_376, "warp_instructions": 439_858_375}}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=1_000_000)
    ap.add_argument("--views", type=int, default=1024)
    ap.add_argument("--samples", type=int, default=256)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-train", action="store_true",
                    help="skip fwd_bwd, train_step, train_full, train_configs, train_ops")
    ap.add_argument("--full-iters", type=int, default=3000,
                    help="iterations of the full-training run with densification (train_full)")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--sections", default="all",
                    help="comma-separated subset of forward,e2e,omega,fwd_bwd,train_step,"
                         "train_full,train_configs,train_ops,cpu (default all; without forward the line "
                         "carries no headline value, for profiling runs)")
    return ap.parse_args()


def wanted(args, name):
    if args.sections == "all":
        return True
    return name in args.sections.split(",")


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return HBM_FALLBACK_GBS, "fallback"


def roof(bytes_, seconds, extra=None):
    peak, kind = peaks()
    gbs = bytes_ / seconds / 1e9
    out = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
           "frac": round(gbs / peak, 4), "peak_source": kind + " (copy bandwidth)"}
    if extra:
        out.update(extra)
    return out


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
        self.device = torch.device("cuda", self.local)

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x):
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x):
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons during a region."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
            if not self.uuid.startswith("GPU-"):
                self.uuid = "GPU-" + self.uuid
        except Exception:
            self.uuid = None

    def start(self):
        self.out = tempfile.TemporaryFile(mode="w+")
        try:
            cmd = ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                   "-lms", "50"]
            if self.uuid:
                cmd[1:1] = ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
            time.sleep(0.2)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.out.seek(0)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def flush_l2(buf, k):
    buf.fill_(float(k % 7))


def make_scene(args, device):
    if args.n == 1_000_000:
        return S.named_scene("sweep_1m", seed=0, device=device)
    return S.make_scene(args.n, (40.0, 40.0, 10.0), (0.05, 0.5), seed=0, device=device)


def rank_views(args, d):
    return S.sweep_views(args.views, samples=args.samples, offset_deg=0.35 * d.rank / max(d.world, 1))


def image_digest(images):
    """(float64 sum, SHA-1 prefix of the bytes) of a step's images; the hash
    is bit-exact, the sum is for reading (its reduction order may vary)."""
    host = images.cpu()
    return (float(host.double().sum().item()),
            hashlib.sha1(host.numpy().tobytes()).hexdigest()[:16])


def _a256(x):
    return (x + 255) // 256 * 256


def listed_pairs(N, inputs, views, n, s, dev, flush):
    """(pixel, listed record) pairs of the compositing of these views: the
    sum over views and tiles of the list length times the tile's pixels,
    read from the per-view forward states (256 x 256 images: every tile is
    16 x 16); and the per-kernel device times of a second such call (after
    an L2 flush), whose selection and compositing run as separate kernels."""
    T = (s // 16) ** 2
    sb = N.state_bytes(n, s, s)
    states = torch.empty(len(views) * sb, dtype=torch.uint8, device=dev)
    img = torch.empty((len(views), s, s), dtype=torch.float32, device=dev)
    N.forward(views, *inputs, img, states=states)
    o = _a256(4 * n)
    counts = states.view(len(views), sb)[:, o:o + 4 * T].contiguous().view(torch.int32)
    total = int(counts.to(torch.int64).sum().item()) * 256
    flush_l2(flush, 0)
    torch.cuda.synchronize()
    N.profile_enable(True)
    N.forward(views, *inputs, img, states=states)
    torch.cuda.synchronize()
    prof = N.profile_read()
    N.profile_enable(False)
    del states
    return total, prof


def bench_forward(args, d):
    from cuda_rasterizer import _native as N
    dev = d.device
    torch.cuda.set_device(dev)
    sc = make_scene(args, dev)
    inputs = N.prepare_inputs(sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
    n, s = args.n, args.samples
    views = [N.make_view(*t) for t in rank_views(args, d)]
    V = len(views)
    images = torch.empty((V, s, s), dtype=torch.float32, device=dev)
    ws = torch.empty(N.workspace_bytes(n, s, s, V), dtype=torch.uint8, device=dev)
    flush = torch.empty((512 << 20) // 4, dtype=torch.float32, device=dev)

    def step():
        N.forward(views, *inputs, images, ws=ws)

    for k in range(args.warmup):
        flush_l2(flush, k)
        step()
    torch.cuda.synchronize()
    checksum0 = image_digest(images)
    d.barrier()

    clocks = Clocks(dev)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    torch.cuda.synchronize()
    d.barrier()
    l0 = N.launch_count()
    for k in range(args.steps):
        flush_l2(flush, k)
        ev[k][0].record()
        step()
        ev[k][1].record()
    torch.cuda.synchronize()
    launches = N.launch_count() - l0
    d.barrier()
    clk = clocks.stop()
    t_ms = sum(a.elapsed_time(b) for a, b in ev)
    t_ms_max = d.max(t_ms)
    value = d.sum(float(V * args.steps)) / (t_ms_max / 1e3)
    checksum = image_digest(images)  # guards against a step doing no work

    # per-kernel device time from the library's event hooks (launch stream)
    N.profile_enable(True)
    rsteps = min(args.steps, 5)
    for k in range(rsteps):
        flush_l2(flush, k)
        step()
    torch.cuda.synchronize()
    prof = N.profile_read()
    N.profile_enable(False)
    kernels = {k: {"ms_per_step": round(v[0] / rsteps, 4), "launches_per_step": v[1] / rsteps,
                   "avg_launch_us": round(v[0] / v[1] * 1e3, 2)}
               for k, v in prof.items() if v[1]}
    # the dominant kernel ("aux" groups several small kernels, so it is not one)
    dominant = max((kv for kv in prof.items() if kv[0] != "aux" and kv[1][1]),
                   key=lambda kv: kv[1][0])[0]
    dom_ms, dom_launches = prof[dominant]
    launch_views = V / (dom_launches / rsteps)
    npix = s * s
    fwd_bytes = 104 * n + 4 * npix * launch_views  # one launch group (SURVEY model, batched)
    dom_s = dom_ms / dom_launches / 1e3
    full = n == 1_000_000 and s == 256 and launch_views == GROUP_VIEWS
    roofline = roof(fwd_bytes, dom_s, {
        "kernel": dominant, "traffic": (NCU[dominant]["dram_bytes"] if full and dominant in NCU
                                        else None),
        "bytes_per_launch": int(fwd_bytes), "views_per_launch": launch_views,
        "avg_launch_us": round(dom_s * 1e6, 2),
        "model": "104 B/Gaussian per launch group + 4 B/pixel per view"})
    groups = -(-V // GROUP_VIEWS)
    step_bytes = 104 * n * groups + 4 * npix * V
    path = roof(step_bytes, t_ms_max / args.steps / 1e3,
                {"bytes_per_step": int(step_bytes), "model": roofline["model"]})
    path["achieved_total_gbs"] = round(path["achieved"] * d.world, 1)

    # the compositing against its instruction-issue bound, timed in a call of
    # one launch group with states, where selection and compositing are
    # separate kernels; image-only calls (the timed steps above) run both in
    # select_render_kernel, whose launch time is set beside their sum
    render_issue = None
    gv = min(V, GROUP_VIEWS)
    pairs, sprof = listed_pairs(N, inputs, views[:gv], n, s, dev, flush)
    if sprof.get("render_kernel", (0.0, 0))[1]:
        r_ms, r_l = sprof["render_kernel"]
        per_launch_pairs = pairs / r_l
        f_hz = (clk["sm_mhz"] if clk else 1965.0) * 1e6
        bound_s = per_launch_pairs * MIN_INSTR_PER_PAIR / 32 / (SMS * SCHEDULERS * f_hz)
        r_s = r_ms / r_l / 1e3
        full_group = n == 1_000_000 and s == 256 and gv == GROUP_VIEWS
        fused = None
        if prof.get("select_render_kernel", (0.0, 0))[1] and gv == GROUP_VIEWS:
            f_ms, f_l = prof["select_render_kernel"]
            sel_ms = sprof.get("select_kernel", (0.0, 0))[0]
            fused = {"select_render_kernel_us": round(f_ms / f_l * 1e3, 2),
                     "select_kernel_plus_render_kernel_us": round((sel_ms + r_ms) / r_l * 1e3, 2)}
        render_issue = {"bound": "issue", "kernel": "render_kernel",
                        "timed_in": f"one {gv}-view call with states",
                        "pairs_per_launch": int(per_launch_pairs),
                        "min_thread_instr_per_pair": MIN_INSTR_PER_PAIR,
                        "bound_us": round(bound_s * 1e6, 2), "achieved_us": round(r_s * 1e6, 2),
                        "frac": round(bound_s / r_s, 4),
                        "ncu_thread_instr_per_pair": (round(NCU["render_kernel"]["warp_instructions"] * 32 /
                                                            per_launch_pairs, 2) if full_group else None),
                        "fused": fused}

    out = {"value": value, "ms_per_step": t_ms_max / args.steps, "launches": launches,
           "clocks": clk, "roofline": roofline, "path_roofline": path, "render_issue": render_issue,
           "kernels": kernels, "checksum": checksum, "checksum_stable": checksum == checksum0,
           "views_per_rank": V, "sc": sc, "inputs": inputs, "views": views, "flush": flush}
    return out


def bench_e2e(args, d, sc, views):
    """Host buffers in, host images out, through the C ABI, K steps as one
    pipeline: each step uploads the scene parameters from pinned host memory
    (upload stream, into one of two device buffer sets), renders its views in
    256-view groups, and copies every group's images back to pinned host
    memory (download stream) while the next group renders; step k+1's upload
    overlaps step k's render. The timed region runs from the first upload to
    the last image copy, so every step's copies lie inside it; L2 is flushed
    (512 MiB write) at the start of every step's render. The host ceiling is
    the same uploads and downloads with no render."""
    from cuda_rasterizer import _native as N
    dev = d.device
    n, s, V = args.n, args.samples, len(views)
    keys = ("means", "cov6", "sigma", "sh")
    h = {k: sc[k].cpu().pin_memory() for k in keys}
    dm = [{k: torch.empty_like(v, device=dev) for k, v in h.items()} for _ in range(2)]
    h_img = torch.empty((V, s, s), dtype=torch.float32).pin_memory()
    d_img = [torch.empty((V, s, s), dtype=torch.float32, device=dev) for _ in range(2)]
    group = GROUP_VIEWS
    ws = torch.empty(N.workspace_bytes(n, s, s, group), dtype=torch.uint8, device=dev)
    comp = torch.cuda.current_stream(dev)
    up = torch.cuda.Stream(dev)
    down = torch.cuda.Stream(dev)
    flush = torch.empty((512 << 20) // 4, dtype=torch.float32, device=dev)
    h2d = sum(v.numel() * 4 for v in h.values())
    d2h = V * s * s * 4

    def run(steps, render=True):
        """Enqueues `steps` pipelined steps; returns (start, end) events."""
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(comp)
        up.wait_event(start)
        down.wait_event(start)
        uploaded, rendered, copied = [], [], []
        for k in range(steps + 1):
            if k < steps:  # upload step k (buffer k % 2 is free once step k - 2 rendered)
                if k >= 2:
                    up.wait_event(rendered[k - 2])
                with torch.cuda.stream(up):
                    for key in keys:
                        dm[k % 2][key].copy_(h[key], non_blocking=True)
                e = torch.cuda.Event()
                e.record(up)
                uploaded.append(e)
            j = k - 1  # render step j while step k uploads
            if j < 0:
                continue
            comp.wait_event(uploaded[j])
            if j >= 2:
                comp.wait_event(copied[j - 2])  # images of step j - 2 are on the host
            if render:
                flush_l2(flush, j)
                inputs = N.prepare_inputs(dm[j % 2]["means"], dm[j % 2]["cov6"], dm[j % 2]["sigma"],
                                          dm[j % 2]["sh"])
            img = d_img[j % 2]
            for g0 in range(0, V, group):
                g1 = min(V, g0 + group)
                if render:
                    N.forward(views[g0:g1], *inputs, img[g0:g1], ws=ws)
                e = torch.cuda.Event()
                e.record(comp)
                down.wait_event(e)
                with torch.cuda.stream(down):
                    h_img[g0:g1].copy_(img[g0:g1], non_blocking=True)
            e = torch.cuda.Event()
            e.record(comp)
            rendered.append(e)
            e = torch.cuda.Event()
            e.record(down)
            copied.append(e)
        comp.wait_stream(down)
        comp.wait_stream(up)
        end.record(comp)
        return start, end

    steps = max(3, min(args.steps, 30))  # the pipeline fills once per timed region
    out = {}
    ok = False
    for render in (True, False):
        a, b = run(2, render)
        b.synchronize()
        d.barrier()
        a, b = run(steps, render)
        b.synchronize()
        t = a.elapsed_time(b)
        if render:
            ok = bool(torch.equal(h_img[V - 1].to(dev), d_img[(steps - 1) % 2][V - 1]))
        d.barrier()
        t_max = d.max(t)
        out[render] = (d.sum(float(V * steps)) / (t_max / 1e3), t_max / steps)
    value, ms = out[True]
    ceil_v, ceil_ms = out[False]
    return {"value": value, "unit": "views/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "steps": steps, "host_copy_verified": ok,
            "host_ceiling": {"value": ceil_v, "unit": "views/s", "ms_per_step": ceil_ms,
                             "what": "the same pinned uploads and image downloads on all ranks, "
                                     "no render", "frac": round(value / ceil_v, 4)},
            "pipeline": "step k+1 upload overlaps step k render; group images copied back "
                        "while the next group renders; one timed region over all steps"}


def bench_omega(args, d, inputs, views, flush):
    """render_sar's full contract (image and Omega) on one 256-view launch
    group per step: views/s, L2 flushed before every step."""
    from cuda_rasterizer import _native as N
    dev = d.device
    n, s = args.n, args.samples
    vs = views[:GROUP_VIEWS]
    V = len(vs)
    images = torch.empty((V, s, s), dtype=torch.float32, device=dev)
    omega = torch.empty((V, n), dtype=torch.float32, device=dev)
    ws = torch.empty(N.workspace_bytes(n, s, s, V, N.SARR_FLAG_OMEGA), dtype=torch.uint8, device=dev)
    steps = max(3, min(args.steps, 10))
    t = 0.0
    for k in range(steps + 2):
        flush_l2(flush, k)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        N.forward(vs, *inputs, images, omega=omega, ws=ws)
        b.record()
        b.synchronize()
        if k >= 2:
            t += a.elapsed_time(b)
    t_max = d.max(t)
    return {"value": d.sum(float(V * steps)) / (t_max / 1e3), "unit": "views/s",
            "ms_per_step": t_max / steps, "views_per_step": V,
            "outputs": "image [Nr, Na] and omega [N] per view (render_sar)"}


def bench_fwd_bwd(args, d, inputs, views, flush):
    """One view per step: forward keeping its state, backward reusing it,
    dense gradients for all N Gaussians (the SARRasterizer training path);
    L2 flushed before every step, each step timed by its own events."""
    from cuda_rasterizer import _native as N
    dev = d.device
    n, s = args.n, args.samples
    img = torch.empty((s, s), dtype=torch.float32, device=dev)
    g = torch.randn((s, s), generator=torch.Generator().manual_seed(1)).to(dev)
    state = torch.empty(N.state_bytes(n, s, s), dtype=torch.uint8, device=dev)
    ws = torch.empty(N.workspace_bytes(n, s, s, 1), dtype=torch.uint8, device=dev)
    gm = torch.empty((n, 3), device=dev)
    gc = torch.empty((n, 6), device=dev)
    gs = torch.empty((n,), device=dev)
    gsh = torch.empty((n, 16), device=dev)
    gn = torch.empty((n,), device=dev)

    def one(k):
        v = [views[k % len(views)]]
        N.forward(v, *inputs, img, states=state, ws=ws)
        N.backward(v, *inputs, g, gm, gc, N.SARR_COV6, gs, gsh, grad_norm=gn, states=state, ws=ws)

    for k in range(8):
        one(k)
    torch.cuda.synchronize()
    d.barrier()
    steps = 200
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for k in range(steps):
        flush_l2(flush, k)
        ev[k][0].record()
        one(k)
        ev[k][1].record()
    torch.cuda.synchronize()
    t = sum(a.elapsed_time(b) for a, b in ev)
    t_max = d.max(t)
    step_s = t_max / steps / 1e3
    b_fb = 312 * n + 8 * s * s
    return {"value": d.sum(float(steps)) / (t_max / 1e3), "unit": "steps/s", "ms_per_step": step_s * 1e3,
            "step": "1 view fwd+bwd, dense grads for 1M Gaussians, 256x256",
            "l2": "flushed before every step (512 MiB device write)",
            "roofline": roof(b_fb, step_s, {"bytes_per_step": b_fb,
                                             "model": "312 B/Gaussian + 8 B/pixel per view"})}


def _targets(N, views_t, n_target, box, scales, dev):
    """Target images of a separate seeded scene (seed 1) for these views."""
    tgt = S.make_scene(n_target, box, scales, seed=1, device=dev)
    vs = [N.make_view(*v) for v in views_t]
    nr, na = views_t[0][8], views_t[0][9]
    out = torch.empty((len(vs), nr, na), dtype=torch.float32, device=dev)
    N.forward(vs, *N.prepare_inputs(tgt["means"], tgt["cov6"], tgt["sigma"], tgt["sh"]), out)
    return out


def _time_trainer(tr, views, targets, steps, warmup, flush, d):
    from cuda_rasterizer import _native as N
    for k in range(warmup):
        tr.step(views, targets)
    torch.cuda.synchronize()
    d.barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    l0 = N.launch_count()
    for k in range(steps):
        flush_l2(flush, k)
        ev[k][0].record()
        tr.step(views, targets)
        ev[k][1].record()
    torch.cuda.synchronize()
    launches = N.launch_count() - l0
    return sum(a.elapsed_time(b) for a, b in ev), launches


def bench_train_step(args, d, flush):
    """The full-training shape, data-parallel: 1M Gaussians, 64 views per
    rank per step (256 x 256 at 0.2 m, azimuth uniform 0-360 deg, incidence
    15 or 17 deg), loss L1 + 0.2 D-SSIM against a seeded 200k-Gaussian target
    scene, Adam (lr 1e-3; SH lr 1e-5); the trainable gradients (80 B per
    Gaussian) summed over the ranks by 4 bucketed NCCL all-reduces, each
    followed by its bucket's Adam update."""
    from cuda_rasterizer import _native as N
    from cuda_rasterizer import multiview
    dev = d.device
    n, s = args.n, args.samples
    box, scales = (40.0, 40.0, 10.0), (0.05, 0.5)
    p = S.make_param_scene(n, box, scales, seed=0, device=dev)
    allv = S.training_views(TRAIN_VIEWS_PER_RANK * d.world, rho=0.2, samples=s)
    mine = allv[d.rank * TRAIN_VIEWS_PER_RANK:(d.rank + 1) * TRAIN_VIEWS_PER_RANK]
    targets = _targets(N, mine, 200_000, box, scales, dev)
    views = [N.make_view(*v) for v in mine]
    tr = multiview.ViewParallelTrainer(p["means"], p["scales"], p["rotations"], p["logits"], p["sh"],
                                       lr=1e-3, buckets=4)
    steps = max(3, min(args.steps, 20))
    t, launches = _time_trainer(tr, views, targets, steps, max(3, args.warmup), flush, d)
    t_max = d.max(t)
    step_ms = t_max / steps
    # the collective alone: the same four buckets, back to back
    ar_ms = 0.0
    if d.world > 1:
        for _ in range(3):
            tr.allreduce_only()
        torch.cuda.synchronize()
        d.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            tr.allreduce_only()
        b.record()
        b.synchronize()
        ar_ms = d.max(a.elapsed_time(b)) / steps
    loss = float(tr.losses[0].item())
    npix = s * s
    b_fb = 312 * n + 8 * npix * TRAIN_VIEWS_PER_RANK  # batched: parameters once per step
    return {"value": 1e3 / step_ms, "unit": "steps/s", "ms_per_step": step_ms,
            "views_per_s": d.world * TRAIN_VIEWS_PER_RANK * 1e3 / step_ms,
            "views_per_rank_per_step": TRAIN_VIEWS_PER_RANK,
            "global_views_per_step": TRAIN_VIEWS_PER_RANK * d.world, "scaling": "weak",
            "n_gaussians": n,
            "allreduce": {"bytes": int(tr.grad.numel() * 4), "buckets": len(tr.bounds),
                          "ms_alone": round(ar_ms, 4),
                          "share_of_step_alone": round(ar_ms / step_ms, 4) if d.world > 1 else 0.0},
            "loss_last_step": loss, "gpu_launches_per_step": launches / steps,
            "roofline": roof(b_fb, step_ms / 1e3,
                             {"model": "312 B/Gaussian per step + 8 B/pixel per view",
                              "bytes_per_step": b_fb}),
            "l2": "flushed before every step (512 MiB device write)",
            "step": "producer, forward (states kept), CombinedLoss(1.0, 0.2) + image gradient, "
                    "backward, sigmoid chain, bucketed NCCL all-reduce (N > 1), Adam"}


def bench_train_full(args, d, flush):
    """Full training with densification, on the schedule of SAR-3DGS's full
    training: 100k Gaussians (40 x 40 x 10 m, scales 0.05-0.5 m) trained
    against a seeded 200k-Gaussian target scene; 64 views per rank per step,
    in turn from a pool of 1,024 views per rank (256 x 256 at 0.2 m, azimuth
    uniform 0-360 deg, incidence 15 or 17 deg); L1 + 0.2 D-SSIM, Adam
    (lr 1e-3; SH lr 1e-5); densify and prune every 100 iterations with the
    reference's rules (clone: norm(scale) below the clone size and means
    gradient above 2e-4; split and prune: norm(scale) above 2 m; prune:
    transmittance below 0.005; cap 2M); SH degree 0 -> 3, one more every
    1,000 iterations; `--full-iters` iterations. The clone size is 1 m: the
    reference's default, 0.01 m, clones nothing among scales of 0.05-0.5 m
    (norms 0.12-0.38 m between the 1st and 50th percentiles), so the set
    would never grow. Each iteration is timed on the device (densifications
    included, L2 flushed between iterations), max over ranks; after 3
    warm-up iterations of a separate trainer."""
    from cuda_rasterizer import _native as N
    from cuda_rasterizer import multiview
    dev = d.device
    s = args.samples
    box, scales = (40.0, 40.0, 10.0), (0.05, 0.5)
    n0, pool, per = 100_000, 1024, TRAIN_VIEWS_PER_RANK
    p = S.make_param_scene(n0, box, scales, seed=0, device=dev)
    allv = S.training_views(pool * d.world, rho=0.2, samples=s)
    mine = allv[d.rank * pool:(d.rank + 1) * pool]
    targets = _targets(N, mine, 200_000, box, scales, dev)
    batches = [[N.make_view(*v) for v in mine[b:b + per]] for b in range(0, pool, per)]
    tbatches = [targets[b:b + per] for b in range(0, pool, per)]
    kw = dict(lr=1e-3, buckets=4, densify_interval=100, grad_threshold=2e-4, size_threshold=1.0,
              large_scale_threshold=2.0, opacity_threshold=0.005, max_gaussians=2_000_000,
              sh_interval=1000, max_sh_degree=3)
    warm = multiview.DensifyingTrainer(p["means"], p["scales"], p["rotations"], p["logits"], p["sh"],
                                       **kw)
    for k in range(3):
        warm.step(batches[k], tbatches[k])
    torch.cuda.synchronize()
    del warm
    dt = multiview.DensifyingTrainer(p["means"], p["scales"], p["rotations"], p["logits"], p["sh"], **kw)
    iters = args.full_iters
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(iters)]
    d.barrier()
    l0 = N.launch_count()
    loss_first = None
    for it in range(iters):
        k = it % len(batches)
        flush_l2(flush, it)
        ev[it][0].record()
        losses = dt.step(batches[k], tbatches[k])
        ev[it][1].record()
        if it == 0:
            loss_first = losses.clone()
    torch.cuda.synchronize()
    launches = N.launch_count() - l0
    t = [a.elapsed_time(b) for a, b in ev]
    total_ms = d.max(sum(t))
    # the loss is each rank's weighted share; the mean over all views is the sum
    loss_last = float(d.sum(float(losses[0].item())))
    loss_first = float(d.sum(float(loss_first[0].item())))
    hist = [list(h) for h in dt.history]
    return {"value": iters * 1e3 / total_ms, "unit": "steps/s", "iterations": iters,
            "total_s": round(total_ms / 1e3, 3), "ms_per_step": total_ms / iters,
            "views_per_rank_per_step": per, "global_views_per_step": per * d.world,
            "scaling": "weak", "n_start": n0, "n_final": dt.n,
            "densify": {"interval": 100, "grad_threshold": 2e-4, "clone_size_m": 1.0,
                        "split_prune_size_m": 2.0, "prune_transmittance": 0.005,
                        "max_gaussians": 2_000_000},
            "densifications": hist,
            "densification_fields": ["iteration", "n_before", "clones", "splits", "prunes", "n_after"],
            "sh_degree_final": multiview.sh_degree_at(iters - 1, 1000, 3),
            "loss_first_step": loss_first, "loss_last_step": loss_last,
            "gpu_launches_per_step": launches / iters,
            "l2": "flushed between iterations (512 MiB device write, outside the timed region)",
            "step": "DensifyingTrainer: producer, forward, CombinedLoss, backward, bucketed NCCL "
                    "all-reduce (N > 1), Adam; densify/prune from the summed gradient every 100 "
                    "iterations (no update that iteration, Adam state cleared, as the reference)"}


def bench_train_configs(args, d, flush):
    """The training step on one GPU on the two smaller training scenes:
    50k Gaussians in 20 x 20 x 6 m, 64 views of 128 x 128 at 0.3 m (targets
    from a separate 20k scene); 500k Gaussians in 60 x 60 x 15 m with scales
    0.02-0.3 m, 16 views of 512 x 512 at 0.1 m, incidence 15-45 deg (targets
    from a separate 100k scene)."""
    from cuda_rasterizer import _native as N
    from cuda_rasterizer import multiview
    dev = d.device
    out = {}
    cfgs = (("train_n50000_128px_64views", 50_000, (20.0, 20.0, 6.0), (0.05, 0.5), 20_000,
             S.training_views(64)),
            ("hires_n500000_512px_16views", 500_000, (60.0, 60.0, 15.0), (0.02, 0.3), 100_000,
             S.hires_views(16)))
    for name, n, box, scales, n_tgt, views_t in cfgs:
        p = S.make_param_scene(n, box, scales, seed=0, device=dev)
        targets = _targets(N, views_t, n_tgt, box, scales, dev)
        views = [N.make_view(*v) for v in views_t]
        tr = multiview.ViewParallelTrainer(p["means"], p["scales"], p["rotations"], p["logits"],
                                           p["sh"], lr=1e-3, buckets=4, distributed=False)
        steps = max(5, min(args.steps, 20))
        t, launches = _time_trainer(tr, views, targets, steps, max(3, args.warmup), flush, d)
        step_ms = t / steps
        npix = views_t[0][8] * views_t[0][9]
        b_fb = 312 * n + 8 * npix * len(views)  # batched: parameters once per step
        out[name] = {"value": 1e3 / step_ms, "unit": "steps/s", "ms_per_step": step_ms,
                     "views_per_step": len(views), "views_per_s": len(views) * 1e3 / step_ms,
                     "gpu_launches_per_step": launches / steps,
                     "roofline": roof(b_fb, step_ms / 1e3, {
                         "bytes_per_step": b_fb,
                         "model": "312 B/Gaussian per step + 8 B/pixel per view"}),
                     "loss_last_step": float(tr.losses[0].item())}
        del tr, p, targets
    return out


def bench_train_ops(args, d):
    """The training-step kernels next to the rasterizer: the Gaussian
    parameter producer over the N Gaussians (72 B per Gaussian: log-scales,
    quaternion and logit read, 3x3 covariance and transmittance written), the
    combined L1 + D-SSIM loss with its gradient over 64 images of the sweep
    size (12 B per pixel: both images read, the gradient written), one
    densify/prune pass over the N Gaussians, and Adam over the 20 trainable
    floats per Gaussian."""
    from cuda_rasterizer import _native as N
    dev = d.device
    n, s = args.n, args.samples
    g = torch.Generator(device=dev).manual_seed(3)
    scales = torch.rand((n, 3), device=dev, generator=g) * 3 - 4
    rot = torch.randn((n, 4), device=dev, generator=g)
    logits = torch.randn((n,), device=dev, generator=g)
    pred = torch.rand((64, s, s), device=dev, generator=g)
    target = torch.rand((64, s, s), device=dev, generator=g)
    peak, peak_kind = peaks()

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b) / reps / 1e3

    t_p = timed(lambda: N.gaussian_params(scales, rot, logits))
    t_l = timed(lambda: N.combined_loss(pred, target, 0.9, 0.1, 5, "plain"))
    bp, bl = 72 * n, 12 * 64 * s * s
    from cuda_rasterizer import densify as DZ
    dm = (torch.rand((n, 3), device=dev, generator=g) - 0.5) * 40
    ds = torch.rand((n, 3), device=dev, generator=g) * 8.0 - 6.5
    dq = torch.randn((n, 4), device=dev, generator=g)
    do = torch.randn((n, 1), device=dev, generator=g) * 2.5
    dsh = torch.randn((n, 16), device=dev, generator=g) * 0.1
    dgr = torch.randn((n, 3), device=dev, generator=g) * 1e-4
    dargs = (1e-4, 0.01, 2.0, 0.05, 10_000_000)
    out, counts = DZ.densify_and_prune_tensors(dm, ds, dq, do, dsh, dgr, *dargs)
    t_d = timed(lambda: DZ.densify_and_prune_tensors(dm, ds, dq, do, dsh, dgr, *dargs), reps=10)
    n_out = int(out[0].shape[0])
    bd = n * (12 + 12 + 16 + 4 + 64 + 12) + n_out * (12 + 12 + 16 + 4 + 64)
    flat = torch.randn(20 * n, device=dev, generator=g)
    grad = torch.randn(20 * n, device=dev, generator=g)
    m, v = torch.zeros_like(flat), torch.zeros_like(flat)
    t_a = timed(lambda: N.adam_step(flat, grad, m, v, [(20 * n, 1e-3)], 1))
    ba = 20 * n * (16 + 12)
    return {"producer": {"gaussians_per_s": n / t_p, "achieved_gbs": round(bp / t_p / 1e9, 1),
                         "frac": round(bp / t_p / 1e9 / peak, 4), "peak_source": peak_kind,
                         "us": round(t_p * 1e6, 2)},
            "loss": {"images_per_s": 64 / t_l, "achieved_gbs": round(bl / t_l / 1e9, 1),
                     "frac": round(bl / t_l / 1e9 / peak, 4), "us_per_64": round(t_l * 1e6, 2)},
            "densify": {"gaussians_per_s": n / t_d, "us": round(t_d * 1e6, 2), "n_out": n_out,
                        "counts": [int(c) for c in counts],
                        "achieved_gbs": round(bd / t_d / 1e9, 1), "frac": round(bd / t_d / 1e9 / peak, 4),
                        "bytes": "120 B read per Gaussian, 108 B written per output Gaussian; "
                                 "includes the host reading the three counts"},
            "adam": {"us": round(t_a * 1e6, 2), "achieved_gbs": round(ba / t_a / 1e9, 1),
                     "frac": round(ba / t_a / 1e9 / peak, 4),
                     "bytes": "20 floats per Gaussian: param, grad, m, v read; param, m, v written"}}


def _cpu_scene(args):
    sc = make_scene(args, "cpu")
    return {k: v.numpy() for k, v in sc.items()}


def cpu_fwd_bwd_sample(O, s, views, budget_s):
    """Oracle forward + backward of single views (the reference's
    render_sar_backward recomputes the forward, .cu:1495-1559) until the
    budget is used: (steps, seconds)."""
    g = np.random.default_rng(1).standard_normal(views[0][8] * views[0][9]).astype(np.float32)
    done, t0 = 0, time.perf_counter()
    while done < 16:
        O.backward_full(O.make_view(*views[done]), s["means"], s["cov6"], s["sigma"], s["sh"], g)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return done, time.perf_counter() - t0


def cpu_baseline(args):
    """CPU restatement of the reference algorithm on a bounded sample of the
    same workloads, all host threads: image-only forward views/s (the
    headline) and forward + backward steps/s (one view per step)."""
    from oracle import oracle as O
    cores = O.set_threads()
    s = _cpu_scene(args)
    views = S.sweep_views(args.views, samples=args.samples)
    done, t0 = 0, time.perf_counter()
    while done < 64:
        O.forward(O.make_view(*views[done]), s["means"], s["cov6"], s["sigma"], s["sh"],
                  want_omega=False)
        done += 1
        if time.perf_counter() - t0 > 12.0:
            break
    dt = time.perf_counter() - t0
    nb, tb = cpu_fwd_bwd_sample(O, s, views, 8.0)
    return {"value": done / dt, "unit": "views/s", "cores": cores, "kind": "port",
            "sample": f"{done} views of the sweep (N={args.n}, {args.samples}x{args.samples}), "
                      "image-only forward, C restatement with OpenMP",
            "fwd_bwd": {"value": nb / tb, "unit": "steps/s", "cores": cores, "kind": "port",
                        "sample": f"{nb} single-view forward + backward steps at N={args.n}"}}


def bench_reference(args, d):
    """Reference arm: the CPU restatement on the host cores (rank 0 only), K
    steps of a bounded 2-view sample; forward + backward steps/s of a bounded
    sample; plus the reference's own CUDA kernels on two views when its
    harness and a GPU are available."""
    if d.rank != 0:
        return None
    from oracle import oracle as O
    cores = O.set_threads()
    s = _cpu_scene(args)
    views = S.sweep_views(args.views, samples=args.samples)
    per_step = 2
    for k in range(args.warmup):
        O.forward(O.make_view(*views[k % len(views)]), s["means"], s["cov6"], s["sigma"], s["sh"],
                  want_omega=False)
    t0 = time.perf_counter()
    for k in range(args.steps):
        for j in range(per_step):
            O.forward(O.make_view(*views[(k * per_step + j) % len(views)]), s["means"], s["cov6"],
                      s["sigma"], s["sh"], want_omega=False)
    dt = time.perf_counter() - t0
    value = args.steps * per_step / dt
    nb, tb = cpu_fwd_bwd_sample(O, s, views, 8.0)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "views/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": config(args),
            "cpu_baseline": {"value": value, "unit": "views/s", "cores": cores,
                             "kind": "port",
                             "sample": f"{per_step} views per step of the sweep, image-only forward"},
            "e2e": {"value": value, "unit": "views/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "fwd_bwd": {"value": nb / tb, "unit": "steps/s", "cores": cores, "kind": "port",
                        "sample": f"{nb} single-view forward + backward steps at N={args.n}"}}
    try:
        line["gpu_reference"] = gpu_reference(args, s, views)
    except Exception as e:  # reported, not fatal: the CPU arm above is the reference arm
        line["gpu_reference"] = {"unavailable": f"{type(e).__name__}: {e}"}
    return line


def gpu_reference(args, s, views):
    from oracle.ref import build_ref
    R = build_ref.load_module()
    dev = torch.device("cuda", 0)
    t = {k: torch.from_numpy(s[k]).to(dev).contiguous() for k in ("means", "cov6", "sigma", "sh")}
    R.render_sar(t["means"], t["cov6"], t["sigma"], t["sh"], *views[0], False, False)
    torch.cuda.synchronize()
    nv = 2
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for j in range(nv):
        R.render_sar(t["means"], t["cov6"], t["sigma"], t["sh"], *views[1 + j], False, False)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b)
    g = torch.randn((views[0][8], views[0][9]), generator=torch.Generator().manual_seed(1)).to(dev)
    R.render_sar_backward(t["means"], t["cov6"], t["sigma"], t["sh"], g, *views[0])
    torch.cuda.synchronize()
    a.record()
    for j in range(nv):
        R.render_sar(t["means"], t["cov6"], t["sigma"], t["sh"], *views[1 + j], False, False)
        R.render_sar_backward(t["means"], t["cov6"], t["sigma"], t["sh"], g, *views[1 + j])
    b.record()
    b.synchronize()
    ms_fb = a.elapsed_time(b)
    return {"value": nv / (ms / 1e3), "unit": "views/s", "kind": "reference",
            "fwd_bwd": {"value": nv / (ms_fb / 1e3), "unit": "steps/s"},
            "sample": f"{nv} views, reference rasterizer_impl_v2.cu kernels (slot-indexing fix), "
                      "render_sar incl. its per-call allocations and Omega host round trip; "
                      "fwd_bwd: render_sar then render_sar_backward per view"}


def config(args):
    return {"workload": f"sar_sweep_n{args.n}_{args.samples}px_{args.views}views",
            "n_gaussians": args.n, "image": [args.samples, args.samples], "rho_m": 0.2,
            "views_per_step_per_gpu": args.views, "scene_box_m": [40, 40, 10],
            "l2": "flushed before every timed step (512 MiB device write)",
            "parallelism": f"view-sharded x{args.gpus}, no data-path collective in the forward",
            "outputs": "images only (the SARRasterizer forward contract); omega: with Omega"}


def main():
    args = parse()
    if args.impl == "reference":
        d = Dist() if int(os.environ.get("WORLD_SIZE", "1")) > 1 else None
        rank = d.rank if d else 0
        line = bench_reference(args, d or type("D", (), {"rank": 0})())
        if rank == 0 and line:
            print(json.dumps(line))
        if d:
            d.close()
        return
    d = Dist()
    if not wanted(args, "forward"):
        # a profiling run of some sections only (no headline value)
        flush = torch.empty((512 << 20) // 4, dtype=torch.float32, device=d.device)
        line = {"metric": METRIC, "sections": args.sections, "n_gpus": d.world}
        if wanted(args, "train_step"):
            line["train_step"] = bench_train_step(args, d, flush)
        if wanted(args, "train_full"):
            line["train_full"] = bench_train_full(args, d, flush)
        if wanted(args, "train_configs") and d.world == 1:
            line["train_configs"] = bench_train_configs(args, d, flush)
        if d.rank == 0:
            print(json.dumps(line))
        d.close()
        return
    r = bench_forward(args, d)
    line = {"metric": METRIC, "value": r["value"], "unit": "views/s", "n_gpus": d.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; the sweep's scene and view distributions)", "config": config(args),
            "roofline": r["roofline"], "gpu_launches": r["launches"], "clocks": r["clocks"],
            "path_roofline": r["path_roofline"], "render_issue": r["render_issue"],
            "kernels": r["kernels"], "image_checksum": r["checksum"][0],
            "image_sha1": r["checksum"][1], "image_checksum_stable": r["checksum_stable"]}
    if not args.no_e2e and wanted(args, "e2e"):
        line["e2e"] = bench_e2e(args, d, r["sc"], r["views"])
    if wanted(args, "omega"):
        line["omega"] = bench_omega(args, d, r["inputs"], r["views"], r["flush"])
    if not args.no_train:
        if wanted(args, "fwd_bwd"):
            line["fwd_bwd"] = bench_fwd_bwd(args, d, r["inputs"], r["views"], r["flush"])
        flush = r["flush"]
        del r
        if wanted(args, "train_step"):
            line["train_step"] = bench_train_step(args, d, flush)
        if wanted(args, "train_full"):
            line["train_full"] = bench_train_full(args, d, flush)
        if d.world == 1:
            if wanted(args, "train_configs"):
                line["train_configs"] = bench_train_configs(args, d, flush)
            if wanted(args, "train_ops"):
                line["train_ops"] = bench_train_ops(args, d)
    if d.rank == 0 and d.world == 1 and not args.no_cpu and wanted(args, "cpu"):
        line["cpu_baseline"] = cpu_baseline(args)
    if d.rank == 0:
        print(json.dumps(line))
    d.close()


if __name__ == "__main__":
    main()
