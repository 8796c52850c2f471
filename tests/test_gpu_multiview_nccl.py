"""View data-parallel training step on 2 GPUs over NCCL: each rank renders and
differentiates its shard of the views, the bucketed all-reduce sums the
trainable gradients, and every rank ends with the gradients of one process's
backward over all views (equal up to float summation order). The training
step (ViewParallelTrainer: bucketed all-reduce overlapped with Adam) leaves
identical parameters on both ranks, equal to one process's training on all
views; full training with densification (DensifyingTrainer) leaves the same
Gaussian set and parameters on both ranks. Skipped with fewer than 2 visible
GPUs."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rel(a, b):
    scale = float(b.abs().max())
    return float((a - b).abs().max()) / scale if scale > 0 else float((a - b).abs().max())


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from cuda_rasterizer import _native
        from cuda_rasterizer import cuda_rasterizer_sar as M
        from cuda_rasterizer import multiview
        from cuda_rasterizer import synthetic as S
        sc = {k: v.to(dev) for k, v in
              S.make_scene(90000, (30.0, 30.0, 8.0), (0.05, 0.5), seed=71).items()}
        views = S.sweep_views(96)[::8]  # 12 views
        args = (sc["means"], sc["cov6"], sc["sigma"], sc["sh"])
        images = M.render_sar_batched(*args, views)
        g = torch.Generator().manual_seed(72)
        gimg = torch.randn(tuple(images.shape), generator=g).to(dev)
        a, b = multiview.shard_range(len(views), rank, world)
        mine = multiview.render_views(*args, views[a:b])
        same_images = bool(torch.equal(mine, images[a:b]))
        gm, gc, gs, gsh, gn = multiview.backward_views(*args, gimg[a:b], views[a:b])
        fm, fc, fs, fsh, fn = M.render_sar_backward_batched(*args, gimg, views, grad_sh_cols=16,
                                                            grad_norm=True)
        torch.cuda.synchronize()
        errs = [_rel(gm, fm), _rel(gs, fs), _rel(gsh, fsh), _rel(gn, fn)]
        # the training step: each rank trains on its shard. After one step the
        # summed gradients equal those of one process training on all views
        # (up to float summation order), and so do the Adam updates wherever
        # the gradient is well above the rounding noise; after a second step
        # the parameters are still identical on both ranks.
        gp = torch.Generator().manual_seed(73)
        n = sc["means"].shape[0]
        scales = (torch.rand((n, 3), generator=gp) * 2.3 - 3.0).to(dev)
        rot = torch.randn((n, 4), generator=gp).to(dev)
        logits = torch.randn((n,), generator=gp).to(dev)
        vs = [_native.make_view(*v) for v in views]
        tr = multiview.ViewParallelTrainer(sc["means"], scales, rot, logits, sc["sh"], buckets=3)
        one = multiview.ViewParallelTrainer(sc["means"], scales, rot, logits, sc["sh"], buckets=3,
                                            distributed=False)
        p0 = one.param.clone()
        targets = images.flip(0).contiguous()
        tr.step(vs[a:b], targets[a:b])
        one.step(vs, targets)
        torch.cuda.synchronize()
        g_tr = torch.cat([x.reshape(-1) for x in tr.gradients()])
        g_one = torch.cat([x.reshape(-1) for x in one.gradients()])
        errs.append(_rel(g_tr, g_one))
        big = g_one.abs() > 1e-3 * g_one.abs().max()  # the parameter layout, as tr.param
        errs.append(_rel((tr.param - p0)[big], (one.param - p0)[big]))
        tr.step(vs[a:b], targets[a:b])
        torch.cuda.synchronize()
        other = tr.param.clone()
        dist.broadcast(other, src=0)
        same_params = bool(torch.equal(other, tr.param))
        # full training with densification (iterations 2 and 4): every rank
        # densifies from the same summed gradient, so the sets stay identical
        dt = multiview.DensifyingTrainer(sc["means"], scales, rot, logits, sc["sh"], buckets=3,
                                         densify_interval=2, grad_threshold=1e-7, size_threshold=1.0,
                                         sh_interval=2)
        for _ in range(5):
            dt.step(vs[a:b], targets[a:b])
        torch.cuda.synchronize()
        n_t = torch.tensor([dt.n], device=dev)
        n_0 = n_t.clone()
        dist.broadcast(n_0, src=0)
        same_dense = bool(torch.equal(n_0, n_t)) and len(dt.history) == 2 and dt.n != n
        if same_dense:
            for t in (dt.tr.param, dt.tr.scales, dt.tr.rotations):
                o = t.clone()
                dist.broadcast(o, src=0)
                same_dense = same_dense and bool(torch.equal(o, t))
        q.put((rank, same_images and same_params and same_dense, errs))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def test_view_parallel_backward_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=300) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
    for rank, same, errs in results:
        assert same is True, (rank, same, errs)
        assert max(errs[:5]) <= 1e-5, (rank, errs)
        assert errs[5] <= 1e-4, (rank, errs)  # the first Adam update
