"""Host logic of view data-parallelism on 2 CPU ranks (gloo): sharding covers
every view once, and the bucketed gradient all-reduce sums exactly; a rank
that raises is reported to the launcher instead of hanging the others."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cuda_rasterizer import multiview


def test_shard_range_partitions():
    for n in (0, 1, 7, 64, 1024, 1025):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                a, b = multiview.shard_range(n, r, world)
                seen.extend(range(a, b))
                assert b - a in (n // world, n // world + 1)
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        multiview.shard_range(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        g = torch.Generator().manual_seed(rank)
        grads = [torch.randn(1000, 3, generator=g), torch.randn(1000, generator=g),
                 torch.randn(1000, 16, generator=g)]
        expect = []
        for r in range(world):
            gr = torch.Generator().manual_seed(r)
            expect.append([torch.randn(1000, 3, generator=gr), torch.randn(1000, generator=gr),
                           torch.randn(1000, 16, generator=gr)])
        total = [sum(e[i] for e in expect) for i in range(3)]
        multiview.allreduce_gradients(grads, bucket_bytes=30_000)  # forces several buckets
        ok = all(torch.allclose(a, b, atol=1e-6) for a, b in zip(grads, total))
        views = list(range(10))
        mine = multiview.shard_views(views, rank, world)
        q.put((rank, ok, mine))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", str(e)))
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(results, key=lambda x: x[0])


def test_densify_schedule_and_sh_ramp():
    """The full-training schedule: densification on multiples of the
    interval past the start while the set is below the cap; the SH degree
    one higher every interval up to the maximum."""
    due = [i for i in range(0, 501) if multiview.densify_due(i, 1000, 100, 0, 2_000_000)]
    assert due == [100, 200, 300, 400, 500]
    assert not multiview.densify_due(200, 2_000_000, 100, 0, 2_000_000)
    assert [i for i in range(0, 301) if multiview.densify_due(i, 10, 100, 100, 50)] == [200, 300]
    degs = [multiview.sh_degree_at(i, 1000, 3) for i in (0, 999, 1000, 2500, 3000, 9000)]
    assert degs == [0, 0, 1, 2, 3, 3]


def test_allreduce_and_sharding_two_ranks():
    res = _run(2)
    assert [r[1] for r in res] == [True, True]
    assert res[0][2] + res[1][2] == list(range(10))


def test_failing_rank_is_reported():
    res = _run(2, fail_rank=1)
    assert res[1][1] == "error" and "injected" in res[1][2]
    # the surviving rank's collective ends with an error (peer gone or the
    # 20 s process-group timeout) instead of hanging
    assert res[0][1] == "error"


def test_bucket_bounds_and_segments():
    for total in (1, 63, 64, 65, 1000, 20 * 12345):
        for buckets in (1, 3, 4, 8):
            b = multiview.bucket_bounds(total, buckets)
            assert len(b) <= buckets and b[0][0] == 0 and b[-1][1] == total
            assert all(x[1] == y[0] for x, y in zip(b, b[1:]))
            assert all(a % 64 == 0 for a, _ in b)
    assert multiview.bucket_bounds(0, 4) == []
    # the parts of each bucket of Gaussians in the flat means | logits | SH
    # layout cover every element once, each with its group
    n, k = 1000, 16
    owner = [None] * (n * (4 + k))
    for g0, g1 in multiview.bucket_bounds(n, 3, align=256):
        for a, b, grp in multiview.flat_segments(n, k, g0, g1):
            for e in range(a, b):
                assert owner[e] is None
                owner[e] = grp
    assert owner == [0] * (3 * n) + [1] * n + [2] * (k * n)
