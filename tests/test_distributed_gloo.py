"""Multi-rank host logic on CPU with gloo (world size 2): view sharding and the
shared-Gaussian gradient all-reduce reproduce the single-process result. The
per-rank renderer here is the CPU torch oracle (no GPU in these tests)."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene():
    g = torch.Generator().manual_seed(0)
    G, V, H, W = 40, 3, 24, 32
    m3 = torch.randn(G, 3, generator=g) * torch.tensor([1.0, 0.7, 0.3]) + torch.tensor([0.0, 0.0, 4.0])
    s3 = torch.exp(torch.randn(G, 3, generator=g) * 0.3 - 1.5)
    q4 = torch.randn(G, 4, generator=g)
    q4 = q4 / q4.norm(dim=-1, keepdim=True)
    op = torch.sigmoid(torch.randn(G, generator=g))
    col = torch.rand(G, 3, generator=g)
    c2w = torch.eye(4).repeat(V, 1, 1)
    c2w[:, 0, 3] = torch.tensor([-0.3, 0.0, 0.3])
    cam = torch.tensor([[40.0, 40.0, W / 2, H / 2]] * V)
    gimg = torch.randn(V, H, W, 3, generator=g)
    return (m3, s3, q4, op, col), c2w, cam, gimg, (H, W)


def _local_grads(params, c2w, cam, gimg, hw, views):
    from oracle import torch_ref as TR

    H, W = hw
    ps = [p.clone().requires_grad_(True) for p in params]
    m3, s3, q4, op, col = ps
    for v in views:
        m2, con, po, dep = TR.project_pinhole(m3[None], s3[None], q4[None], op[None], c2w[v:v + 1], cam[v:v + 1],
                                              1e-4)
        img = TR.saturating_reference(m2, con, col[None], po, dep, H, W)
        img.backward(gimg[v:v + 1])
    return ps


def _worker(rank, world, port, out_q):
    sys.path[:0] = [str(ROOT), str(ROOT / "fast-mac-gsplat_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    from torch_gsplat_bridge_fast.distributed import SharedGradAllReduce, shard_views

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        params, c2w, cam, gimg, hw = _scene()
        views = shard_views(c2w.shape[0], world, rank)
        ps = _local_grads(params, c2w, cam, gimg, hw, views)
        sync = SharedGradAllReduce(ps, bucket_bytes=256)  # several small buckets
        sync()
        out_q.put((rank, views, [p.grad.clone() for p in ps]))
    finally:
        dist.destroy_process_group()


def test_shard_views_round_robin():
    from torch_gsplat_bridge_fast.distributed import shard_views

    assert shard_views(8, 8, 3) == [3]
    assert shard_views(4, 2, 1) == [1, 3]
    assert sorted(sum((shard_views(10, 4, r) for r in range(4)), [])) == list(range(10))
    with pytest.raises(ValueError):
        shard_views(4, 2, 2)


def test_shared_gradient_allreduce_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    params, c2w, cam, gimg, hw = _scene()
    ref = _local_grads(params, c2w, cam, gimg, hw, range(c2w.shape[0]))
    assert sorted(v for _, views, _ in results for v in views) == [0, 1, 2]
    for _, _, grads in results:
        for g, r in zip(grads, ref):
            assert torch.allclose(g, r.grad, rtol=1e-5, atol=1e-6)


def _silent_worker(rank, world, port, out_q):
    """Rank 1 joins the group and then never takes part in the all-reduce (a
    rank that hangs); rank 0 must get an error from the process group's
    timeout instead of waiting for ever."""
    sys.path[:0] = [str(ROOT), str(ROOT / "fast-mac-gsplat_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import time

    from torch_gsplat_bridge_fast.distributed import SharedGradAllReduce

    # The rendezvous may wait for a slow peer start; only the all-reduce's group
    # has the short timeout under test.
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    group = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=4))
    err = None
    t0 = time.perf_counter()
    try:
        if rank == 0:
            p = torch.zeros(64, requires_grad=True)
            p.grad = torch.ones(64)
            try:
                SharedGradAllReduce([p], group=group)()
            except Exception as e:  # the expected outcome
                err = type(e).__name__
        else:
            time.sleep(12)
    finally:
        out_q.put((rank, err, time.perf_counter() - t0))
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_that_never_joins_the_allreduce_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_silent_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = {r: (err, t) for r, err, t in (q.get(timeout=120) for _ in procs)}
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    err, waited = results[0]
    assert err is not None, "rank 0 returned from an all-reduce its peer never joined"
    assert waited < 30.0, waited
