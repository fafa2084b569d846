"""The NVLink peer-memory gradient sum (PeerGradAllReduce over
gsb_peer_allreduce_sum) against the same sum computed on the CPU.

Each rank fills the .grad of a few shared parameters from seeds every rank
knows, so every rank can compute the expected sum itself. The sum is taken in
rank order on both sides, so the comparison is exact. The multi-rank case runs
one process per GPU and is skipped with fewer than two GPUs; the one-rank case
(no kernel, the buffer is its own sum) runs anywhere with a GPU.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(1000, 3), (1000, 4), (1000,), (1001, 3), (300_001,)]  # odd total: the buffer pads to 4 floats


def _grads(step: int, rank: int):
    return [torch.randn(s, generator=torch.Generator().manual_seed(1000 * step + 10 * rank + i))
            for i, s in enumerate(SHAPES)]


def _expected(step: int, world: int):
    per_rank = [_grads(step, r) for r in range(world)]
    out = []
    for i in range(len(SHAPES)):
        acc = per_rank[0][i].clone()
        for r in range(1, world):
            acc = acc + per_rank[r][i]
        out.append(acc)
    return out


def _worker(rank: int, world: int, port: int, q, views: bool = True) -> None:
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "fast-mac-gsplat_b200")]
        from torch_gsplat_bridge_fast.distributed import PeerGradAllReduce

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        dev = torch.device("cuda", rank)
        params = [torch.zeros(s, device=dev, requires_grad=True) for s in SHAPES]
        red = PeerGradAllReduce(params, grads_as_views=views)
        worst = 0.0
        for step in range(3):
            for p, g in zip(params, _grads(step, rank)):
                p.grad = g.to(dev)
            red()
            for p, want in zip(params, _expected(step, world)):
                worst = max(worst, float((p.grad.cpu() - want).abs().max()))
        red.check_errors()
        red.close()
        dist.destroy_process_group()
        q.put((rank, worst, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, views: bool = True) -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, views)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in range(world):
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, worst, err in sorted(results, key=lambda r: r[0]):
        assert err is None, f"rank {rank}: {err}"
        assert worst == 0.0, f"rank {rank}: max abs error {worst}"


def test_peer_allreduce_one_rank_leaves_the_buffer():
    _run(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("views", [True, False])
def test_peer_allreduce_two_ranks_matches_cpu_sum(views):
    _run(2, views)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs four GPUs")
def test_peer_allreduce_four_ranks_matches_cpu_sum():
    _run(4)


class _RawInt32:
    """A raw device allocation seen by torch.as_tensor as int32 (no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False), "version": 3,
                                         "strides": None}


@pytest.mark.parametrize("case", ["timeout", "poisoned", "ahead"])
def test_peer_allreduce_gives_up_and_reports(case):
    """Failure detection without a GPU fault: rank 0 of a 2-rank sum whose
    second buffer (on the same GPU) belongs to a rank that never launches, so
    only this one kernel waits and no two waiting kernels share the GPU.

    timeout:  the peer's flags are never set; the start barrier's bounded wait
              (1 s here) runs out.
    poisoned: the peer has marked an abort of this epoch in rank 0's buffer
              (it gave up the call); rank 0 must give up at once.
    ahead:    the peer's start slot already holds a later epoch (it left this
              call without rank 0); rank 0 must give up at once.
    In every case the kernel records GSB_DEVERR_PEER_TIMEOUT at the start
    barrier, marks its own abort in both buffers, leaves the data untouched and
    returns; the context stays usable."""
    import ctypes as C
    import time

    from torch_gsplat_bridge_fast import _native as N

    L = N.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n, epoch = 4096, 5
    bases = []
    for _ in range(2):
        b = C.c_void_p()
        N.check(L.gsb_peer_buffer_alloc(n * 4, C.byref(b)), "gsb_peer_buffer_alloc")
        bases.append(b.value)
    try:
        flags = [torch.as_tensor(_RawInt32(b, N.GSB_PEER_FLAG_BYTES // 4), device=dev) for b in bases]
        data = [torch.as_tensor(_RawInt32(b + N.GSB_PEER_FLAG_BYTES, n), device=dev).view(torch.float32)
                for b in bases]
        for r, d in enumerate(data):
            d.copy_(torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * r)
        if case == "poisoned":
            flags[0][16 + 1] = epoch  # rank 1's abort slot in rank 0's buffer
        elif case == "ahead":
            flags[0][0 + 1] = epoch + 1  # rank 1's start slot in rank 0's buffer
        torch.cuda.synchronize()
        status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=dev)
        arr = (C.c_void_p * 2)(*bases)
        wait_ns = 1_000_000_000 if case == "timeout" else 4_000_000_000
        t0 = time.perf_counter()
        N.check(L.gsb_peer_allreduce_sum(0, 2, arr, n, epoch, wait_ns, N.ptr(status), N.stream_ptr(dev)),
                "gsb_peer_allreduce_sum")
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        err = int(status[N.GSB_STATUS_ERROR].item())
        assert err & N.GSB_DEVERR_PEER_TIMEOUT, err
        assert int(status[N.GSB_STATUS_ERROR_SITE].item()) == 7  # the start barrier
        if case == "timeout":
            assert 0.9 < waited < 30.0, waited
        else:
            assert waited < 2.0, waited  # no wait for the 4 s limit
        for f in flags:  # rank 0's abort mark for this epoch, in both buffers
            assert int(f[16 + 0].item()) == epoch
        assert int(flags[0][32].item()) == 0 and int(flags[0][33].item()) == 0  # counter and failure word reset
        for r, d in enumerate(data):
            assert torch.equal(d, torch.arange(n, device=dev, dtype=torch.float32) + 1000.0 * r)
        assert "peer rank" in N.decode_device_error(err, 7)
        x = torch.arange(10, device=dev, dtype=torch.float32)
        assert float(x.sum().item()) == 45.0  # the context is still usable
    finally:
        for b in bases:
            L.gsb_peer_buffer_free(C.c_void_p(b))
