"""Multi-GPU plumbing for the rasterizer: one process per GPU.

The reference is single-device (it chunks the view batch serially,
variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:910-938). Here:

* Independent views (a [B,G,...] batch of 2D splats, or several cameras of one 3D
  scene) are sharded round-robin over ranks. Each rank renders and
  differentiates its own views; there is no collective on the data path
  (weak scaling).
* Shared 3D Gaussians (every rank renders a different camera of the same
  scene): the per-Gaussian gradients of the shared parameters are summed
  across ranks. `PeerGradAllReduce` does it with this library's own kernel
  over NVLink peer memory (gsb_peer_allreduce_sum: CUDA IPC buffers, a
  two-shot reduce in one kernel per rank). `SharedGradAllReduce` does it with
  NCCL all-reduce (sum, fp32) in buckets, asynchronously; it is the baseline,
  and the one that runs on CPU tensors with the gloo backend (tests).
"""
from __future__ import annotations

import ctypes as C
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def shard_views(num_views: int, world_size: int, rank: int) -> List[int]:
    """Round-robin assignment of view indices to a rank."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("invalid world_size/rank")
    return list(range(rank, num_views, world_size))


class _FlatGrads:
    """The .grad of the shared parameters packed into one flat fp32 buffer."""

    def _init_flat(self, params: Sequence[torch.Tensor], flat: Optional[torch.Tensor] = None) -> None:
        if not params:
            raise ValueError("no parameters")
        self.params = list(params)
        self.numels = [p.numel() for p in self.params]
        self.total = sum(self.numels)
        dev = self.params[0].device
        self.flat = flat if flat is not None else torch.zeros(self.total, dtype=torch.float32, device=dev)

    def _pack(self) -> None:
        off = 0
        for p, n in zip(self.params, self.numels):
            seg = self.flat[off:off + n]
            if p.grad is None:
                seg.zero_()
            else:
                seg.copy_(p.grad.reshape(-1))
            off += n

    def _unpack(self) -> None:
        off = 0
        for p, n in zip(self.params, self.numels):
            g = self.flat[off:off + n].view_as(p)
            if p.grad is None:
                p.grad = g.clone()
            else:
                p.grad.copy_(g)
            off += n

    def _unpack_views(self) -> None:
        off = 0
        for p, n in zip(self.params, self.numels):
            p.grad = self.flat[off:off + n].view_as(p)
            off += n

    @property
    def bytes(self) -> int:
        return self.total * 4


class SharedGradAllReduce(_FlatGrads):
    """Sums the .grad of shared parameters across ranks with NCCL (or gloo).

    params: the shared leaf tensors (e.g. means3d, scales, quats, opacities, colors).
    bucket_bytes: size of each all-reduce bucket (fp32 elements * 4).
    """

    def __init__(self, params: Sequence[torch.Tensor], bucket_bytes: int = 64 << 20,
                 group: Optional[dist.ProcessGroup] = None):
        self._init_flat(params)
        self.group = group
        elems = max(1, bucket_bytes // 4)
        self.buckets = [(s, min(self.total, s + elems)) for s in range(0, self.total, elems)]
        self._works = []

    def start(self) -> None:
        """Packs the local gradients and launches the bucketed async all-reduce."""
        self._pack()
        self._works = [dist.all_reduce(self.flat[s:e], op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                       for s, e in self.buckets]

    def finish(self) -> None:
        """Waits for the reduction and writes the summed gradients back."""
        for w in self._works:
            w.wait()
        self._works = []
        self._unpack()

    def __call__(self) -> None:
        self.start()
        self.finish()


class _DeviceArray:
    """A raw device allocation seen by torch.as_tensor (no copy, no ownership)."""

    def __init__(self, ptr: int, n_floats: int):
        self.__cuda_array_interface__ = {"shape": (n_floats,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGradAllReduce(_FlatGrads):
    """Sums the .grad of shared parameters across the ranks of one node with
    gsb_peer_allreduce_sum: each rank owns a CUDA IPC buffer that every other
    rank maps; one kernel per call barriers on flags in those buffers, adds
    rank r's shard of all buffers over NVLink and writes the sum into all of
    them. One process per GPU, all ranks on one node, at most 8 ranks; `group`
    is used only to exchange the IPC handles (any backend).

    grads_as_views: after a call each parameter's .grad is a view into the
    summed buffer (no copy back), valid until the next call, as with DDP's
    gradient_as_bucket_view. False copies the sums into the .grad tensors.
    wait_s: bound of each barrier wait inside the kernel. A rank that waits
    longer, or that meets a peer that gave up, raises the kernel's error flag
    (the sums of that call are then not valid on that rank). Each call copies
    the flag to host memory without waiting, and the next call (or
    check_errors()) raises RuntimeError before touching the buffer, so a failed
    sum never reaches a second step silently.
    """

    def __init__(self, params: Sequence[torch.Tensor], group: Optional[dist.ProcessGroup] = None,
                 grads_as_views: bool = True, wait_s: float = 10.0):
        from . import _native as N

        self._N = N
        self._L = N.load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > N.GSB_PEER_MAX_RANKS:
            raise ValueError(f"PeerGradAllReduce supports at most {N.GSB_PEER_MAX_RANKS} ranks")
        dev = params[0].device
        if dev.type != "cuda":
            raise ValueError("PeerGradAllReduce needs CUDA parameters")
        total = sum(p.numel() for p in params)
        self.padded = (total + 3) // 4 * 4  # the kernel moves 16-byte vectors
        with torch.cuda.device(dev):
            base = C.c_void_p()
            N.check(self._L.gsb_peer_buffer_alloc(self.padded * 4, C.byref(base)), "gsb_peer_buffer_alloc")
            self._own = base.value
            handle = (C.c_char * N.GSB_PEER_HANDLE_BYTES)()
            N.check(self._L.gsb_peer_handle(C.c_void_p(self._own), handle), "gsb_peer_handle")
            handles: List[Optional[bytes]] = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self._opened = []
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                peer = C.c_void_p()
                N.check(self._L.gsb_peer_open(C.create_string_buffer(h, len(h)), C.byref(peer)), "gsb_peer_open")
                self._opened.append(peer.value)
                bases.append(peer.value)
            self._bases = (C.c_void_p * self.world)(*bases)
            data = torch.as_tensor(_DeviceArray(self._own + N.GSB_PEER_FLAG_BYTES, self.padded), device=dev)
            data.zero_()
        self._init_flat(params, flat=data[:total])
        self._data = data
        self.status = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, device=dev)
        self._status_host = torch.zeros(N.GSB_STATUS_WORDS, dtype=torch.int32, pin_memory=True)
        self._status_copied = torch.cuda.Event()
        self._pending = False
        self.epoch = 0
        self.wait_ns = max(1, int(wait_s * 1e9))
        self.grads_as_views = grads_as_views

    def __call__(self) -> None:
        self._raise_if_failed(sync=False)
        self._pack()
        self.epoch += 1
        dev = self._data.device
        stream = torch.cuda.current_stream(dev)
        self._N.check(self._L.gsb_peer_allreduce_sum(self.rank, self.world, self._bases, self.padded,
                                                     self.epoch & 0xFFFFFFFF, self.wait_ns,
                                                     self._N.ptr(self.status), stream.cuda_stream),
                      "gsb_peer_allreduce_sum")
        self._status_host.copy_(self.status, non_blocking=True)
        self._status_copied.record(stream)
        self._pending = True
        if self.grads_as_views:
            self._unpack_views()
        else:
            self._unpack()

    def _raise_if_failed(self, sync: bool) -> None:
        if not self._pending:
            return
        if sync or not self._status_copied.query():
            self._status_copied.synchronize()
        self._pending = False
        flags = int(self._status_host[self._N.GSB_STATUS_ERROR]) & 0xFFFFFFFF
        if flags:
            raise RuntimeError(f"gsplat_b200 peer all-reduce (epoch {self.epoch}): a rank did not reach a barrier "
                               f"in time or gave up the call; its sums are not valid (device error flags {flags})")

    def check_errors(self) -> None:
        """Raises if the last call timed out waiting for a peer or met a peer
        that gave up (waits for that call's status copy)."""
        self._raise_if_failed(sync=True)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (collective: every rank calls it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self._data.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            self._L.gsb_peer_close(C.c_void_p(p))
        dist.barrier(group=self.group)
        self._L.gsb_peer_buffer_free(C.c_void_p(self._own))
        self._own = None
