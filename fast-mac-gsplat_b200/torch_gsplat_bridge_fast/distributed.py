"""Multi-GPU plumbing for the rasterizer: one process per GPU.

The reference is single-device (it chunks the view batch serially,
variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:910-938). Here:

* Independent views (a [B,G,...] batch of 2D splats, or several cameras of one 3D
  scene) are sharded round-robin over ranks. Each rank renders and
  differentiates its own views; there is no collective on the data path
  (weak scaling).
* Shared 3D Gaussians (every rank renders a different camera of the same
  scene): the per-Gaussian gradients of the shared parameters are summed
  across ranks with NCCL all-reduce (sum, fp32) over NVLink. The gradients are
  packed into one flat buffer, cut into buckets and reduced asynchronously;
  `start()` can be called on a side stream while other work proceeds.

The same code runs on CPU tensors with the gloo backend (tests).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist


def shard_views(num_views: int, world_size: int, rank: int) -> List[int]:
    """Round-robin assignment of view indices to a rank."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("invalid world_size/rank")
    return list(range(rank, num_views, world_size))


class SharedGradAllReduce:
    """Sums the .grad of shared parameters across ranks.

    params: the shared leaf tensors (e.g. means3d, scales, quats, opacities, colors).
    bucket_bytes: size of each all-reduce bucket (fp32 elements * 4).
    """

    def __init__(self, params: Sequence[torch.Tensor], bucket_bytes: int = 64 << 20,
                 group: Optional[dist.ProcessGroup] = None):
        if not params:
            raise ValueError("no parameters")
        self.params = list(params)
        self.group = group
        dev = self.params[0].device
        self.numels = [p.numel() for p in self.params]
        self.total = sum(self.numels)
        self.flat = torch.zeros(self.total, dtype=torch.float32, device=dev)
        elems = max(1, bucket_bytes // 4)
        self.buckets = [(s, min(self.total, s + elems)) for s in range(0, self.total, elems)]
        self._works = []

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

    @property
    def bytes(self) -> int:
        return self.total * 4
