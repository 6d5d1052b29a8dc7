"""Batch-sharded data parallelism for DDPM training over NCCL (NVLink/NVSwitch).

The reference has no multi-GPU code. Samples of a DDPM batch are independent
in the forward pass; the only cross-sample coupling is the sum of the
parameter gradients (generator and fuse weights/biases: 259,840 values at
C=64, K=3). So one process per GPU holds a full replica, takes its slice of
the global batch, runs forward+backward, and averages the four parameter
gradients with NCCL all-reduces. Nothing on the data path crosses GPUs.

Gradients are bucketed in the order backward produces them: the fuse conv's
gradients are ready first (it is the last layer), the generator's last, so
with ``overlap=True`` the fuse bucket's all-reduce runs on NCCL's stream while
the DDPM filter backward is still computing.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn


def shard_batch(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Contiguous slice ``rank`` of ``world`` along the batch dimension.

    The global batch must divide evenly: a ragged shard would change each
    rank's weight in the averaged gradient.
    """
    n = t.shape[0]
    if n % world != 0:
        raise ValueError(f"global batch {n} is not divisible by world size {world}")
    per = n // world
    return t[rank * per : (rank + 1) * per]


def broadcast_parameters(module: nn.Module, src: int = 0, group=None) -> None:
    """Make every rank's replica identical to ``src``'s."""
    for p in module.parameters():
        dist.broadcast(p.data, src=src, group=group)


def default_buckets(module: nn.Module) -> list[list[nn.Parameter]]:
    """Fuse-conv parameters first, then everything else (generator)."""
    fuse = [p for n, p in module.named_parameters() if n.startswith("fuse.") and p.requires_grad]
    rest = [p for n, p in module.named_parameters() if not n.startswith("fuse.") and p.requires_grad]
    return [b for b in (fuse, rest) if b]


class GradAllReducer:
    """Average parameter gradients across ranks, one flat all-reduce per bucket.

    Usage (per step): ``loss.backward(); reducer.all_reduce()``. With
    ``overlap=True`` each bucket starts its all-reduce from a
    post-accumulate-grad hook as soon as its last gradient exists, and
    ``all_reduce()`` only waits for them.
    """

    def __init__(self, module: nn.Module, group=None, overlap: bool = False,
                 buckets: list[list[nn.Parameter]] | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.buckets = buckets if buckets is not None else default_buckets(module)
        backend = dist.get_backend(group)
        self.op = dist.ReduceOp.AVG if backend == "nccl" else dist.ReduceOp.SUM
        self.divide = self.op != dist.ReduceOp.AVG
        self.overlap = overlap
        self._pending: dict[int, tuple[object, torch.Tensor]] = {}
        self._ready: dict[int, int] = {}
        self._hooks = []
        if overlap:
            for bi, bucket in enumerate(self.buckets):
                for p in bucket:
                    self._hooks.append(p.register_post_accumulate_grad_hook(self._make_hook(bi)))

    def _make_hook(self, bi: int):
        def hook(_p):
            self._ready[bi] = self._ready.get(bi, 0) + 1
            if self._ready[bi] == len(self.buckets[bi]):
                self._launch(bi, async_op=True)
        return hook

    def _launch(self, bi: int, async_op: bool):
        grads = [p.grad for p in self.buckets[bi]]
        if any(g is None for g in grads):
            raise RuntimeError("a parameter in the bucket has no gradient")
        flat = torch.cat([g.reshape(-1) for g in grads])
        work = dist.all_reduce(flat, op=self.op, group=self.group, async_op=async_op)
        self._pending[bi] = (work, flat)

    def all_reduce(self) -> None:
        """Finish the step's gradient averaging (launching what has not started)."""
        for bi in range(len(self.buckets)):
            if bi not in self._pending:
                self._launch(bi, async_op=False)
        for bi, (work, flat) in sorted(self._pending.items()):
            if work is not None:
                work.wait()
            if self.divide:
                flat.div_(self.world)
            off = 0
            for p in self.buckets[bi]:
                n = p.grad.numel()
                p.grad.copy_(flat[off : off + n].view_as(p.grad))
                off += n
        self._pending.clear()
        self._ready.clear()

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()


__all__ = ["GradAllReducer", "broadcast_parameters", "default_buckets", "shard_batch"]
