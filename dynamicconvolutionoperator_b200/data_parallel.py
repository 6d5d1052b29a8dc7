"""Batch-sharded data parallelism for DDPM training over NCCL (NVLink/NVSwitch).

The reference has no multi-GPU code. Samples of a DDPM batch are independent
in the forward pass; the only cross-sample coupling is the sum of the
parameter gradients (generator and fuse weights/biases: 259,840 values at
C=64, K=3). So one process per GPU holds a full replica, takes its slice of
the global batch, runs forward+backward, and averages the four parameter
gradients with NCCL all-reduces. Nothing on the data path crosses GPUs.

Gradients are bucketed in the order backward produces them: the fuse conv's
gradients are ready first (it is the last layer), the generator's last. Each
bucket owns one flat buffer, and the library's backward kernels write the
bucket's gradients straight into it (``_gradbuf``), so ``param.grad`` is a view
of the flat buffer and the all-reduce needs no gather or scatter copy. With
``overlap=True`` (the default) a bucket's all-reduce is launched from a
post-accumulate-grad hook as soon as its last gradient exists, so the fuse
bucket's all-reduce runs on NCCL's stream while the generator backward is
still computing; with ``early=True`` the generator bucket's all-reduce starts
inside the generator backward, right after its weight-gradient kernel and
before its data-gradient kernel, so that one overlaps too. The whole step,
collectives included, can be captured in one CUDA graph.
"""

from __future__ import annotations

import contextlib

import torch
import torch.distributed as dist
from torch import nn

from . import _gradbuf


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
    """Make every rank's replica identical to ``src``'s.

    Broadcasts into each parameter itself (under ``no_grad``), not into
    ``p.data``: the in-place write then bumps the parameter's version counter
    like any other in-place update.
    """
    with torch.no_grad():
        for p in module.parameters():
            dist.broadcast(p, src=src, group=group)


def default_buckets(module: nn.Module) -> list[list[nn.Parameter]]:
    """Fuse-conv parameters first, then everything else (generator)."""
    fuse = [p for n, p in module.named_parameters() if n.startswith("fuse.") and p.requires_grad]
    rest = [p for n, p in module.named_parameters() if not n.startswith("fuse.") and p.requires_grad]
    return [b for b in (fuse, rest) if b]


class GradAllReducer:
    """Average parameter gradients across ranks, one flat all-reduce per bucket.

    Usage per step: ``loss.backward(); reducer.all_reduce()``. With
    ``overlap=True`` each bucket's all-reduce starts from a post-accumulate-grad
    hook once its last gradient exists, and ``all_reduce()`` waits for them
    (on the device: the current stream waits for NCCL's, the host does not
    block). For gradient accumulation, run every micro-batch but the last
    under ``with reducer.no_sync():``; a second backward outside ``no_sync``
    before ``all_reduce()`` raises, since its gradients would miss the
    all-reduce already launched.

    ``flat=True`` gives every bucket whose parameters share a dtype and device
    one flat gradient buffer that the library's backward writes into; when a
    gradient did not land there (another autograd function produced it) the
    bucket falls back to gathering into the flat buffer and copying back.

    ``early=True`` (with ``overlap`` and ``flat``) launches a bucket's
    all-reduce as soon as the library's backward reports that it has written
    all of the bucket's gradients into the flat buffer (``_gradbuf``), before
    the rest of that backward runs. It requires that each of the bucket's
    parameters gets its gradient from one use in the backward: a second
    contribution would be added after the all-reduce started.
    """

    def __init__(self, module: nn.Module, group=None, overlap: bool = True,
                 buckets: list[list[nn.Parameter]] | None = None, flat: bool = True,
                 early: bool = False):
        self.group = group
        self.world = dist.get_world_size(group)
        self.buckets = buckets if buckets is not None else default_buckets(module)
        backend = dist.get_backend(group)
        self.op = dist.ReduceOp.AVG if backend == "nccl" else dist.ReduceOp.SUM
        self.divide = self.op != dist.ReduceOp.AVG
        self.overlap = overlap
        self._pending: dict[int, tuple[object, torch.Tensor, bool]] = {}
        self._ready: dict[int, int] = {}
        self._early: set[int] = set()
        self._sync = True
        self._hooks = []
        self._listener = None
        self.flat: list[torch.Tensor | None] = []
        for bucket in self.buckets:
            buf = None
            if flat and len({(p.dtype, p.device) for p in bucket}) == 1:
                buf = torch.zeros(sum(p.numel() for p in bucket), dtype=bucket[0].dtype,
                                  device=bucket[0].device)
                off = 0
                for p in bucket:
                    _gradbuf.attach(p, buf[off : off + p.numel()].view_as(p))
                    off += p.numel()
            self.flat.append(buf)
        if overlap:
            for bi, bucket in enumerate(self.buckets):
                for p in bucket:
                    self._hooks.append(p.register_post_accumulate_grad_hook(self._make_hook(bi)))
            if early and flat:
                self._listener = self._on_written
                _gradbuf.add_listener(self._listener)

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside accumulate gradients without an all-reduce."""
        prev, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = prev

    def _on_written(self, params, buffers):
        """``early``: the backward wrote ``params``' gradients into ``buffers``;
        launch the matching bucket now if they are its flat-buffer views."""
        if not self._sync:
            return
        ids = sorted(id(p) for p in params)
        for bi, bucket in enumerate(self.buckets):
            if self.flat[bi] is None or bi in self._pending or sorted(id(p) for p in bucket) != ids:
                continue
            for p, buf in zip(params, buffers):
                view = _gradbuf.view_of(p)
                if (buf is None or view is None or buf.data_ptr() != view.data_ptr()
                        or buf.numel() != view.numel()):
                    return
            work = dist.all_reduce(self.flat[bi], op=self.op, group=self.group, async_op=True)
            self._pending[bi] = (work, self.flat[bi], True)
            self._early.add(bi)
            return

    def _make_hook(self, bi: int):
        def hook(_p):
            if not self._sync:
                return
            if bi in self._early:  # launched from inside the backward
                self._ready[bi] = self._ready.get(bi, 0) + 1
                return
            if bi in self._pending:
                raise RuntimeError(
                    "backward ran again before all_reduce(): wrap the accumulation "
                    "micro-batches in reducer.no_sync()")
            self._ready[bi] = self._ready.get(bi, 0) + 1
            if self._ready[bi] == len(self.buckets[bi]):
                self._launch(bi, async_op=True)
        return hook

    def _in_place(self, bi: int) -> bool:
        """Whether every gradient of bucket ``bi`` already lives in its flat buffer."""
        if self.flat[bi] is None:
            return False
        for p in self.buckets[bi]:
            view = _gradbuf.view_of(p)
            if view is None or p.grad is None or p.grad.data_ptr() != view.data_ptr():
                return False
        return True

    def _launch(self, bi: int, async_op: bool):
        bucket = self.buckets[bi]
        if any(p.grad is None for p in bucket):
            raise RuntimeError("a parameter in the bucket has no gradient")
        in_place = self._in_place(bi)
        if in_place:
            flat = self.flat[bi]
        else:  # gather (some gradients may alias the flat buffer: use a fresh one)
            flat = torch.cat([p.grad.reshape(-1) for p in bucket])
        work = dist.all_reduce(flat, op=self.op, group=self.group, async_op=async_op)
        self._pending[bi] = (work, flat, in_place)

    def all_reduce(self) -> None:
        """Finish the step's gradient averaging (launching what has not started)."""
        for bi in range(len(self.buckets)):
            if bi not in self._pending:
                self._launch(bi, async_op=False)
        for bi, (work, flat, in_place) in sorted(self._pending.items()):
            if work is not None:
                work.wait()
            if self.divide:
                flat.div_(self.world)
            if bi in self._early:
                # launched before autograd stored the gradients: each must now
                # be the flat-buffer view (or, if autograd copied it, get the
                # averaged values copied in)
                for p in self.buckets[bi]:
                    view = _gradbuf.view_of(p)
                    if p.grad is None:
                        raise RuntimeError("a parameter in the bucket has no gradient")
                    if p.grad.data_ptr() != view.data_ptr():
                        p.grad.copy_(view.view_as(p.grad))
            elif not in_place:
                off = 0
                for p in self.buckets[bi]:
                    n = p.grad.numel()
                    p.grad.copy_(flat[off : off + n].view_as(p.grad))
                    off += n
        self._pending.clear()
        self._ready.clear()
        self._early.clear()
        for bucket in self.buckets:
            for p in bucket:
                _gradbuf.arm(p)

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
        if self._listener is not None:
            _gradbuf.remove_listener(self._listener)
            self._listener = None
        for bucket in self.buckets:
            for p in bucket:
                _gradbuf.detach(p)


__all__ = ["GradAllReducer", "broadcast_parameters", "default_buckets", "shard_batch"]
