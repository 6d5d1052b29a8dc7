"""Batch-sharded data parallelism on CPU: two ``gloo`` ranks (world_size 2).

The replica model here is the oracle's CPU restatement of the reference
module (same parameters as the drop-in ``DDPM``); the code under test is the
host-side data-parallel logic — sharding, parameter broadcast, bucketed
gradient averaging with and without backward-overlapped hooks — which is the
same for the CUDA model over NCCL.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dynamicconvolutionoperator_b200.data_parallel import (
    GradAllReducer,
    broadcast_parameters,
    default_buckets,
    shard_batch,
)
from oracle import ddpm_oracle as orc

WORLD = 2
SHAPE = (4, 4, 9, 7)  # global batch 4 -> 2 samples per rank
KS = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_batch_grads():
    """Single-process reference: mean-over-batch loss on the whole batch."""
    model = orc.make_model(SHAPE[1], KS, dtype=torch.float64, seed=0)
    x, y, g = orc.make_inputs(SHAPE, dtype=torch.float64, seed=5, grad_seed=6)
    loss = (model(x, y) * g).sum() / SHAPE[0]
    loss.backward()
    return {n: p.grad.clone() for n, p in model.named_parameters()}


def _rank_main(rank, port, overlap, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        # ranks start from different weights; broadcast makes them rank 0's
        model = orc.make_model(SHAPE[1], KS, dtype=torch.float64, seed=0 if rank == 0 else 99)
        broadcast_parameters(model)
        reducer = GradAllReducer(model, overlap=overlap)
        x, y, g = orc.make_inputs(SHAPE, dtype=torch.float64, seed=5, grad_seed=6)
        xs, ys, gs = (shard_batch(t, rank, WORLD) for t in (x, y, g))
        loss = (model(xs, ys) * gs).sum() / xs.shape[0]
        loss.backward()
        reducer.all_reduce()
        reducer.remove_hooks()
        grads = {n: p.grad.clone() for n, p in model.named_parameters()}
        params = {n: p.detach().clone() for n, p in model.named_parameters()}
        torch.save({"grads": grads, "params": params}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("overlap", [False, True])
def test_two_rank_gradients_match_full_batch(tmp_path, overlap):
    mp.spawn(_rank_main, args=(_free_port(), overlap, str(tmp_path)), nprocs=WORLD, join=True)
    gold = _full_batch_grads()
    results = [torch.load(tmp_path / f"rank{r}.pt") for r in range(WORLD)]
    ref_params = orc.make_model(SHAPE[1], KS, dtype=torch.float64, seed=0).state_dict()
    for res in results:
        for name, p in res["params"].items():
            assert torch.equal(p, ref_params[name]), name  # broadcast from rank 0
        for name, grad in res["grads"].items():
            torch.testing.assert_close(grad, gold[name], rtol=1e-10, atol=1e-12)
    # every rank ends the step with identical gradients
    for name in gold:
        assert torch.equal(results[0]["grads"][name], results[1]["grads"][name])


def test_shard_batch_slices_and_rejects_ragged():
    t = torch.arange(12).reshape(6, 2)
    assert torch.equal(shard_batch(t, 1, 3), t[2:4])
    assert torch.equal(torch.cat([shard_batch(t, r, 2) for r in range(2)]), t)
    with pytest.raises(ValueError, match="not divisible"):
        shard_batch(t, 0, 4)


def test_default_buckets_put_fuse_first():
    model = orc.make_model(4, 3)
    buckets = default_buckets(model)
    names = {id(p): n for n, p in model.named_parameters()}
    assert [names[id(p)] for p in buckets[0]] == ["fuse.weight", "fuse.bias"]
    assert [names[id(p)] for p in buckets[1]] == ["generator.weight", "generator.bias"]


def _missing_grad_main(rank, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        model = orc.make_model(4, 3)
        reducer = GradAllReducer(model)
        try:
            reducer.all_reduce()  # no backward ran: no gradients
            msg = "no error"
        except RuntimeError as e:
            msg = str(e)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_all_reduce_without_gradients_raises_on_every_rank(tmp_path):
    mp.spawn(_missing_grad_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for r in range(WORLD):
        assert "no gradient" in (tmp_path / f"rank{r}.txt").read_text()


# ---- flat gradient buffers written by the backward itself (no gather/scatter) ----
class _AffineFn(torch.autograd.Function):
    """y = x w^T + b whose backward writes dW and db into the parameters'
    attached gradient buffers, the way the library's backward kernels do."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.bias = b
        return x @ w.t() + b

    @staticmethod
    def backward(ctx, g):
        from dynamicconvolutionoperator_b200 import _gradbuf

        x, w = ctx.saved_tensors
        gw = _gradbuf.grad_buffer(w, w.shape, w.dtype, w.device)
        torch.matmul(g.t(), x, out=gw)
        gb = _gradbuf.grad_buffer(ctx.bias, ctx.bias.shape, w.dtype, w.device)
        torch.sum(g, 0, out=gb)
        _gradbuf.grads_written((w, ctx.bias), (gw, gb))  # before the input gradient, as the library
        return g @ w, gw, gb


class _Toy(torch.nn.Module):
    """Two affine layers named like the DDPM's (``fuse`` is the last layer)."""

    def __init__(self, seed):
        super().__init__()
        gen = torch.Generator().manual_seed(seed)
        self.generator = torch.nn.Linear(6, 5).double()
        self.fuse = torch.nn.Linear(5, 3).double()
        with torch.no_grad():
            for p in self.parameters():
                p.copy_(torch.randn(p.shape, generator=gen, dtype=torch.float64))

    def forward(self, x):
        h = _AffineFn.apply(x, self.generator.weight, self.generator.bias)
        return _AffineFn.apply(torch.tanh(h), self.fuse.weight, self.fuse.bias)


TOY_BATCH = 8


def _toy_data():
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(TOY_BATCH, 6, generator=gen, dtype=torch.float64)
    g = torch.randn(TOY_BATCH, 3, generator=gen, dtype=torch.float64)
    return x, g


def _toy_full_batch_grads():
    model = _Toy(0)
    x, g = _toy_data()
    ((model(x) * g).sum() / TOY_BATCH).backward()
    return {n: p.grad.clone() for n, p in model.named_parameters()}


def _toy_rank_main(rank, port, mode, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        model = _Toy(0)
        reducer = GradAllReducer(model, overlap=mode != "sync", early=mode == "early")
        x, g = _toy_data()
        xs, gs = shard_batch(x, rank, WORLD), shard_batch(g, rank, WORLD)
        per = xs.shape[0]
        result = {}
        for step in range(2):  # the second step reuses the re-armed buffers
            model.zero_grad(set_to_none=True)
            if mode == "accumulate":  # two micro-batches, the first without sync
                half = per // 2
                with reducer.no_sync():
                    ((model(xs[:half]) * gs[:half]).sum() / per).backward()
                ((model(xs[half:]) * gs[half:]).sum() / per).backward()
            else:
                ((model(xs) * gs).sum() / per).backward()
            if mode == "early":
                # both buckets were launched from inside the backward
                result.setdefault("early", []).append(sorted(reducer._early))
            if mode == "double":
                try:
                    ((model(xs) * gs).sum() / per).backward()
                    result["error"] = "no error"
                except RuntimeError as e:
                    result["error"] = str(e)
                break
            reducer.all_reduce()
        flat_ptrs = [(b.data_ptr(), b.data_ptr() + b.numel() * b.element_size())
                     for b in reducer.flat]
        result["in_flat"] = {
            n: any(lo <= p.grad.data_ptr() < hi for lo, hi in flat_ptrs)
            for n, p in model.named_parameters()
        }
        result["grads"] = {n: p.grad.clone() for n, p in model.named_parameters()}
        reducer.remove_hooks()
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["sync", "overlap", "accumulate", "early"])
def test_flat_buffers_hold_the_averaged_gradients(tmp_path, mode):
    """The backward writes each bucket's gradients into its flat buffer
    (param.grad is a view of it, no gather or scatter copy), the all-reduce
    averages them in place, and the result equals the full-batch gradient —
    also with two accumulated micro-batches and over two steps."""
    mp.spawn(_toy_rank_main, args=(_free_port(), mode, str(tmp_path)), nprocs=WORLD, join=True)
    gold = _toy_full_batch_grads()
    for r in range(WORLD):
        res = torch.load(tmp_path / f"rank{r}.pt")
        assert all(res["in_flat"].values()), res["in_flat"]
        if mode == "early":
            assert res["early"] == [[0, 1], [0, 1]], res["early"]
        for name, grad in res["grads"].items():
            torch.testing.assert_close(grad, gold[name], rtol=1e-12, atol=1e-12)


def test_second_backward_before_all_reduce_raises(tmp_path):
    """With overlapped all-reduces a second backward would add gradients the
    launched all-reduce never sees: it must raise instead of averaging wrong."""
    mp.spawn(_toy_rank_main, args=(_free_port(), "double", str(tmp_path)), nprocs=WORLD,
             join=True)
    for r in range(WORLD):
        assert "no_sync" in torch.load(tmp_path / f"rank{r}.pt")["error"]


def test_grad_buffer_is_handed_out_once_per_arming():
    from dynamicconvolutionoperator_b200 import _gradbuf

    p = torch.nn.Parameter(torch.zeros(4, 3))
    buf = torch.zeros(12)
    _gradbuf.attach(p, buf.view(4, 3))
    try:
        first = _gradbuf.grad_buffer(p, (4, 3), p.dtype, p.device)
        assert first.data_ptr() == buf.data_ptr()
        # second request in the same backward (layer applied twice): fresh memory
        second = _gradbuf.grad_buffer(p, (4, 3), p.dtype, p.device)
        assert second.data_ptr() != buf.data_ptr()
        _gradbuf.arm(p)
        p.grad = torch.ones(4, 3)  # an existing gradient is accumulated into: fresh memory
        assert _gradbuf.grad_buffer(p, (4, 3), p.dtype, p.device).data_ptr() != buf.data_ptr()
        p.grad = None
        assert _gradbuf.grad_buffer(p, (4, 3), p.dtype, p.device).data_ptr() == buf.data_ptr()
        with pytest.raises(ValueError):
            _gradbuf.attach(p, torch.zeros(5))
    finally:
        _gradbuf.detach(p)
