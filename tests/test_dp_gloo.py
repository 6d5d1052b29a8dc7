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
