"""Multi-rank host logic on CPU (gloo, world_size 2): every rank derives the same
balanced shards, the shards cover the batch exactly once, and the single
all-reduce sums the joint-weight gradients and loss sums of all ranks."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from asr_b200.shard import allreduce_joint, balance_shards, shard_imbalance


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(7)
    il = rng.integers(200, 501, 64)
    tl = rng.integers(20, 121, 64)
    shards = balance_shards(il, tl, world)
    mine = torch.tensor(shards[rank])
    gathered = [torch.zeros(len(s), dtype=torch.int64) for s in shards]
    dist.all_gather(gathered, mine)
    dW = torch.full((3, 4), float(rank + 1))
    dWd = torch.full((2, 4), 10.0 * (rank + 1))
    loss = torch.tensor([0.5 * (rank + 1)])
    flat = allreduce_joint([dW, dWd, loss])
    out[rank] = {
        "cover": sorted(torch.cat(gathered).tolist()),
        "dW": dW.clone(), "dWd": dWd.clone(), "loss": float(loss), "flat": flat.numel(),
    }
    dist.barrier()
    dist.destroy_process_group()


def test_shards_and_allreduce_world2():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        assert res[r]["cover"] == list(range(64))
        assert torch.equal(res[r]["dW"], torch.full((3, 4), 3.0))
        assert torch.equal(res[r]["dWd"], torch.full((2, 4), 30.0))
        assert res[r]["loss"] == pytest.approx(1.5)
        assert res[r]["flat"] == 3 * 4 + 2 * 4 + 1


def test_balance_is_deterministic_and_tight():
    rng = np.random.default_rng(0)
    il = rng.integers(200, 501, 512)
    tl = rng.integers(20, 121, 512)
    for world in (1, 2, 4, 8):
        a = balance_shards(il, tl, world)
        b = balance_shards(il, tl, world)
        assert all(np.array_equal(x, y) for x, y in zip(a, b))
        assert sorted(np.concatenate(a).tolist()) == list(range(512))
        assert shard_imbalance(il, tl, a) < 1.01


def test_single_rank_allreduce_is_identity():
    x = torch.arange(6.0).reshape(2, 3)
    y = torch.tensor([1.0])
    flat = allreduce_joint([x, y])
    assert torch.equal(flat, torch.tensor([0.0, 1, 2, 3, 4, 5, 1]))
