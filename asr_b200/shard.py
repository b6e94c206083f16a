"""Batch-sharded data parallelism for the sequence losses.

The loss is per utterance, so a global batch is split across ranks by
utterance with no data-path collective; the only exchange is one all-reduce of
the joint-weight gradients and the loss sums (see ``allreduce_joint``).
Utterances are balanced by joint cost T_b * (U_b + 1) (proportional to the
GEMM work of their lattice) with the lattice recursion length T_b + U_b as the
tie-break, in the spirit of the reference's frame-budget bucketing
(src/asr/data/bucket_dataset.py:13-127).
"""

from __future__ import annotations

import heapq
from collections.abc import Sequence

import numpy as np


def utterance_cost(in_lens: Sequence[int], tgt_lens: Sequence[int]) -> np.ndarray:
    """Number of lattice nodes T_b * (U_b + 1) per utterance."""
    t = np.asarray(in_lens, np.int64)
    u = np.asarray(tgt_lens, np.int64)
    return t * (u + 1)


def balance_shards(in_lens: Sequence[int], tgt_lens: Sequence[int], world: int) -> list[np.ndarray]:
    """Greedy longest-first assignment of utterances to `world` ranks.

    Returns, per rank, the utterance indices sorted by length (so a rank's
    padded batch tensors stay tight). Every utterance appears exactly once.
    """
    if world < 1:
        raise ValueError(f"world must be >= 1, got {world}")
    t = np.asarray(in_lens, np.int64)
    u = np.asarray(tgt_lens, np.int64)
    cost = utterance_cost(t, u)
    order = sorted(range(len(cost)), key=lambda i: (-int(cost[i]), -int(t[i] + u[i]), i))
    heap = [(0, 0, r) for r in range(world)]  # (load, recursion length, rank)
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, dp, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(cost[i]), max(dp, int(t[i] + u[i])), r))
    return [np.array(sorted(s, key=lambda i: (int(t[i]), int(u[i]), i)), dtype=np.int64) for s in shards]


def shard_imbalance(in_lens, tgt_lens, shards) -> float:
    """max / mean of the per-rank joint cost (1.0 = perfectly balanced)."""
    cost = utterance_cost(in_lens, tgt_lens)
    loads = np.array([cost[s].sum() for s in shards], np.float64)
    return float(loads.max() / max(loads.mean(), 1.0))


def allreduce_joint(tensors, group=None):
    """Sums `tensors` (joint-weight gradients, loss sums, ...) over the process
    group with ONE collective: they are packed into a flat buffer, reduced, and
    the reduced values are copied back in place. Returns the flat buffer."""
    import torch
    import torch.distributed as dist

    flat = torch.cat([t.reshape(-1) for t in tensors])
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
        off = 0
        for t in tensors:
            n = t.numel()
            t.copy_(flat[off:off + n].view_as(t))
            off += n
    return flat
