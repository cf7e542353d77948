"""Sequence sharding of a decode step across GPUs (one process per GPU).

MiniServe is single-GPU; the path shards naturally by whole sequences: each rank owns its KV
pool, block tables and plan and runs its share of requests, so there is no data-path collective.
Sequences are assigned by context length (the bytes each rank must stream per layer) with greedy
longest-processing-time-first, which keeps every rank's sum of context tokens within one
sequence of the mean.  The only collective is an optional gather of per-rank results (sampled
token ids, or attention rows when validating).
"""

from __future__ import annotations

import heapq
from collections.abc import Sequence

import torch


def shard_by_tokens(context_lens: Sequence[int], world: int) -> list[list[int]]:
    """Indices of the sequences each rank serves (greedy LPT on context length).

    Returns ``world`` lists; every index appears exactly once; each list is in ascending order so a
    rank's flat batch keeps the global order of its sequences.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(context_lens)), key=lambda i: (-int(context_lens[i]), i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(context_lens[i]), r))
    return [sorted(s) for s in shards]


def shard_loads(context_lens: Sequence[int], shards: list[list[int]]) -> list[int]:
    return [sum(int(context_lens[i]) for i in s) for s in shards]


def gather_rows(local: torch.Tensor, shards: list[list[int]], rank: int,
                group: torch.distributed.ProcessGroup | None = None) -> torch.Tensor:
    """All-gather per-rank rows (one row per sequence, in the rank's shard order) and return them
    in global sequence order on every rank.  Works with NCCL (CUDA tensors) and gloo (CPU)."""
    import torch.distributed as dist

    world = len(shards)
    if local.shape[0] != len(shards[rank]):
        raise ValueError("local rows must match this rank's shard")
    width = max(len(s) for s in shards)
    padded = local.new_zeros((width, *local.shape[1:]))
    padded[: local.shape[0]] = local
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    total = sum(len(s) for s in shards)
    out = local.new_empty((total, *local.shape[1:]))
    for r, s in enumerate(shards):
        if s:
            out[torch.tensor(s, device=local.device)] = bufs[r][: len(s)]
    return out
