"""Seeded synthetic batches with the shapes of the five benchmark configurations.

MiniServe's own workloads are seeded random token ids (bench/promptsets.py:15-26); the attention
path only sees the batch geometry (which sequences, how many new and cached tokens, which
blocks) and random activations, so that is what these generators produce.  Block tables are a
seeded random permutation of the pool, handed out to sequences in order.

    1  8 decode rows, context U[1,512], pool 1070 blocks (fp32 in the CPU reference)
    2  256 decode rows, context U[256,4096], pool = 1.1 x blocks needed
    3  48 decode rows (context U[128,2048]) + 2 prefill chunks of 1000 tokens over 512 cached
    4  512 rows sharing a 64-block (1024-token) prefix, U[64,256] unique tokens, 5-token verify
    5  8192 decode rows, context logU[512,32768], sharded by tokens over the ranks
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .attention import SeqChunk
from .kv_pool import BLOCK_SIZE

NUM_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
NUM_LAYERS = 28
ROPE_THETA = 1e6
RMS_EPS = 1e-6


@dataclass
class Batch:
    """One step's batch geometry."""

    name: str
    chunks: list[SeqChunk]
    num_blocks: int  # pool size (per layer)
    shared_blocks: int = 0  # blocks referenced by every table (config 4's prefix)

    @property
    def num_tokens(self) -> int:
        return sum(c.num_new for c in self.chunks)

    @property
    def positions(self) -> np.ndarray:
        return np.concatenate(
            [np.arange(c.num_cached, c.context_len, dtype=np.int64) for c in self.chunks]
        ) if self.chunks else np.zeros(0, dtype=np.int64)

    @property
    def slots(self) -> np.ndarray:
        out = []
        for c in self.chunks:
            p = np.arange(c.num_cached, c.context_len, dtype=np.int64)
            tab = np.asarray(c.block_table, dtype=np.int64)
            out.append(tab[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE)
        return np.concatenate(out) if out else np.zeros(0, dtype=np.int64)

    @property
    def max_position(self) -> int:
        return max((c.context_len for c in self.chunks), default=0)

    def kv_tokens_read(self) -> int:
        """Context tokens each row attends to, summed over sequences (logical, per layer)."""
        return sum(c.context_len for c in self.chunks)

    def unique_kv_tokens(self) -> int:
        """Tokens of distinct physical blocks read (a shared prefix block counts once)."""
        seen: set[int] = set()
        for c in self.chunks:
            nb = -(-c.context_len // BLOCK_SIZE)
            seen.update(c.block_table[:nb])
        return len(seen) * BLOCK_SIZE


def _assemble(name: str, rows: list[tuple[int, int]], rng: np.random.Generator,
              pool_blocks: int | None = None, slack: float = 1.1, shared: int = 0) -> Batch:
    """rows: (num_new, num_cached) per sequence, in flat-batch order."""
    need = [-(-(n + c) // BLOCK_SIZE) for n, c in rows]
    own = [max(0, b - shared) for b in need]
    total = shared + sum(own)
    nblocks = pool_blocks if pool_blocks is not None else math.ceil(slack * total)
    if total > nblocks:
        raise ValueError(f"{name}: {total} blocks needed, pool has {nblocks}")
    perm = rng.permutation(nblocks).astype(np.int64)
    prefix = perm[:shared].tolist()
    cursor = shared
    chunks = []
    flat = 0
    for (n, c), k in zip(rows, own, strict=True):
        table = prefix + perm[cursor : cursor + k].tolist()
        cursor += k
        chunks.append(SeqChunk(flat, n, c, table))
        flat += n
    return Batch(name, chunks, nblocks, shared)


def config1(seed: int = 0) -> Batch:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 513, size=8)
    return _assemble("cfg1", [(1, int(L) - 1) for L in ctx], rng, pool_blocks=1070)


def config2(seed: int = 0, num_seqs: int = 256, rank: int = 0, world: int = 1) -> Batch:
    """256 decode rows, contexts U[256, 4096].  With ``world`` > 1 (weak scaling, fixed work per
    GPU): one global batch of ``num_seqs * world`` rows whose contexts are ``world`` copies of the
    single-GPU batch's, split over the ranks by context tokens (greedy LPT,
    ``sharding.shard_by_tokens``), so every rank streams the single-GPU batch's KV bytes; each
    rank's share gets its own pool and permuted tables.  With one rank it is the single-GPU batch
    itself."""
    from .sharding import shard_by_tokens

    rng = np.random.default_rng(seed)
    ctx = rng.integers(256, 4097, size=num_seqs)
    if world == 1:
        return _assemble("cfg2", [(1, int(L) - 1) for L in ctx], rng)
    everyone = np.tile(ctx, world)
    mine = shard_by_tokens(everyone.tolist(), world)[rank]
    return _assemble(f"cfg2[{rank}/{world}]", [(1, int(everyone[i]) - 1) for i in mine],
                     np.random.default_rng([seed, rank]))


def config3(seed: int = 0) -> Batch:
    rng = np.random.default_rng(seed)
    ctx = rng.integers(128, 2049, size=48)
    rows = [(1, int(L) - 1) for L in ctx] + [(1000, 512), (1000, 512)]
    return _assemble("cfg3", rows, rng)


def config4(seed: int = 0, num_seqs: int = 512) -> Batch:
    rng = np.random.default_rng(seed)
    prefix = 1024
    uniq = rng.integers(64, 257, size=num_seqs)
    rows = [(5, prefix + int(u)) for u in uniq]
    return _assemble("cfg4", rows, rng, shared=prefix // BLOCK_SIZE)


def config5_contexts(seed: int = 0, num_seqs: int = 8192) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.exp(rng.uniform(math.log(512), math.log(32768), size=num_seqs)).astype(np.int64)


def config5(rank: int = 0, world: int = 1, seed: int = 0, num_seqs: int = 8192,
            pool_bytes: float = 150e9, num_kv_heads: int = NUM_KV_HEADS) -> Batch:
    """This rank's share of the box-scale batch: 8192 decode rows, context logU[512, 32768],
    split across ranks by context tokens (greedy LPT).

    The whole batch needs ~7 TB of KV for 28 layers, far beyond a GPU's HBM, so (as the benchmark
    plan prescribes) one pool of about ``pool_bytes`` is shared by all layers and block ids are
    taken modulo the pool when the rank's blocks exceed it.  Reads stay HBM-streamed: the pool is
    far larger than L2.  ``num_blocks`` is the pool size; ``aliased`` says whether ids wrapped.
    """
    from .sharding import shard_by_tokens

    ctx = config5_contexts(seed, num_seqs)
    mine = shard_by_tokens(ctx.tolist(), world)[rank]
    need = [-(-int(ctx[i]) // BLOCK_SIZE) for i in mine]
    total = sum(need)
    block_bytes = num_kv_heads * 2 * BLOCK_SIZE * HEAD_DIM * 2
    cap = max(1, int(pool_bytes // block_bytes))
    nblocks = min(total, cap)
    rng = np.random.default_rng(seed + 1 + rank)
    ids = (rng.permutation(total) % nblocks).astype(np.int64)
    chunks, cursor = [], 0
    for k, (i, nb) in enumerate(zip(mine, need, strict=True)):
        L = int(ctx[i])
        chunks.append(SeqChunk(k, 1, L - 1, ids[cursor : cursor + nb].tolist()))
        cursor += nb
    b = Batch(f"cfg5[{rank}/{world}]", chunks, nblocks)
    b.aliased = total > nblocks  # type: ignore[attr-defined]
    return b


def custom(rows: list[tuple[int, int]], seed: int = 0, pool_blocks: int | None = None,
           shared: int = 0, name: str = "custom") -> Batch:
    """A batch from explicit (num_new, num_cached) rows."""
    return _assemble(name, rows, np.random.default_rng(seed), pool_blocks, shared=shared)


CONFIGS = {"cfg1": config1, "cfg2": config2, "cfg3": config3, "cfg4": config4}


def rope_tables(head_dim: int, max_positions: int, theta: float, device: "object" = "cpu"):
    """fp32 cos/sin tables ``[max_positions, head_dim]`` the way the model builds them
    (layers.py:43-50): angle(t, i) = t * theta**(-2i/head_dim), pair table repeated twice."""
    import torch

    exps = torch.arange(0, head_dim, 2, dtype=torch.int64, device=device).float() / head_dim
    inv_freq = 1.0 / (theta**exps)
    ang = torch.outer(torch.arange(max_positions, dtype=torch.float32, device=device), inv_freq)
    emb = torch.cat((ang, ang), dim=-1)
    return emb.cos(), emb.sin()
