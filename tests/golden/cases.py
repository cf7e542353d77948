"""Seeded parity cases shared by ``make_golden.py`` (which runs the MiniServe reference itself)
and the tests (which rerun the oracle and the CUDA path on the same inputs).

Each case is a batch geometry plus seeded activations: the fused qkv projection output
``[T, 4096]``, q/k norm weights ``1 + 0.1 N(0,1)``, eps 1e-6, RoPE theta 1e6, and a KV pool
already holding N(0,1) keys/values in every slot (the "cached" context).  Inputs are regenerated
from the seed (torch's CPU generator is deterministic), and a SHA-256 of them is stored with the
golden outputs so a drift in generation is caught.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import numpy as np
import torch

from miniserve_b200.workloads import Batch, config1, custom

H, KVH, D = 16, 8, 128
EPS = 1e-6
THETA = 1e6


@dataclass
class CaseInputs:
    batch: Batch
    dtype: torch.dtype
    qkv: torch.Tensor  # [T, (H + 2 KVH) * D]
    q_weight: torch.Tensor  # [D]
    k_weight: torch.Tensor
    k_slots: torch.Tensor  # reference layout [num_blocks * 16, KVH, D]
    v_slots: torch.Tensor
    max_positions: int

    def digest(self) -> str:
        h = hashlib.sha256()
        for t in (self.qkv, self.q_weight, self.k_weight, self.k_slots, self.v_slots):
            h.update(t.float().contiguous().numpy().tobytes())
        h.update(np.asarray([c.flat_start for c in self.batch.chunks], np.int64).tobytes())
        for c in self.batch.chunks:
            h.update(np.asarray([c.num_new, c.num_cached, *c.block_table], np.int64).tobytes())
        return h.hexdigest()


def _batch(name: str) -> Batch:
    if name == "cfg1_fp32":
        return config1(seed=11)
    if name == "mixed_bf16":
        # decode rows, a 5-token verify, a 9-token chunk (just over SHORT_QUERY), a chunk over a
        # cache that is not block aligned, and a fresh prompt (plain causal path).
        rows = [(1, 300), (1, 0), (1, 15), (1, 16), (5, 70), (9, 33), (24, 40), (20, 0)]
        return custom(rows, seed=12, name=name)
    if name == "prefix_verify_bf16":
        rows = [(5, 64 + u) for u in (3, 17, 40, 64, 65, 100)]
        return custom(rows, seed=13, shared=4, name=name)
    if name == "groups_bf16":
        # 24 decode rows of ~1k context: (n+1) * ctx0 > 16384 splits them into several gather
        # groups in the reference (backends.py:90-96), with ragged lengths inside each group.
        g = np.random.default_rng(14)
        rows = [(1, int(c)) for c in g.integers(700, 1300, size=24)]
        return custom(rows, seed=14, name=name)
    if name == "prefill_bf16":
        # chunks longer than 64 tokens (the tensor-core prefill path): over a non-aligned cache,
        # a fresh prompt just over one 64-token tile, a chunk over a long cache; plus a decode row.
        rows = [(80, 37), (66, 0), (1, 20), (70, 130)]
        return custom(rows, seed=15, name=name)
    raise KeyError(name)


CASES = ("cfg1_fp32", "mixed_bf16", "prefix_verify_bf16", "groups_bf16", "prefill_bf16")
# Cases whose q/k/v arrays are stored as SHA-256 digests (only the attention output in full).
COMPACT = ("prefill_bf16",)


def make_inputs(name: str) -> CaseInputs:
    batch = _batch(name)
    dtype = torch.float32 if name.endswith("fp32") else torch.bfloat16
    return random_inputs(batch, sum(map(ord, name)), dtype)


def random_inputs(batch: Batch, seed: int, dtype: torch.dtype = torch.bfloat16) -> CaseInputs:
    """Seeded activations and pool contents for any batch geometry."""
    g = torch.Generator().manual_seed(seed)
    t = batch.num_tokens
    slots = batch.num_blocks * 16
    qkv = torch.randn(t, (H + 2 * KVH) * D, generator=g).to(dtype)
    qw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    kw = (1 + 0.1 * torch.randn(D, generator=g)).to(dtype)
    k_slots = torch.randn(slots, KVH, D, generator=g).to(dtype)
    v_slots = torch.randn(slots, KVH, D, generator=g).to(dtype)
    return CaseInputs(batch, dtype, qkv, qw, kw, k_slots, v_slots, batch.max_position + 8)
