"""Loading the golden fixtures and running the oracle on a case (test helpers, CPU only)."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from golden.cases import D, EPS, H, KVH, THETA, CaseInputs, make_inputs
from oracle import attention_oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str, dtype: torch.dtype) -> dict[str, torch.Tensor | str]:
    z = np.load(GOLDEN / f"{name}.npz")
    out: dict[str, torch.Tensor | str] = {"digest": bytes(z["digest"]).decode()}
    for key in ("q_rot", "k_rot", "k_at_slots", "v_at_slots", "out"):
        if key not in z.files:
            out[key + "_sha256"] = bytes(z[key + "_sha256"]).decode()
            continue
        a = z[key]
        if a.dtype == np.uint16:
            out[key] = torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
        else:
            out[key] = torch.from_numpy(a.copy()).to(dtype)
    return out


def oracle_meta(inp: CaseInputs) -> orc.OracleMeta:
    chunks = [orc.SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table))
              for c in inp.batch.chunks]
    return orc.build_metadata(chunks, torch.from_numpy(inp.batch.slots), 16)


def run_oracle(inp: CaseInputs) -> dict[str, torch.Tensor]:
    """The oracle's layer on the case's inputs (CPU, the case's dtype)."""
    cos, sin = orc.rope_tables(D, inp.max_positions, THETA)
    k_cache, v_cache = inp.k_slots.clone(), inp.v_slots.clone()
    positions = torch.from_numpy(inp.batch.positions)
    slots = torch.from_numpy(inp.batch.slots)
    q, k, v, out = orc.attention_layer(
        inp.qkv, inp.q_weight, inp.k_weight, EPS, cos, sin, positions, k_cache, v_cache,
        oracle_meta(inp), H, KVH, D,
    )
    return {"q_rot": q, "k_rot": k, "k_at_slots": k_cache[slots], "v_at_slots": v_cache[slots],
            "out": out, "k_cache": k_cache, "v_cache": v_cache}


def tensor_sha256(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes in the layout make_golden.py hashes (bf16 as uint16)."""
    import hashlib

    c = t.contiguous()
    if c.dtype == torch.bfloat16:
        c = c.view(torch.int16)
    return hashlib.sha256(c.numpy().tobytes()).hexdigest()


def matches(got: torch.Tensor, gold: dict, key: str) -> bool:
    """Bit equality with a stored array, or with its stored digest for compact cases."""
    if key in gold:
        return torch.equal(got, gold[key])
    return tensor_sha256(got) == gold[key + "_sha256"]


__all__ = ["load_golden", "make_inputs", "matches", "oracle_meta", "run_oracle", "tensor_sha256"]
