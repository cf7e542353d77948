"""Generate the golden fixtures by running the MiniServe reference itself.

Run in a checkout that has the reference source next to it::

    MINISERVE_SRC=/path/to/MiniServe/src python tests/golden/make_golden.py

For every case in ``cases.py`` this builds the seeded inputs, then runs the reference's own code,
unmodified, on the CPU: ``RotaryEmbedding.build`` + ``RMSNorm`` + ``apply_rope`` in the op
order of ``Qwen3Attention.forward`` (src/miniserve/model/qwen3.py:94-98), the runner's slot
arithmetic (src/miniserve/runner/model_runner.py:189), ``build_attention_metadata`` and
``paged_attention`` (src/miniserve/attention/backends.py:80-197).  It stores the rotated q and k,
the scattered K/V rows, the attention output and a digest of the inputs in
``tests/golden/<case>.npz``.  The tests never import the reference; they read these files.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))

from cases import CASES, COMPACT, D, EPS, H, KVH, THETA, make_inputs  # noqa: E402
import hashlib  # noqa: E402


def _as_np(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def run_reference(name: str) -> dict[str, np.ndarray]:
    from miniserve.attention.backends import SeqChunk, build_attention_metadata, paged_attention
    from miniserve.model.layers import RMSNorm, RotaryEmbedding, apply_rope

    inp = make_inputs(name)
    b = inp.batch
    rope = RotaryEmbedding(D, inp.max_positions, THETA)
    rope.build(torch.device("cpu"))
    qn, kn = RMSNorm(D, EPS), RMSNorm(D, EPS)
    with torch.no_grad():
        qn.weight.copy_(inp.q_weight.float())
        kn.weight.copy_(inp.k_weight.float())
    qn, kn = qn.to(inp.dtype), kn.to(inp.dtype)

    t = b.num_tokens
    positions = torch.from_numpy(b.positions)
    slot_mapping = torch.from_numpy(b.slots)
    chunks = [SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table)) for c in b.chunks]
    k_cache, v_cache = inp.k_slots.clone(), inp.v_slots.clone()
    with torch.inference_mode():
        cos, sin = rope(positions)
        q, k, v = inp.qkv.split([H * D, KVH * D, KVH * D], dim=-1)
        q = qn(q.reshape(t, H, D))
        k = kn(k.reshape(t, KVH, D))
        v = v.reshape(t, KVH, D)
        q, k = apply_rope(q, k, cos, sin)
        meta = build_attention_metadata(chunks, slot_mapping, 16)
        out = paged_attention(q, k, v, k_cache, v_cache, meta, D**-0.5)
    arrays = {
        "digest": np.frombuffer(inp.digest().encode(), dtype=np.uint8),
        "q_rot": _as_np(q),
        "k_rot": _as_np(k),
        "k_at_slots": _as_np(k_cache[slot_mapping]),
        "v_at_slots": _as_np(v_cache[slot_mapping]),
        "out": _as_np(out),
        "n_groups": np.asarray([len(meta.groups)]),
        "n_prefills": np.asarray([len(meta.prefills)]),
    }
    if name in COMPACT:
        for key in ("q_rot", "k_rot", "k_at_slots", "v_at_slots"):
            digest = hashlib.sha256(np.ascontiguousarray(arrays[key]).tobytes()).hexdigest()
            arrays[key + "_sha256"] = np.frombuffer(digest.encode(), dtype=np.uint8)
            del arrays[key]
    return arrays


def main() -> None:
    src = os.environ.get("MINISERVE_SRC")
    if not src:
        raise SystemExit("set MINISERVE_SRC to the reference's src/ directory")
    sys.path.insert(0, src)
    torch.set_num_threads(os.cpu_count() or 1)
    only = sys.argv[1:]
    for name in CASES:
        if only and name not in only:
            continue
        arrays = run_reference(name)
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
        print(name, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
