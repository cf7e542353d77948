"""Pin the CPU oracle: it must reproduce the reference's own outputs on the golden cases.

The golden files were produced by running MiniServe's unmodified code
(``tests/golden/make_golden.py``); the oracle is a restatement, so on the same CPU the two must
agree bit for bit on every elementwise result and the scatter, and to fp32/bf16 rounding on the
attention output (both call PyTorch's CPU SDPA on the same gathered tensors).
"""

from __future__ import annotations

import pytest
import torch

from golden.cases import CASES, D
from golden_io import load_golden, make_inputs, matches, run_oracle
from oracle import attention_oracle as orc


@pytest.mark.parametrize("name", CASES)
def test_oracle_reproduces_reference_golden(name: str) -> None:
    inp = make_inputs(name)
    gold = load_golden(name, inp.dtype)
    assert inp.digest() == gold["digest"], "seeded input generation drifted"
    got = run_oracle(inp)
    for key in ("q_rot", "k_rot", "k_at_slots", "v_at_slots"):
        assert matches(got[key], gold, key), key
    tol = 1e-6 if inp.dtype == torch.float32 else 1e-2
    torch.testing.assert_close(got["out"].float(), gold["out"].float(), atol=tol, rtol=0)


@pytest.mark.parametrize("name", CASES)
def test_grouped_oracle_matches_direct_attention(name: str) -> None:
    """The reference's gather/group/mask formulation equals plain per-query attention."""
    inp = make_inputs(name)
    got = run_oracle(inp)
    direct = orc.direct_attention(
        got["q_rot"], got["k_cache"], got["v_cache"], inp.batch.chunks, 16, D**-0.5
    )
    tol = 1e-5 if inp.dtype == torch.float32 else 2e-2
    torch.testing.assert_close(got["out"].double(), direct, atol=tol, rtol=0)


def test_slot_arithmetic_matches_runner() -> None:
    """slot = table[p // 16] * 16 + p % 16 for the new tokens (model_runner.py:189)."""
    inp = make_inputs("mixed_bf16")
    ref = []
    for c in inp.batch.chunks:
        ref.extend(orc.slots_for(orc.SeqChunk(c.flat_start, c.num_new, c.num_cached,
                                              list(c.block_table)), 16))
    assert ref == inp.batch.slots.tolist()
