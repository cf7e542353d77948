"""Known-answer test of the oracle against Hugging Face's independent Qwen3 implementation.

The reference pins its attention path this way (tests/correctness/test_model_vs_hf.py:17-43):
a tiny random Qwen3 in float64 on the CPU, logits compared through a fresh prefill, a chunk that
attends to cached keys, and one-token decodes.  Here the same check runs the oracle's attention
(and the harness forward) against transformers' Qwen3ForCausalLM.
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention_oracle as orc
from qwen3_harness import Qwen3Weights, Shapes, forward, logits, oracle_attention

transformers = pytest.importorskip("transformers")

TINY = dict(vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
            num_attention_heads=4, num_key_value_heads=2, head_dim=16,
            max_position_embeddings=1024, rms_norm_eps=1e-6, tie_word_embeddings=True)
BLOCK = 4


def _hf(seed: int = 0, **over):
    torch.manual_seed(seed)
    model = transformers.Qwen3ForCausalLM(transformers.Qwen3Config(**{**TINY, **over}))
    return model.to(torch.float64).eval()


def _theta(hf) -> float:
    d = hf.config.to_dict()
    return float(d.get("rope_theta") or (d.get("rope_parameters") or {}).get("rope_theta") or 1e4)


def _ours(hf) -> Qwen3Weights:
    s = Shapes(512, 64, 128, 2, 4, 2, 16, 1e-6, _theta(hf))
    return Qwen3Weights.from_hf_state_dict(s, hf.state_dict(), torch.float64, "cpu")


def _caches(w: Qwen3Weights, slots: int):
    shape = (slots, w.s.kv_heads, w.s.head_dim)
    return [(torch.zeros(shape, dtype=torch.float64), torch.zeros(shape, dtype=torch.float64))
            for _ in range(w.s.layers)]


def _run_chunk(w: Qwen3Weights, caches, ids: list[int], start: int) -> torch.Tensor:
    """One chunk of one sequence whose blocks are 0, 1, 2, ... (tests/helpers.py:26-49)."""
    n = len(ids)
    table = list(range(-(-(start + n) // BLOCK)))
    chunk = orc.SeqChunk(0, n, start, table)
    slots = torch.tensor(orc.slots_for(chunk, BLOCK))
    meta = orc.build_metadata([chunk], slots, BLOCK)
    cos, sin = orc.rope_tables(w.s.head_dim, 1024, w.s.theta)
    pos = torch.arange(start, start + n)
    hidden = forward(w, torch.tensor(ids), oracle_attention(w, caches, meta, cos[pos], sin[pos]))
    return logits(w, hidden)


@torch.no_grad()
def test_prefill_logits_match_hf() -> None:
    hf = _hf()
    ids = torch.randint(0, 512, (40,), generator=torch.Generator().manual_seed(0)).tolist()
    ref = hf(torch.tensor([ids])).logits[0].double()
    w = _ours(hf)
    got = _run_chunk(w, _caches(w, 40), ids, 0)
    torch.testing.assert_close(got.double(), ref, atol=1e-6, rtol=1e-5)


@torch.no_grad()
def test_chunked_prefill_and_decode_match_hf() -> None:
    hf = _hf()
    ids = torch.randint(0, 512, (50,), generator=torch.Generator().manual_seed(1)).tolist()
    ref = hf(torch.tensor([ids])).logits[0].double()
    w = _ours(hf)
    kv = _caches(w, 64)
    parts = [_run_chunk(w, kv, ids[:20], 0), _run_chunk(w, kv, ids[20:43], 20)]
    parts += [_run_chunk(w, kv, [ids[p]], p) for p in range(43, 50)]
    torch.testing.assert_close(torch.cat(parts).double(), ref, atol=1e-6, rtol=1e-5)


@torch.no_grad()
def test_untied_lm_head() -> None:
    hf = _hf(seed=3, tie_word_embeddings=False)
    ids = list(range(5, 25))
    ref = hf(torch.tensor([ids])).logits[0].double()
    w = _ours(hf)
    torch.testing.assert_close(_run_chunk(w, _caches(w, 20), ids, 0).double(), ref, atol=1e-6,
                               rtol=1e-5)
