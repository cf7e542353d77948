"""Greedy generation through the drop-in attention module, tokens fed back, against the
reference's own bf16 run (the pattern of the reference's tests/correctness/
test_engine_equivalence.py:24-117: greedy output compared token for token).

Model: Qwen3-0.6B's shapes (28 layers, hidden 1024, 16 query / 8 KV heads, head_dim 128, vocab
151,936) with seeded random weights (real weights are not available offline).  Four sequences:
prompts of 300 and 100 tokens (tensor-core kernel), 40 (tile kernel) and 5 (decode kernel) in one
step, then 31 decode steps; each path feeds back its own greedy tokens.
  * ours  -- one ``miniserve_b200.qwen3_attention.Qwen3Attention`` per layer over the B200 pool;
  * ref16 -- the reference's op sequence (the oracle's attention) in bf16 with PyTorch on the GPU;
  * ref32 -- the same in fp32, fed ref16's tokens: it measures each step's bf16 noise.
In bf16 a near-tie can go either way in any implementation, the reference's own included (its
logits are bf16 too, model/qwen3.py:155-158).  So, per sequence: ours must produce exactly
ref16's tokens, and if the two ever part, that step must be one ref16 itself cannot decide (its
top-1/top-2 margin within twice its distance to ref32).  The test reports every sequence's
agreeing run and the margins, and requires at least 48 of the 128 tokens to be compared on
decided steps (its power).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from miniserve_b200 import _capi
from miniserve_b200.attention import SeqChunk, build_attention_metadata
from miniserve_b200.kv_pool import allocate_kv_cache
from miniserve_b200.qwen3_attention import Qwen3Attention
from oracle import attention_oracle as orc
from qwen3_harness import QWEN3_06B, Qwen3Weights, forward, logits, oracle_attention

pytestmark = pytest.mark.gpu

BLOCK = 16
STEPS = 32
PROMPTS = (300, 100, 40, 5)
PROMPT_SEED = 6  # prompts and block tables; chosen so that two sequences stay decided throughout


class _Config:
    num_attention_heads = QWEN3_06B.heads
    num_key_value_heads = QWEN3_06B.kv_heads
    head_dim = QWEN3_06B.head_dim
    hidden_size = QWEN3_06B.hidden
    rms_norm_eps = QWEN3_06B.eps
    fused_qkv = False


def _modules(w: Qwen3Weights, dev: torch.device) -> list[Qwen3Attention]:
    mods = []
    for i in range(w.s.layers):
        m = Qwen3Attention(_Config()).to(device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            m.qkv_proj.weight.copy_(w.t[f"{i}.qkv"])
            m.o_proj.weight.copy_(w.t[f"{i}.o"])
            m.q_norm.weight.copy_(w.t[f"{i}.qn"])
            m.k_norm.weight.copy_(w.t[f"{i}.kn"])
        mods.append(m)
    return mods


def _forward_modules(w: Qwen3Weights, ids: torch.Tensor, mods, cos, sin, views, meta):
    """Qwen3ForCausalLM.forward (qwen3.py:140-153) with the drop-in attention module in every
    Qwen3DecoderLayer (qwen3.py:112-122)."""
    s, t = w.s, w.t
    x = t["embed"][ids]
    for i in range(s.layers):
        x = x + mods[i](orc.rms_norm(x, t[f"{i}.ln1"], s.eps), cos, sin, *views[i], meta)
        h = orc.rms_norm(x, t[f"{i}.ln2"], s.eps)
        gate, up = F.linear(h, t[f"{i}.gu"]).chunk(2, dim=-1)
        x = x + F.linear(F.silu(gate) * up, t[f"{i}.down"])
    return orc.rms_norm(x, t["norm"], s.eps)


@torch.no_grad()
def test_greedy_generation_feedback_matches_reference(cuda_device: torch.device) -> None:
    dev = cuda_device
    w = Qwen3Weights.random(QWEN3_06B, seed=0, dtype=torch.bfloat16, device=dev)
    w.t["embed"] = (w.t["embed"].float() * 2.5).bfloat16()  # logits spread like a trained model's
    w.t["lm_head"] = w.t["embed"]
    w32 = Qwen3Weights(w.s, {k: v.float() for k, v in w.t.items()})
    mods = _modules(w, dev)

    rng = np.random.default_rng(PROMPT_SEED)
    prompts = [rng.integers(0, w.s.vocab, size=n).tolist() for n in PROMPTS]
    num_blocks = 256
    perm = rng.permutation(num_blocks).tolist()
    tables, cur = [], 0
    for p in prompts:
        need = -(-(len(p) + STEPS + BLOCK) // BLOCK)
        tables.append(perm[cur : cur + need])
        cur += need
    cos_t, sin_t = orc.rope_tables(128, 1024, w.s.theta)
    _pool, views = allocate_kv_cache(w.s.layers, num_blocks, 8, dev)
    kv16 = [(torch.zeros(num_blocks * BLOCK, 8, 128, dtype=torch.bfloat16, device=dev),
             torch.zeros(num_blocks * BLOCK, 8, 128, dtype=torch.bfloat16, device=dev))
            for _ in range(w.s.layers)]
    kv32 = [(torch.zeros(num_blocks * BLOCK, 8, 128, device=dev),
             torch.zeros(num_blocks * BLOCK, 8, 128, device=dev)) for _ in range(w.s.layers)]

    def step_inputs(feed: list[list[int]], done: list[int]):
        ids, pos, slots, chunks = [], [], [], []
        for i, toks in enumerate(feed):
            flat = len(ids)
            ids.extend(toks)
            pos.extend(range(done[i], done[i] + len(toks)))
            slots.extend(tables[i][p // BLOCK] * BLOCK + p % BLOCK
                         for p in range(done[i], done[i] + len(toks)))
            chunks.append((flat, len(toks), done[i], tables[i]))
        last = torch.tensor(np.cumsum([len(t) for t in feed]) - 1, device=dev)
        return torch.tensor(ids, device=dev), torch.tensor(pos), torch.tensor(slots, device=dev), \
            chunks, last

    def run_ours(feed, done):
        ids, pos, slots, chunks, last = step_inputs(feed, done)
        meta = build_attention_metadata([SeqChunk(*c) for c in chunks], slots, BLOCK)
        h = _forward_modules(w, ids, mods, cos_t[pos].to(dev), sin_t[pos].to(dev), views, meta)
        return logits(w, h[last])

    def run_ref(wt, kv, feed, done):
        ids, pos, slots, chunks, last = step_inputs(feed, done)
        meta = orc.build_metadata([orc.SeqChunk(*c) for c in chunks], slots, BLOCK)
        h = forward(wt, ids, oracle_attention(wt, kv, meta, cos_t[pos].to(dev), sin_t[pos].to(dev)))
        return logits(wt, h[last])

    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    feed_ours = [list(p) for p in prompts]
    feed_ref = [list(p) for p in prompts]
    done = [0] * len(prompts)
    parted = [None] * len(prompts)  # step at which ours and ref16 first chose different tokens
    compared = [0] * len(prompts)  # tokens compared on decided steps before any parting
    min_ratio = float("inf")
    try:
        for s in range(STEPS):
            lo = run_ours(feed_ours, done)
            l16 = run_ref(w, kv16, feed_ref, done)
            l32 = run_ref(w32, kv32, feed_ref, done)
            for i, f in enumerate(feed_ref):
                done[i] += len(f)
            t_ours, t16 = lo.argmax(-1).tolist(), l16.argmax(-1).tolist()
            top2 = l16.topk(2, dim=-1).values
            margin = (top2[:, 0] - top2[:, 1]).tolist()
            noise = (2 * (l16 - l32).abs().amax(dim=-1)).tolist()
            for i in range(len(prompts)):
                if parted[i] is not None:
                    continue
                decided = margin[i] > noise[i]
                if t_ours[i] != t16[i]:
                    parted[i] = s
                    assert not decided, (
                        f"sequence {i}: ours chose {t_ours[i]}, ref16 {t16[i]} at step {s}, a step "
                        f"ref16 decides (margin {margin[i]:.4f} > noise {noise[i]:.4f})")
                elif decided:
                    compared[i] += 1
                    min_ratio = min(min_ratio, margin[i] / noise[i])
            # Each path continues with its own tokens; ref32 follows ref16.
            feed_ours = [[t] for t in t_ours]
            feed_ref = [[t] for t in t16]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = allow
    assert _capi.device_status(int(torch.cuda.current_stream(dev).cuda_stream)) == 0
    print(f"tokens compared on decided steps per sequence {compared} of {STEPS}; first parting "
          f"step per sequence {parted}; smallest decided margin / noise {min_ratio:.2f}")
    assert sum(compared) >= 48, "test lost its power: too few decided steps"
