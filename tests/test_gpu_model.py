"""Greedy-token identity over a full forward (Qwen3-0.6B shapes, 28 layers, seeded random
weights; real weights are not available offline).

Three engine-like steps over four sequences exercise every kernel: fresh prefills of 300 and 100
tokens (tensor-core kernel), a 40-token prompt (tile kernel), a 5-token prompt (decode kernel);
then a 300-token decode, an 80-token chunk over 100 cached tokens, a decode, and a 5-token
speculative verify; then decodes.  Three paths run the same weights and tokens:
  * ref32 -- the reference's op sequence (the oracle's attention) with everything in fp32;
  * ref16 -- the same in bf16, as MiniServe runs on a GPU (PyTorch ops on CUDA);
  * ours  -- bf16, kernel A + kernels B/C/D through the C ABI over the B200 pool (parametrized:
             the qkv projection by cuBLAS then kernel A, or kernel E doing both).
All paths are fed the fp32 reference's greedy tokens, and the argmax of every row of every step
is compared (about 535 rows).  In bf16 a near-tie can flip in any implementation, the reference's
own included, so the bar is: ours picks the same token as ref16 on every row whose ref16
top-1/top-2 margin exceeds that row's own bf16 noise (twice its largest |ref16 - ref32| logit
difference); ours is no further from ref32 than ref16 is (mean logit error within 25%); and ours
agrees with ref32 on as many rows as ref16 does within 2.5% of the rows (about 2.4 standard
deviations of the near-tie flip count; measured 516 vs 524 of 535 with equal per-layer error).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from miniserve_b200.attention import SeqChunk, attend, build_attention_metadata
from miniserve_b200.kv_pool import allocate_kv_cache
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter, qkv_proj_norm_rope_scatter
from oracle import attention_oracle as orc
from qwen3_harness import QWEN3_06B, Qwen3Weights, forward, logits, oracle_attention

pytestmark = pytest.mark.gpu

BLOCK = 16


class Seq:
    def __init__(self, prompt: list[int], table: list[int]) -> None:
        self.tokens = list(prompt)
        self.prompt_len = len(prompt)
        self.done = 0  # tokens already in the KV cache
        self.table = table


def _run_step(w, w32, plan, seqs, ref_kv, ref32_kv, pool_views, cos_t, sin_t, dev, fused_qkv):
    """plan: list of (seq index, tokens to feed).  Returns (ref32, ref16, ours) logits of all rows."""
    s = w.s
    chunks_ref, chunks_ours, ids, pos, slots = [], [], [], [], []
    for si, toks in plan:
        q = seqs[si]
        flat = len(ids)
        ids.extend(toks)
        pos.extend(range(q.done, q.done + len(toks)))
        slots.extend(q.table[p // BLOCK] * BLOCK + p % BLOCK for p in range(q.done, q.done + len(toks)))
        chunks_ref.append(orc.SeqChunk(flat, len(toks), q.done, q.table))
        chunks_ours.append(SeqChunk(flat, len(toks), q.done, q.table))
    ids_t = torch.tensor(ids, device=dev)
    pos_t = torch.tensor(pos)
    slot_t = torch.tensor(slots, device=dev)
    cos_rows, sin_rows = cos_t[pos_t].to(dev), sin_t[pos_t].to(dev)

    meta_ref = orc.build_metadata(chunks_ref, slot_t, BLOCK)
    ref_hidden = forward(w, ids_t, oracle_attention(w, ref_kv, meta_ref, cos_rows, sin_rows))
    ref32_hidden = forward(w32, ids_t, oracle_attention(w32, ref32_kv, meta_ref, cos_rows, sin_rows))

    meta = build_attention_metadata(chunks_ours, slot_t, BLOCK)

    def ours(i: int, att_in: torch.Tensor) -> torch.Tensor:
        kc, vc = pool_views[i]
        if fused_qkv:  # att_in = normalised hidden states; kernel E does the projection
            q = qkv_proj_norm_rope_scatter(att_in, w.t[f"{i}.qkv"], w.t[f"{i}.qn"], w.t[f"{i}.kn"],
                                           s.eps, cos_rows, sin_rows, slot_t, kc, vc, s.heads)
        else:  # att_in = the projection output (cuBLAS); kernel A
            q = qk_norm_rope_scatter(att_in, w.t[f"{i}.qn"], w.t[f"{i}.kn"], s.eps, cos_rows,
                                     sin_rows, slot_t, kc, vc, s.heads)
        return attend(q, kc, vc, meta, s.head_dim**-0.5).reshape(len(ids), s.heads * s.head_dim)

    our_hidden = forward(w, ids_t, ours, from_hidden=fused_qkv)
    for si, toks in plan:
        seqs[si].done += len(toks)
    return logits(w32, ref32_hidden), logits(w, ref_hidden), logits(w, our_hidden)


@torch.no_grad()
@pytest.mark.parametrize("fused_qkv", [False, True], ids=["cublas_qkv+kernel_a", "kernel_e"])
def test_greedy_tokens_identical_full_forward(fused_qkv: bool, cuda_device: torch.device) -> None:
    dev = cuda_device
    w = Qwen3Weights.random(QWEN3_06B, seed=0, dtype=torch.bfloat16, device=dev)
    w.t["embed"] = (w.t["embed"].float() * 2.5).bfloat16()  # logits spread like a trained model's
    w.t["lm_head"] = w.t["embed"]
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 151936, size=n).tolist() for n in (300, 180, 40, 5)]
    num_blocks = 128
    perm = rng.permutation(num_blocks).tolist()
    seqs, cur = [], 0
    for p in prompts:
        need = -(-(len(p) + 16) // BLOCK)
        seqs.append(Seq(p, perm[cur : cur + need]))
        cur += need
    w32 = Qwen3Weights(w.s, {k: v.float() for k, v in w.t.items()})
    ref_kv = [(torch.zeros(num_blocks * BLOCK, 8, 128, dtype=torch.bfloat16, device=dev),
               torch.zeros(num_blocks * BLOCK, 8, 128, dtype=torch.bfloat16, device=dev))
              for _ in range(w.s.layers)]
    ref32_kv = [(torch.zeros(num_blocks * BLOCK, 8, 128, device=dev),
                 torch.zeros(num_blocks * BLOCK, 8, 128, device=dev)) for _ in range(w.s.layers)]
    _pool, views = allocate_kv_cache(w.s.layers, num_blocks, 8, dev)
    cos_t, sin_t = orc.rope_tables(128, 1024, w.s.theta)

    rows_all = []  # (ref32, ref16, ours) logits of every checked row

    def compare(res, rows: list[int]) -> list[int]:
        r32, r16, o = (x[rows] for x in res)
        rows_all.append((r32, r16, o))
        return r32.argmax(-1).tolist()

    def run(plan):
        return _run_step(w, w32, plan, seqs, ref_kv, ref32_kv, views, cos_t, sin_t, dev, fused_qkv)

    # step 1: prefills (B only its first 100 tokens)
    plan = [(0, prompts[0]), (1, prompts[1][:100]), (2, prompts[2]), (3, prompts[3])]
    res = run(plan)
    offs = np.cumsum([0] + [len(t) for _, t in plan])
    last = [int(offs[1]) - 1, int(offs[3]) - 1, int(offs[4]) - 1]  # last rows of A, C, D
    nxt = [res[0][i].argmax().item() for i in last]
    compare(res, list(range(int(offs[-1]))))
    # step 2: A decode, B 80-token chunk over its cache, C decode, D 5-token verify
    drafts = rng.integers(0, 151936, size=4).tolist()
    plan = [(0, [nxt[0]]), (1, prompts[1][100:]), (2, [nxt[1]]), (3, [nxt[2], *drafts])]
    res = run(plan)
    step2 = [res[0][i].argmax().item() for i in (0, 80, 81)]  # A, B's last prompt row, C
    compare(res, list(range(87)))
    # step 3: decodes for A, B, C
    compare(run([(0, [step2[0]]), (1, [step2[1]]), (2, [step2[2]])]), [0, 1, 2])

    r32 = torch.cat([x[0] for x in rows_all])
    r16 = torch.cat([x[1] for x in rows_all])
    ours = torch.cat([x[2] for x in rows_all])
    noise = 2 * (r16 - r32).abs().amax(dim=-1)  # per row
    top2 = r16.topk(2, dim=-1).values
    margin = top2[:, 0] - top2[:, 1]
    t32, t16, tours = r32.argmax(-1), r16.argmax(-1), ours.argmax(-1)
    decided = margin > noise
    n = len(t32)
    agree32, ref_agree32 = int((tours == t32).sum()), int((t16 == t32).sum())
    print(f"rows {n}: ours==ref16 {int((tours == t16).sum())}, ours==ref32 {agree32}, "
          f"ref16==ref32 {ref_agree32}; rows decided beyond bf16 noise {int(decided.sum())}, "
          f"ours==ref16 on those {int((tours == t16)[decided].sum())}; max |ours-ref32| "
          f"{(ours - r32).abs().max().item():.4f}, max |ref16-ref32| {(r16 - r32).abs().max().item():.4f}")
    assert n == 535
    assert int(decided.sum()) >= n // 2, "test lost its power: too few decided rows"
    assert bool((tours == t16)[decided].all()), "a token flipped on a row decided beyond bf16 noise"
    mean_ours = (ours - r32).abs().mean().item()
    mean_ref = (r16 - r32).abs().mean().item()
    print(f"mean |ours-ref32| {mean_ours:.5f}, mean |ref16-ref32| {mean_ref:.5f}")
    assert mean_ours <= 1.25 * mean_ref
    assert agree32 >= ref_agree32 - (25 * n) // 1000
