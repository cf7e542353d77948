"""CPU oracle for MiniServe's per-step attention path.  TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, what MiniServe v0.5.0 computes for one decoder
layer between "qkv projected" and "attention output ready for o_proj", plus the once-per-step
batch metadata.  It is the checker for the CUDA path in ``miniserve_b200``: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``)
may import it.  Nothing in the product package imports or calls it.

Pinning: ``tests/golden/make_golden.py`` ran the reference's own functions (imported from its
source tree) on seeded inputs and stored the outputs as ``tests/golden/*.npz``;
``tests/test_oracle_golden.py`` checks this restatement against them, and
``tests/test_oracle_hf.py`` checks it end to end against Hugging Face's independent Qwen3
(the reference's own known-answer test, ``tests/correctness/test_model_vs_hf.py:17-43``).

Reference locations are ``path:line`` inside the MiniServe project:
  * ``src/miniserve/attention/backends.py`` -- metadata, scatter, gathered SDPA
  * ``src/miniserve/model/layers.py``       -- RMSNorm, RoPE tables, rotate-half RoPE
  * ``src/miniserve/model/qwen3.py``        -- the attention module's op order
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor

# backends.py:32-33 -- the two constants that decide grouping.
SHORT_QUERY = 8
MAX_GATHER_TOKENS = 16384


@dataclass
class SeqChunk:
    """One scheduled sequence as the attention sees it (backends.py:36-47)."""

    flat_start: int
    num_new: int
    num_cached: int
    block_table: list[int]

    @property
    def context_len(self) -> int:
        return self.num_cached + self.num_new


@dataclass
class OracleGroup:
    """A padded batch of short-query sequences (backends.py:50-56)."""

    q_index: Tensor  # [b, Q] int64
    valid_rows: Tensor | None  # [n] or None when every sequence has Q queries
    out_index: Tensor  # [n]
    ctx_slots: Tensor  # [b, L]
    mask: Tensor  # [b, Q, L] bool


@dataclass
class OraclePrefill:
    """One long query chunk (backends.py:59-64)."""

    q_start: int
    q_end: int
    ctx_slots: Tensor | None
    mask: Tensor | None


@dataclass
class OracleMeta:
    slot_mapping: Tensor
    groups: list[OracleGroup]
    prefills: list[OraclePrefill]


# ---------------------------------------------------------------------------------------------
# RMSNorm and RoPE (layers.py)
# ---------------------------------------------------------------------------------------------


def rope_tables(head_dim: int, max_positions: int, theta: float) -> tuple[Tensor, Tensor]:
    """fp32 cos/sin tables ``[max_positions, head_dim]`` (layers.py:43-50).

    Angle of (position t, pair i) is ``t * theta**(-2i/head_dim)``; the pair table is repeated
    twice along the last axis because the rotation pairs dimension i with i + head_dim/2.
    """
    half_exps = torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim
    inv_freq = 1.0 / (theta**half_exps)
    angles = torch.outer(torch.arange(max_positions, dtype=torch.float32), inv_freq)
    both = torch.cat((angles, angles), dim=-1)
    return both.cos(), both.sin()


def rms_norm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    """Per-row RMSNorm with the reference's rounding points (layers.py:18-22).

    fp32 mean of squares, ``rsqrt``, multiply, round back to ``x.dtype``, then multiply by the
    weight in the weight's / activation's dtype.
    """
    out_dtype = x.dtype
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return weight * (xf * inv).to(out_dtype)


def _rotate_half(x: Tensor) -> Tensor:
    lo, hi = x.chunk(2, dim=-1)
    return torch.cat((-hi, lo), dim=-1)


def apply_rope(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:
    """Rotate-half RoPE in the activation dtype (layers.py:56-65); cos/sin ``[T, head_dim]``."""
    c = cos.unsqueeze(1).to(q.dtype)
    s = sin.unsqueeze(1).to(q.dtype)
    return q * c + _rotate_half(q) * s, k * c + _rotate_half(k) * s


# ---------------------------------------------------------------------------------------------
# Metadata (backends.py:74-142) and the runner's slot arithmetic (model_runner.py:187-189)
# ---------------------------------------------------------------------------------------------


def slots_for(chunk: SeqChunk, block_size: int) -> list[int]:
    """KV slot of each new token: ``table[p // bs] * bs + p % bs`` (model_runner.py:189)."""
    t = chunk.block_table
    return [
        t[p // block_size] * block_size + p % block_size
        for p in range(chunk.num_cached, chunk.num_cached + chunk.num_new)
    ]


def prepare_step(scheduled: list[tuple[int, int, list[int]]], block_size: int
                 ) -> tuple[list[SeqChunk], list[int], list[int]]:
    """The attention inputs of ModelRunner.prepare (src/miniserve/runner/model_runner.py:
    162-205): flatten the scheduled sequences' tokens in batch order; each token's position in
    its own sequence (:185) and slot ``table[p // bs] * bs + p % bs`` (:187-188); one SeqChunk
    per sequence at its flat offset (:189).  ``scheduled`` holds ``(num_new, num_cached,
    block_table)``; token ids, logits rows and sampling are outside the attention path."""
    positions: list[int] = []
    slots: list[int] = []
    chunks: list[SeqChunk] = []
    for n, start, table in scheduled:
        flat = len(positions)
        positions.extend(range(start, start + n))
        slots.extend(table[p // block_size] * block_size + p % block_size
                     for p in range(start, start + n))
        chunks.append(SeqChunk(flat, n, start, list(table)))
    return chunks, positions, slots


def _page_lookup(tables: Tensor, length: int, block_size: int) -> Tensor:
    """Slot of every context position 0..length-1 through a table (backends.py:74-77)."""
    pos = torch.arange(length, device=tables.device)
    return tables[..., pos // block_size] * block_size + pos % block_size


def _short_group(chunks: list[SeqChunk], block_size: int, device: torch.device) -> OracleGroup:
    """Pad a set of short-query sequences into one batch (backends.py:101-132)."""
    q_len = max(c.num_new for c in chunks)
    n_blocks = -(-max(c.context_len for c in chunks) // block_size)
    padded_len = n_blocks * block_size
    tables = []
    for c in chunks:
        row = list(c.block_table[:n_blocks])
        tables.append(row + [0] * (n_blocks - len(row)))
    q_index, q_pos, out_index, valid = [], [], [], []
    for b, c in enumerate(chunks):
        q_index.append([c.flat_start + min(i, c.num_new - 1) for i in range(q_len)])
        q_pos.append([c.num_cached + min(i, c.num_new - 1) for i in range(q_len)])
        out_index.extend(c.flat_start + i for i in range(c.num_new))
        valid.extend(b * q_len + i for i in range(c.num_new))
    everyone_full = all(c.num_new == q_len for c in chunks)
    idx = dict(dtype=torch.long, device=device)
    key_pos = torch.arange(padded_len, device=device)
    qp = torch.tensor(q_pos, **idx)
    return OracleGroup(
        q_index=torch.tensor(q_index, **idx),
        valid_rows=None if everyone_full else torch.tensor(valid, **idx),
        out_index=torch.tensor(out_index, **idx),
        ctx_slots=_page_lookup(torch.tensor(tables, **idx), padded_len, block_size),
        mask=key_pos[None, None, :] <= qp[:, :, None],
    )


def _long_chunk(c: SeqChunk, block_size: int, device: torch.device) -> OraclePrefill:
    """A chunk with more than SHORT_QUERY queries (backends.py:135-142)."""
    end = c.flat_start + c.num_new
    if c.num_cached == 0:
        return OraclePrefill(c.flat_start, end, None, None)
    n_blocks = -(-c.context_len // block_size)
    table = torch.tensor(c.block_table[:n_blocks], dtype=torch.long, device=device)
    ctx = _page_lookup(table, c.context_len, block_size)
    mask = torch.ones(c.num_new, c.context_len, dtype=torch.bool, device=device).tril(c.num_cached)
    return OraclePrefill(c.flat_start, end, ctx, mask)


def build_metadata(chunks: list[SeqChunk], slot_mapping: Tensor, block_size: int) -> OracleMeta:
    """Group short rows longest-context-first under the gather cap (backends.py:80-98).

    Index tensors and masks live on the slot mapping's device, as in the reference."""
    device = slot_mapping.device
    short = sorted(
        (c for c in chunks if c.num_new <= SHORT_QUERY), key=lambda c: c.context_len, reverse=True
    )
    groups: list[OracleGroup] = []
    pending: list[SeqChunk] = []
    for c in short:
        if pending and (len(pending) + 1) * pending[0].context_len > MAX_GATHER_TOKENS:
            groups.append(_short_group(pending, block_size, device))
            pending = []
        pending.append(c)
    if pending:
        groups.append(_short_group(pending, block_size, device))
    longs = [_long_chunk(c, block_size, device) for c in chunks if c.num_new > SHORT_QUERY]
    return OracleMeta(slot_mapping, groups, longs)


# ---------------------------------------------------------------------------------------------
# Scatter + attention (backends.py:145-197)
# ---------------------------------------------------------------------------------------------


def paged_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    meta: OracleMeta,
    scale: float,
) -> Tensor:
    """Scatter this step's K/V into ``[slots, kv_heads, dim]`` caches, then attend.

    Same algorithm as backends.py:145-197: the scatter happens before any read; short rows are
    gathered per group with GQA folded into the query axis and a boolean mask; long chunks use
    repeated KV heads with causal SDPA (fresh prompt) or the shifted ``tril`` mask.
    """
    k_cache.index_copy_(0, meta.slot_mapping, k)
    v_cache.index_copy_(0, meta.slot_mapping, v)
    out = torch.empty_like(q)
    n_heads, n_kv, dim = q.shape[1], k.shape[1], q.shape[2]
    rep = n_heads // n_kv

    for g in meta.groups:
        b, ql = g.q_index.shape
        qg = q[g.q_index].view(b, ql, n_kv, rep, dim).permute(0, 2, 3, 1, 4)
        qg = qg.reshape(b, n_kv, rep * ql, dim)
        kg = k_cache[g.ctx_slots].transpose(1, 2)
        vg = v_cache[g.ctx_slots].transpose(1, 2)
        if ql == 1:
            m = g.mask.unsqueeze(1)
        else:
            m = g.mask.unsqueeze(1).expand(b, rep, ql, -1).reshape(b, 1, rep * ql, -1)
        og = F.scaled_dot_product_attention(qg, kg, vg, attn_mask=m, scale=scale)
        og = og.view(b, n_kv, rep, ql, dim).permute(0, 3, 1, 2, 4).reshape(b * ql, n_heads, dim)
        out[g.out_index] = og if g.valid_rows is None else og[g.valid_rows]

    for p in meta.prefills:
        qp = q[p.q_start : p.q_end].transpose(0, 1).unsqueeze(0)
        if p.ctx_slots is None:
            kp, vp = k[p.q_start : p.q_end], v[p.q_start : p.q_end]
        else:
            kp, vp = k_cache[p.ctx_slots], v_cache[p.ctx_slots]
        kp = kp.repeat_interleave(rep, dim=1).transpose(0, 1).unsqueeze(0)
        vp = vp.repeat_interleave(rep, dim=1).transpose(0, 1).unsqueeze(0)
        if p.mask is None:
            op = F.scaled_dot_product_attention(qp, kp, vp, is_causal=True, scale=scale)
        else:
            op = F.scaled_dot_product_attention(qp, kp, vp, attn_mask=p.mask, scale=scale)
        out[p.q_start : p.q_end] = op[0].transpose(0, 1)
    return out


def norm_rope(
    qkv: Tensor,
    q_weight: Tensor,
    k_weight: Tensor,
    eps: float,
    cos_rows: Tensor,
    sin_rows: Tensor,
    n_heads: int,
    n_kv: int,
    dim: int,
) -> tuple[Tensor, Tensor, Tensor]:
    """The attention module's pre-attention ops (qwen3.py:94-98): split, q/k norm, RoPE."""
    t = qkv.shape[0]
    q, k, v = qkv.split([n_heads * dim, n_kv * dim, n_kv * dim], dim=-1)
    q = rms_norm(q.reshape(t, n_heads, dim), q_weight, eps)
    k = rms_norm(k.reshape(t, n_kv, dim), k_weight, eps)
    v = v.reshape(t, n_kv, dim)
    q, k = apply_rope(q, k, cos_rows, sin_rows)
    return q, k, v


def attention_layer(
    qkv: Tensor,
    q_weight: Tensor,
    k_weight: Tensor,
    eps: float,
    cos: Tensor,
    sin: Tensor,
    positions: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    meta: OracleMeta,
    n_heads: int = 16,
    n_kv: int = 8,
    dim: int = 128,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """One layer of the path: returns ``(q_rotated, k_rotated, v, attention_out)``.

    ``cos``/``sin`` are the full fp32 tables; they are gathered by each token's own position
    the way ``Qwen3ForCausalLM.forward`` does once per step (qwen3.py:149).
    """
    q, k, v = norm_rope(
        qkv, q_weight, k_weight, eps, cos[positions], sin[positions], n_heads, n_kv, dim
    )
    out = paged_attention(q, k, v, k_cache, v_cache, meta, dim**-0.5)
    return q, k, v, out


# ---------------------------------------------------------------------------------------------
# A second, independent statement of the same attention (direct per-row loops), used to
# cross-check the gathered/grouped formulation above on small cases.
# ---------------------------------------------------------------------------------------------


def direct_attention(
    q: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    chunks: list[SeqChunk],
    block_size: int,
    scale: float,
) -> Tensor:
    """fp64 per-query attention over the context each query is allowed to see.

    Query i of a chunk sits at position ``num_cached + i`` and sees keys ``0..num_cached + i``
    (the mask rule of backends.py:123-125 and :140-142).  Rows not covered by a chunk are zero.
    """
    n_heads, dim = q.shape[1], q.shape[2]
    rep = n_heads // k_cache.shape[1]
    out = torch.zeros(q.shape, dtype=torch.float64)
    for c in chunks:
        ctx = _page_lookup(torch.tensor(c.block_table, dtype=torch.long), c.context_len, block_size)
        kk = k_cache[ctx].double()
        vv = v_cache[ctx].double()
        for i in range(c.num_new):
            vis = c.num_cached + i + 1
            for h in range(n_heads):
                s = (kk[:vis, h // rep] @ q[c.flat_start + i, h].double()) * scale
                w = torch.softmax(s, dim=0)
                out[c.flat_start + i, h] = w @ vv[:vis, h // rep]
    return out
