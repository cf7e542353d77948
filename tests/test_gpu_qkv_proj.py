"""Kernel E (qkv projection + kernel A's epilogue, one tcgen05 launch) against cuBLAS + kernel A.

The reference path for this op is `self.qkv_proj(x)` followed by split / q_norm / k_norm /
apply_rope (src/miniserve/model/qwen3.py:94-98) and the K/V scatter (backends.py:159-160).

Two kinds of inputs:
  * "exact": x and W hold small multiples of 1/4 and 1/8, so every fp32 partial sum of the
    projection is exact and any accumulation order gives the same bf16 output.  There kernel E
    must equal torch.matmul (cuBLAS) + kernel A bit for bit: q, the K rows and the V rows, and no
    pool slot outside slot_mapping may change.
  * "gaussian": ordinary random inputs.  The GEMM's accumulation order (kernel E's tcgen05
    tiles, split-K pairs for small steps, against cuBLAS) moves a few projection outputs by a
    bf16 ulp and, where the fp32 sum cancels, by more; RMSNorm and RoPE carry that into q and k.
    Bounds: every element within the order tolerance derived in `_order_tolerance`, 99.9 % of
    elements within one bf16 ulp, and both paths within a fixed distance of the fp32 CPU
    restatement of the whole op.
"""

from __future__ import annotations

import pytest
import torch

from gpu_harness import bf16_ulp_diff
from miniserve_b200 import _capi
from miniserve_b200.kv_pool import allocate_kv_cache, layer_as_slots
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter, qkv_proj_norm_rope_scatter
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

H, KVH, D, HIDDEN, EPS, THETA = 16, 8, 128, 1024, 1e-6, 1e6


def _inputs(t: int, kind: str, seed: int, num_blocks: int, max_pos: int = 4096):
    g = torch.Generator().manual_seed(seed)
    width = (H + 2 * KVH) * D
    if kind == "exact":
        x = torch.randint(-3, 4, (t, HIDDEN), generator=g).float() / 4
        w = torch.randint(-3, 4, (width, HIDDEN), generator=g).float() / 8
    else:
        x = torch.randn(t, HIDDEN, generator=g)
        w = torch.randn(width, HIDDEN, generator=g) / HIDDEN**0.5
    qw = 1 + 0.1 * torch.randn(D, generator=g)
    kw = 1 + 0.1 * torch.randn(D, generator=g)
    positions = torch.randint(0, max_pos, (t,), generator=g, dtype=torch.int64)
    slots = torch.randperm(num_blocks * 16, generator=g)[:t].to(torch.int64)
    return x.bfloat16(), w.bfloat16(), qw.bfloat16(), kw.bfloat16(), positions, slots


def _bf16_spacing(m: torch.Tensor) -> torch.Tensor:
    """The spacing of bf16 numbers at magnitude m: 2^(floor(log2 m) - 7)."""
    m = m.abs().clamp_min(2.0**-126)
    return torch.exp2(torch.floor(torch.log2(m)) - 7)


def _order_tolerance(x, w, qw, kw, positions, outs_a, outs_b):
    """Per-element bound on |a - b| between two implementations of the op that differ only in
    the projection's fp32 accumulation order (float64 tensors, [T, heads, D] for q, k, v).

    Two terms.  (1) The accumulation: any fp32 order of a K-term dot product of bf16 values is
    within K * 2^-24 * sum|x_i w_i| of the exact sum (K = 1024: 2^-14), tensor-core rounding
    included with a factor 2, and two orders are within twice that: 2^-12 * sum|x_i w_i|.  RMSNorm
    scales that error by rsqrt(mean p^2) * |weight|; RoPE combines two such errors with |cos| and
    |sin|.  (2) The rounding chain: a projection that moved by one ulp can flip the bf16 rounding
    of the norm (two roundings) and of RoPE's products and sum (layers.py:18-22, 56-65): 4 ulps
    at the largest operand of the last rounding (for RoPE the larger product; where the products
    cancel, that is far above the result's own spacing).  On the oracle itself, orders from 1 to
    1024 partial sums stay within 0.83 of this bound at 64 to 4096 tokens."""
    t = x.shape[0]
    xd, wd = x.double(), w.double()
    p = xd @ wd.t()
    err = 2.0**-12 * (xd.abs() @ wd.abs().t())
    cos_t, sin_t = orc.rope_tables(D, 4096, THETA)
    c = cos_t[positions].unsqueeze(1).double()
    sn = sin_t[positions].unsqueeze(1).double()
    sizes = [H * D, KVH * D, KVH * D]
    ps, es = p.split(sizes, dim=-1), err.split(sizes, dim=-1)
    bounds = []
    for i, (nh, wt) in enumerate(((H, qw), (KVH, kw))):
        pp, ee = ps[i].reshape(t, nh, D), es[i].reshape(t, nh, D)
        inv = torch.rsqrt(pp.pow(2).mean(-1, keepdim=True) + EPS)
        n = pp * inv * wt.double()
        en = ee * inv * wt.double().abs()
        lo, hi = n.chunk(2, dim=-1)
        rot = torch.cat((-hi, lo), dim=-1)
        elo, ehi = en.chunk(2, dim=-1)
        erot = torch.cat((ehi, elo), dim=-1)
        scale = torch.maximum(torch.maximum((n * c).abs(), (rot * sn).abs()),
                              torch.maximum(outs_a[i].abs(), outs_b[i].abs()))
        bounds.append(4 * _bf16_spacing(scale) + en * c.abs() + erot * sn.abs())
    v_scale = torch.maximum(outs_a[2].abs(), outs_b[2].abs())
    bounds.append(4 * _bf16_spacing(v_scale) + es[2].reshape(t, KVH, D))
    return bounds


def _run(path: str, x, w, qw, kw, positions, slots, num_blocks: int, device, positions_mode=False):
    cos_t, sin_t = orc.rope_tables(D, 4096, THETA)
    pool, views = allocate_kv_cache(1, num_blocks, KVH, device)
    pool.normal_(generator=torch.Generator(device=device).manual_seed(7))
    k_cache, v_cache = views[0]
    xd, wd = x.to(device), w.to(device)
    qwd, kwd = qw.to(device), kw.to(device)
    pos_d, slots_d = positions.to(device), slots.to(device)
    if positions_mode:
        cos, sin, pos_arg = cos_t.to(device), sin_t.to(device), pos_d
    else:
        cos, sin, pos_arg = cos_t[positions].to(device), sin_t[positions].to(device), None
    if path == "fused":
        q = qkv_proj_norm_rope_scatter(xd, wd, qwd, kwd, EPS, cos, sin, slots_d, k_cache, v_cache,
                                       H, positions=pos_arg)
    else:
        # cuBLAS, bf16 output (qwen3.py:94), with fp32 reductions throughout.
        flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        try:
            qkv = xd @ wd.t()
        finally:
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag
        q = qk_norm_rope_scatter(qkv, qwd, kwd, EPS, cos, sin, slots_d, k_cache, v_cache, H,
                                 positions=pos_arg)
    status = _capi.device_status(int(torch.cuda.current_stream(device).cuda_stream))
    return q, layer_as_slots(k_cache), layer_as_slots(v_cache), status


# 1, 77, 128 and 256 tokens run the split-K pairs (one-head tiles, two CTAs per tile), 300 the
# one-head-per-tile form; 1024, 2400 and 4096 the two-heads-per-tile form (2400 leaves a ragged
# last token block).
@pytest.mark.parametrize("t", [1, 77, 128, 256, 300, 1024, 2400, 4096])
def test_exact_inputs_bit_equal_to_cublas_plus_kernel_a(t: int, cuda_device) -> None:
    nb = (t + 15) // 16 + 8
    inp = _inputs(t, "exact", seed=t, num_blocks=nb)
    qa, ka, va, sa = _run("fused", *inp, nb, cuda_device)
    qb, kb, vb, sb = _run("cublas", *inp, nb, cuda_device)
    assert sa == 0 and sb == 0
    assert torch.equal(qa, qb)
    # Every slot: the written ones hold identical rows, the others the same untouched contents.
    assert torch.equal(ka, kb)
    assert torch.equal(va, vb)


@pytest.mark.parametrize("t", [64, 200, 2048, 4096])
def test_gaussian_inputs_within_stated_ulps(t: int, cuda_device) -> None:
    nb = (t + 15) // 16 + 8
    inp = _inputs(t, "gaussian", seed=100 + t, num_blocks=nb)
    x, w, qw, kw, positions, slots = inp
    qa, ka, va, sa = _run("fused", *inp, nb, cuda_device)
    qb, kb, vb, sb = _run("cublas", *inp, nb, cuda_device)
    assert sa == 0 and sb == 0
    s = slots.to(cuda_device)
    outs_a = [o.cpu().double() for o in (qa, ka[s], va[s])]
    outs_b = [o.cpu().double() for o in (qb, kb[s], vb[s])]
    bounds = _order_tolerance(x, w, qw, kw, positions, outs_a, outs_b)
    for name, a, b, bound in zip("qkv", outs_a, outs_b, bounds):
        ratio = (a - b).abs() / bound
        worst = int(ratio.argmax())
        assert ratio.max().item() <= 1.0, (
            f"{name}: |a - b| / bound = {ratio.max().item():.3f} at flat index {worst}: "
            f"{a.flatten()[worst].item()} vs {b.flatten()[worst].item()}")
        # Almost every element sits where the order does not matter: within one bf16 ulp.
        assert (bf16_ulp_diff(a.bfloat16(), b.bfloat16()) <= 1).float().mean().item() >= 0.999, name
    # Untouched slots stay untouched.
    mask = torch.ones(nb * 16, dtype=torch.bool, device=cuda_device)
    mask[s] = False
    assert torch.equal(ka[mask], kb[mask]) and torch.equal(va[mask], vb[mask])
    # Both paths against the fp32 CPU restatement of the op (projection in fp32, then the
    # reference's norm / RoPE rounding points): same bound for both.
    qkv32 = (x.float() @ w.float().t()).bfloat16()
    cos_t, sin_t = orc.rope_tables(D, 4096, THETA)
    q_ref, k_ref, _ = orc.norm_rope(qkv32, qw, kw, EPS, cos_t[positions], sin_t[positions], H,
                                    KVH, D)
    for got in (qa, qb):
        assert (got.cpu().float() - q_ref.float()).abs().max().item() <= 0.0625
    for got in (ka, kb):
        assert (got[s].cpu().float() - k_ref.float()).abs().max().item() <= 0.0625


def test_positions_mode_equals_gathered_rows(cuda_device) -> None:
    t, nb = 300, 40
    inp = _inputs(t, "gaussian", seed=5, num_blocks=nb)
    qa, ka, va, _ = _run("fused", *inp, nb, cuda_device, positions_mode=False)
    qb, kb, vb, _ = _run("fused", *inp, nb, cuda_device, positions_mode=True)
    assert torch.equal(qa, qb) and torch.equal(ka, kb) and torch.equal(va, vb)


def test_bad_slot_reported_and_row_skipped(cuda_device) -> None:
    """A slot outside the pool sets MS_DEV_BAD_SLOT and that token's K/V rows are not written;
    its query row and every other token are still produced."""
    t, nb = 40, 8
    x, w, qw, kw, positions, slots = _inputs(t, "exact", seed=9, num_blocks=nb)
    bad = slots.clone()
    bad[3] = nb * 16 + 5  # the kernel's own bounds check turns this into a status bit
    qa, ka, va, sa = _run("fused", x, w, qw, kw, positions, bad, nb, cuda_device)
    qb, kb, vb, sb = _run("cublas", x, w, qw, kw, positions, bad, nb, cuda_device)
    assert sa == _capi.DEV_BAD_SLOT and sb == _capi.DEV_BAD_SLOT
    assert torch.equal(qa, qb) and torch.equal(ka, kb) and torch.equal(va, vb)


def test_argument_checks(cuda_device) -> None:
    t, nb = 16, 4
    x, w, qw, kw, positions, slots = _inputs(t, "exact", seed=1, num_blocks=nb)
    pool, views = allocate_kv_cache(1, nb, KVH, cuda_device)
    cos_t, sin_t = orc.rope_tables(D, 4096, THETA)
    cos, sin = cos_t[positions].to(cuda_device), sin_t[positions].to(cuda_device)
    args = (qw.to(cuda_device), kw.to(cuda_device), EPS, cos, sin, slots.to(cuda_device),
            *views[0], H)
    with pytest.raises(ValueError):  # hidden mismatch between x and w
        qkv_proj_norm_rope_scatter(x[:, :512].contiguous().to(cuda_device), w.to(cuda_device), *args)
    with pytest.raises(ValueError):  # hidden not a multiple of 64 (rejected by the C ABI)
        qkv_proj_norm_rope_scatter(x[:, :1000].contiguous().to(cuda_device),
                                   w[:, :1000].contiguous().to(cuda_device), *args)


@pytest.mark.parametrize("kind", ["exact", "gaussian"])
def test_drop_in_module_fused_flag(kind: str, cuda_device) -> None:
    """Qwen3Attention (the reference's module shape) with fused_qkv on and off: equal outputs on
    exact inputs, within the stated tolerance on gaussian ones."""
    from types import SimpleNamespace

    from miniserve_b200.attention import SeqChunk, build_attention_metadata
    from miniserve_b200.qwen3_attention import Qwen3Attention

    t, nb = 300, 40
    x, w, qw, kw, positions, _ = _inputs(t, kind, seed=21, num_blocks=nb)
    positions = torch.arange(t)  # one sequence's prefill
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(3)).tolist()
    slots = torch.tensor([table[p // 16] * 16 + p % 16 for p in range(t)], dtype=torch.int64)
    cos_t, sin_t = orc.rope_tables(D, 4096, THETA)
    cos, sin = cos_t[positions].to(cuda_device), sin_t[positions].to(cuda_device)
    outs = []
    for fused in (False, True):
        cfg = SimpleNamespace(num_attention_heads=H, num_key_value_heads=KVH, head_dim=D,
                              hidden_size=HIDDEN, rms_norm_eps=EPS, fused_qkv=fused)
        mod = Qwen3Attention(cfg).to(device=cuda_device, dtype=torch.bfloat16)
        with torch.no_grad():
            mod.qkv_proj.weight.copy_(w)
            mod.o_proj.weight.copy_(
                (torch.randn(HIDDEN, H * D, generator=torch.Generator().manual_seed(4)) / 64).bfloat16())
            mod.q_norm.weight.copy_(qw)
            mod.k_norm.weight.copy_(kw)
        pool, views = allocate_kv_cache(1, nb, KVH, cuda_device)
        slot_d = slots.to(cuda_device)
        meta = build_attention_metadata([SeqChunk(0, t, 0, table)], slot_d, 16)
        flag = torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction
        torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
        try:
            with torch.no_grad():
                outs.append(mod(x.to(cuda_device), cos, sin, *views[0], meta))
        finally:
            torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = flag
        assert _capi.device_status(int(torch.cuda.current_stream(cuda_device).cuda_stream)) == 0
    if kind == "exact":
        assert torch.equal(outs[0], outs[1])
    else:
        ulps = bf16_ulp_diff(outs[0], outs[1])
        assert (ulps <= 2).float().mean().item() >= 0.99
        assert (outs[0].float() - outs[1].float()).abs().max().item() <= 0.05
