"""The allocation-free attention entry point, ms_paged_attention_noalloc.

It exists for callers that cannot call cudaMalloc (a host engine that owns all GPU memory
through its own arena, a custom-op interface with no allocator, a loop that cannot afford
cudaMalloc's implicit synchronisation).  Instead of a caller-provided workspace it keeps the
split-KV partials in a fixed 16 MiB array built into the library.  These tests call it through
the C ABI with ctypes and compare it with the regular entry point, ms_paged_attention, on a plan
that splits almost every tile (so the scratch is really used), twice in a row (the second call
runs over the first call's leftovers).  Both run the same kernels on the same plan, so their rows
must be bit-identical; the regular entry point is itself checked against the fp32 oracle.  They
also check that a plan too big for the array is refused before anything is launched.

This file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from golden.cases import EPS, H, THETA
from golden_io import make_inputs
from gpu_harness import covered_rows, setup_pool
from miniserve_b200 import _capi
from miniserve_b200.attention import attend, build_attention_metadata, plan_batch
from miniserve_b200.kv_pool import layer_as_slots
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter
from miniserve_b200.workloads import custom
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

ATOL = 2e-2  # the attention tolerance used by the other parity tests
SCRATCH_BYTES = 16 * 1024 * 1024


def _fp32_oracle_out(inp, q: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor) -> torch.Tensor:
    """The oracle's attention in fp32 over the bf16 queries and pool the kernels read."""
    ks = layer_as_slots(k_cache).float().cpu()
    vs = layer_as_slots(v_cache).float().cpu()
    slots = torch.from_numpy(inp.batch.slots)
    chunks = [orc.SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table))
              for c in inp.batch.chunks]
    meta = orc.build_metadata(chunks, slots, 16)
    return orc.paged_attention(q.float().cpu(), ks[slots], vs[slots], ks, vs, meta, 128**-0.5)


def _noalloc(q: torch.Tensor, out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
             meta, scale: float) -> int:
    lib = _capi.load()
    stream = int(torch.cuda.current_stream(q.device).cuda_stream)
    return lib.ms_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), q.shape[1], k_cache.shape[1],
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], meta.plan.data_ptr(),
        C.byref(meta.info), float(scale), stream,
    )


def test_noalloc_matches_workspace_entry_point_twice(cuda_device: torch.device) -> None:
    inp = make_inputs("mixed_bf16")
    b = inp.batch
    _pool, k_cache, v_cache = setup_pool(inp, cuda_device)
    cos_t, sin_t = orc.rope_tables(128, inp.max_positions, THETA)
    pos = torch.from_numpy(b.positions)
    slots = torch.from_numpy(b.slots).to(cuda_device)
    q = qk_norm_rope_scatter(
        inp.qkv.to(cuda_device), inp.q_weight.to(cuda_device), inp.k_weight.to(cuda_device), EPS,
        cos_t[pos].to(cuda_device), sin_t[pos].to(cuda_device), slots, k_cache, v_cache, H,
    )
    meta = build_attention_metadata(b.chunks, slots, 16, pages_per_split=2)
    assert meta.info.n_combine > 0, "the case must exercise split-KV partials"
    need = meta.info.workspace_bytes_per_kv_head * k_cache.shape[1]
    assert 0 < need <= SCRATCH_BYTES
    scale = 128**-0.5

    expected = attend(q, k_cache, v_cache, meta, scale)
    rows = covered_rows(inp).to(cuda_device)
    # The regular entry point against the fp32 oracle on the same bf16 queries and pool, so the
    # exact comparisons below compare with a checked result.
    ref32 = _fp32_oracle_out(inp, q, k_cache, v_cache)
    err32 = (expected[rows].float().cpu() - ref32[rows.cpu()]).abs().max().item()
    assert err32 <= ATOL, err32
    for call in range(2):
        got = torch.full_like(q, float("nan"))
        rc = _noalloc(q, got, k_cache, v_cache, meta, scale)
        _capi.check(rc, "ms_paged_attention_noalloc")
        torch.cuda.synchronize(cuda_device)
        assert _capi.device_status(int(torch.cuda.current_stream(cuda_device).cuda_stream)) == 0
        # Same kernels on the same plan, only the scratch differs: bit-identical rows.
        assert torch.equal(got[rows], expected[rows]), call


def test_noalloc_rejects_plans_larger_than_its_scratch(cuda_device: torch.device) -> None:
    # 24 sequences of 4000 cached tokens split into one-page ranges: about 24 * 251 * 2 partial
    # rows * 8 heads * 516 B = 50 MB of partials, more than the 16 MiB array.
    b = custom([(1, 4000)] * 24, seed=3)
    packed, info = plan_batch(b.chunks, b.num_tokens, 16, 148, 1)
    assert info.workspace_bytes_per_kv_head * 8 > SCRATCH_BYTES
    _pool, k_cache, v_cache = setup_pool(make_inputs("mixed_bf16"), cuda_device)
    plan_dev = torch.from_numpy(packed).to(cuda_device)
    q = torch.zeros(b.num_tokens, H, 128, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty_like(q)
    lib = _capi.load()
    rc = lib.ms_paged_attention_noalloc(
        q.data_ptr(), q.stride(0), out.data_ptr(), out.stride(0), H, 8, k_cache.data_ptr(),
        v_cache.data_ptr(), k_cache.shape[0], plan_dev.data_ptr(), C.byref(info), 0.1,
        int(torch.cuda.current_stream(cuda_device).cuda_stream),
    )
    assert rc == _capi.MS_ERR_CAPACITY
    assert b"built-in scratch" in lib.ms_last_error()
