"""A CPU stand-in for libmsattn.so's device entry points (TEST INFRASTRUCTURE ONLY).

It lets the reference's own engine run on the CPU with the drop-in modules swapped in, so a test
can show that the reference's runner and model drive ``miniserve_b200`` correctly: the call
shapes, the arguments each C-ABI call receives, the pool layout and the plan's sequence records.
The host-only entry points (``ms_plan_build``, ``ms_plan_capacity``, ``ms_prepare_step``,
``ms_version``, ``ms_last_error``) are forwarded to the real library.  The device entry points
are replaced: they read and write the (host) memory behind the pointers they are given, doing
the reference's own math through the oracle (``oracle/attention_oracle.py``) in the pointers'
dtype -- kernel A as ``norm_rope`` + the pool scatter, the attention as ``paged_attention`` over
the sequences decoded from the packed plan.  Every call is recorded in ``calls``.

This checks the wiring, not the kernels; the kernels are checked on a B200 by the ``gpu`` tests.
"""

from __future__ import annotations

import ctypes as C
from typing import Any

import torch

from miniserve_b200 import _capi
from oracle import attention_oracle as orc

D = 128
BLOCK = 16
PAGE = BLOCK * D  # bf16 elements of one K (or V) page of one (block, head)

_CTYPES = {torch.bfloat16: C.c_uint16, torch.float32: C.c_float, torch.int64: C.c_int64,
           torch.int32: C.c_int32}


def host_tensor(ptr: int, count: int, dtype: torch.dtype) -> torch.Tensor:
    """A tensor over ``count`` elements of host memory at ``ptr`` (no copy)."""
    if not ptr:
        raise AssertionError("null pointer passed where the ABI needs one")
    return torch.frombuffer((_CTYPES[dtype] * count).from_address(ptr), dtype=dtype)


def rows(ptr: int, n: int, width: int, stride: int, dtype: torch.dtype) -> torch.Tensor:
    """``[n, width]`` rows ``stride`` elements apart."""
    if n == 0:
        return torch.empty(0, width, dtype=dtype)
    return host_tensor(ptr, (n - 1) * stride + width, dtype).as_strided((n, width), (stride, 1))


def layer_pool(k_cache: int, v_cache: int, num_blocks: int, kv_heads: int) -> torch.Tensor:
    """One layer's pool region ``[blocks, kv_heads, 2 (K, V), 2 (d // 64), 16, 64]``."""
    if v_cache != k_cache + 2 * PAGE:
        raise AssertionError("v_cache must be k_cache + 4 KiB (the pool's page-pair layout)")
    region = host_tensor(k_cache, num_blocks * kv_heads * 2 * PAGE, torch.bfloat16)
    return region.view(num_blocks, kv_heads, 2, 2, BLOCK, D // 2)


def scatter(pool: torch.Tensor, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """``k_cache.index_copy_(0, slots, k)`` and the same for v (backends.py:159-160), in the
    pool's layout."""
    t, kvh = k.shape[0], k.shape[1]
    b, o = slots // BLOCK, slots % BLOCK
    pool[b, :, 0, :, o, :] = k.reshape(t, kvh, 2, D // 2)
    pool[b, :, 1, :, o, :] = v.reshape(t, kvh, 2, D // 2)


def pool_as_slots(pool: torch.Tensor, which: int) -> torch.Tensor:
    """A copy of K (which=0) or V (1) in the reference layout ``[slots, kv_heads, 128]``."""
    nb, kvh = pool.shape[0], pool.shape[1]
    return pool[:, :, which].permute(0, 3, 1, 2, 4).reshape(nb * BLOCK, kvh, D).clone()


class EmulatedLib:
    def __init__(self) -> None:
        self._real = _capi.load()
        self.calls: list[tuple[str, dict[str, Any]]] = []

    # ---- host-only entry points: the real library -----------------------------------------
    def ms_version(self) -> int:
        return self._real.ms_version()

    def ms_last_error(self) -> bytes:
        return self._real.ms_last_error()

    def ms_plan_capacity(self, *a: Any) -> int:
        return self._real.ms_plan_capacity(*a)

    def ms_plan_build(self, *a: Any) -> int:
        rc = self._real.ms_plan_build(*a)
        self.calls.append(("ms_plan_build", {"num_seqs": a[0], "num_tokens": a[6], "rc": rc}))
        return rc

    def ms_prepare_step(self, *a: Any) -> int:
        return self._real.ms_prepare_step(*a)

    def ms_device_status(self, stream: Any, flags: Any, clear: int) -> int:
        flags._obj.value = 0
        return _capi.MS_OK

    # ---- device entry points: the reference's math on the host memory behind the pointers --
    def ms_qk_norm_rope_scatter(self, qkv, qkv_stride, t, h, kvh, q_w, k_w, eps, cos, sin,
                                cs_stride, positions, max_pos, slots, q_out, q_stride, k_cache,
                                v_cache, num_blocks, stream) -> int:
        width = (h + 2 * kvh) * D
        self.calls.append(("ms_qk_norm_rope_scatter", {
            "num_tokens": t, "num_heads": h, "num_kv_heads": kvh, "qkv_row_stride": qkv_stride,
            "q_out_row_stride": q_stride, "cs_row_stride": cs_stride, "eps": eps,
            "positions": positions is not None, "num_blocks": num_blocks}))
        if t == 0:
            return _capi.MS_OK
        x = rows(qkv, t, width, qkv_stride, torch.bfloat16).clone()
        qw = host_tensor(q_w, D, torch.bfloat16).clone()
        kw = host_tensor(k_w, D, torch.bfloat16).clone()
        if positions is not None:
            pos = host_tensor(positions, t, torch.int64)
            cos_r = rows(cos, max_pos, D, cs_stride, torch.float32)[pos]
            sin_r = rows(sin, max_pos, D, cs_stride, torch.float32)[pos]
        else:
            cos_r = rows(cos, t, D, cs_stride, torch.float32).clone()
            sin_r = rows(sin, t, D, cs_stride, torch.float32).clone()
        q, k, v = orc.norm_rope(x, qw, kw, eps, cos_r, sin_r, h, kvh, D)
        rows(q_out, t, h * D, q_stride, torch.bfloat16).copy_(q.reshape(t, h * D))
        sl = host_tensor(slots, t, torch.int64).clone()
        scatter(layer_pool(k_cache, v_cache, num_blocks, kvh), sl, k, v)
        return _capi.MS_OK

    def ms_kv_scatter(self, k, k_stride, v, v_stride, t, kvh, slots, k_cache, v_cache,
                      num_blocks, stream) -> int:
        self.calls.append(("ms_kv_scatter", {"num_tokens": t, "num_kv_heads": kvh}))
        if t == 0:
            return _capi.MS_OK
        kk = rows(k, t, kvh * D, k_stride, torch.bfloat16).reshape(t, kvh, D).clone()
        vv = rows(v, t, kvh * D, v_stride, torch.bfloat16).reshape(t, kvh, D).clone()
        sl = host_tensor(slots, t, torch.int64).clone()
        scatter(layer_pool(k_cache, v_cache, num_blocks, kvh), sl, kk, vv)
        return _capi.MS_OK

    def ms_paged_attention(self, q, q_stride, out, out_stride, h, kvh, k_cache, v_cache,
                           num_blocks, plan_dev, info_ref, workspace, ws_bytes, scale,
                           stream) -> int:
        info = info_ref._obj
        need = int(info.workspace_bytes_per_kv_head) * kvh
        if ws_bytes < need or (need > 0 and not workspace):
            raise AssertionError(f"workspace of {ws_bytes} bytes given, the plan needs {need}")
        plan = host_tensor(plan_dev, int(info.total_ints), torch.int32)
        recs = plan[info.off_seqs : info.off_seqs + 8 * info.num_seqs].view(-1, 8).tolist()
        chunks = [orc.SeqChunk(r[0], r[1], r[2],
                               plan[info.off_tables + r[4] : info.off_tables + r[4] + r[5]].tolist())
                  for r in recs]
        self.calls.append(("ms_paged_attention", {
            "num_tokens": int(info.num_tokens), "num_heads": h, "num_kv_heads": kvh,
            "num_seqs": int(info.num_seqs), "n_tc_items": int(info.n_tc_items),
            "n_tile_items": int(info.n_tile_items), "n_decode_items": int(info.n_decode_items),
            "n_cascade": int(info.n_cascade), "scale": scale, "chunks": chunks}))
        t = int(info.num_tokens)
        pool = layer_pool(k_cache, v_cache, num_blocks, kvh)
        ks, vs = pool_as_slots(pool, 0), pool_as_slots(pool, 1)
        slots = torch.tensor([s for c in chunks for s in orc.slots_for(c, BLOCK)], dtype=torch.long)
        flat = torch.tensor([c.flat_start + i for c in chunks for i in range(c.num_new)],
                            dtype=torch.long)
        if not torch.equal(flat, torch.arange(t)):
            raise AssertionError("the runner's flat batch is its sequences' tokens in order")
        qq = rows(q, t, h * D, q_stride, torch.bfloat16).reshape(t, h, D).clone()
        meta = orc.build_metadata(chunks, slots, BLOCK)
        # The pool already holds this step's K/V (kernel A or ms_kv_scatter wrote them), so the
        # oracle's own scatter rewrites the same values.
        o = orc.paged_attention(qq, ks[slots], vs[slots], ks, vs, meta, scale)
        rows(out, t, h * D, out_stride, torch.bfloat16).copy_(o.reshape(t, h * D))
        return _capi.MS_OK
