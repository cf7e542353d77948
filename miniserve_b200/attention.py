"""Drop-in replacement for MiniServe's attention backend (src/miniserve/attention/backends.py).

Same names and call shapes as the reference module:

* ``SeqChunk(flat_start, num_new, num_cached, block_table)``            (backends.py:36-47)
* ``build_attention_metadata(chunks, slot_mapping, block_size)``       (backends.py:80-98)
* ``paged_attention(q, k, v, k_cache, v_cache, meta, scale) -> [T, H, D]`` (backends.py:145-197)
* ``SHORT_QUERY`` and ``MAX_GATHER_TOKENS`` (backends.py:32-33; the runner's profiler imports the
  latter, model_runner.py:21,111).

What changes underneath: the metadata is one packed int32 plan built by the native planner and
uploaded with a single pinned, non-blocking copy; the KV pool uses the layout of
``miniserve_b200.kv_pool``; the scatter and the attention are hand-written sm_100a kernels that
read the pool in place (no gather copy, no padding, no masks in memory).  Everything runs on the
caller's current CUDA stream and never synchronises; errors surface as ``ValueError`` /
``RuntimeError`` like the reference's.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from itertools import chain

import numpy as np
import torch
from torch import Tensor

from . import _capi
from .kv_pool import BLOCK_SIZE, HEAD_DIM, check_layer_views

SHORT_QUERY = 8  # rows with at most this many new tokens take the decode kernel
MAX_GATHER_TOKENS = 16384  # kept for the runner's profiler; nothing is gathered here


@dataclass
class SeqChunk:
    """What attention needs to know about one scheduled sequence (backends.py:36-47)."""

    flat_start: int  # where its new tokens start in the flattened batch
    num_new: int  # new tokens this step (its queries)
    num_cached: int  # tokens already in the KV cache before this step
    block_table: list[int]

    @property
    def context_len(self) -> int:
        return self.num_cached + self.num_new


@dataclass
class AttentionMetadata:
    """The per-step plan, built once and shared by every layer (backends.py:67-71)."""

    slot_mapping: Tensor  # [T] int64 slot of each new token, on the device
    plan: Tensor  # packed int32 plan on the device
    info: _capi.MsPlanInfo  # host-side description of the plan
    num_tokens: int
    _workspace: dict[tuple[int, int], Tensor] = field(default_factory=dict, repr=False)
    _num_sms: int = field(default=148, repr=False)
    _pages_per_split: int = field(default=0, repr=False)

    def update(self, chunks: list[SeqChunk], slot_mapping: Tensor | None = None) -> bool:
        """Plan a new step into this metadata's device buffers, for CUDA-graph replay.

        A graph captured over calls that use this metadata keeps the addresses of its plan and
        slot mapping and the launch shapes derived from ``info`` (grid sizes, section offsets,
        workspace size).  When the new step's plan has the same shape (same item counts, offsets
        and split workspace: for example, the same batch again, or contexts that grew inside their
        last pages), its plan and, if given, its slot mapping are copied into the existing buffers
        on the current stream (after the work already queued there, so no kernel of the previous
        step sees them) and True is returned.  Otherwise nothing changes and False is returned:
        build new metadata and capture again.  No reference counterpart (MiniServe captures no
        graphs).
        """
        if slot_mapping is not None and tuple(slot_mapping.shape) != tuple(self.slot_mapping.shape):
            return False
        packed, info = plan_batch(chunks, self.num_tokens, BLOCK_SIZE, self._num_sms,
                                  self._pages_per_split)
        if not same_launch_shape(info, self.info):
            return False
        self.plan.copy_(torch.from_numpy(packed).pin_memory(), non_blocking=True)
        if slot_mapping is not None and slot_mapping.data_ptr() != self.slot_mapping.data_ptr():
            self.slot_mapping.copy_(slot_mapping, non_blocking=True)
        return True

    def workspace(self, num_kv_heads: int, device: torch.device) -> Tensor | None:
        """Split-KV scratch for this step (allocated once, reused by every layer)."""
        need = int(self.info.workspace_bytes_per_kv_head) * num_kv_heads
        if need == 0:
            return None
        key = (str(device), num_kv_heads)  # a tensor's device always carries its index
        ws = self._workspace.get(key)
        if ws is None:
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            self._workspace[key] = ws
        return ws


_SM_COUNT: dict[int, int] = {}


def _num_sms(device: torch.device) -> int:
    if device.type != "cuda":
        raise RuntimeError("miniserve_b200 attention runs on CUDA only (no CPU fallback)")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


def plan_batch(
    chunks: list[SeqChunk],
    num_tokens: int,
    block_size: int = BLOCK_SIZE,
    num_sms: int = 148,
    pages_per_split: int = 0,
) -> tuple[np.ndarray, _capi.MsPlanInfo]:
    """Run the native planner on the host; returns ``(packed int32 plan, info)``."""
    lib = _capi.load()
    n = len(chunks)
    flat = np.fromiter((c.flat_start for c in chunks), dtype=np.int32, count=n)
    new = np.fromiter((c.num_new for c in chunks), dtype=np.int32, count=n)
    cached = np.fromiter((c.num_cached for c in chunks), dtype=np.int32, count=n)
    lens = np.fromiter((len(c.block_table) for c in chunks), dtype=np.int64, count=n)
    offsets = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    total = int(offsets[-1])
    tables = np.fromiter(chain.from_iterable(c.block_table for c in chunks), dtype=np.int32,
                         count=total)
    cap = int(lib.ms_plan_capacity(n, num_tokens, total))
    out = np.empty(cap, dtype=np.int32)
    info = _capi.MsPlanInfo()
    rc = lib.ms_plan_build(
        n, flat.ctypes.data, new.ctypes.data, cached.ctypes.data, offsets.ctypes.data,
        tables.ctypes.data if total else None, num_tokens, block_size, num_sms, pages_per_split,
        out.ctypes.data, cap, C.byref(info),
    )
    _capi.check(rc, "build_attention_metadata")
    return out[: info.total_ints], info


def prepare_arrays(num_new: np.ndarray, num_cached: np.ndarray, table_offsets: np.ndarray,
                   tables: np.ndarray, positions_out: np.ndarray, slots_out: np.ndarray
                   ) -> tuple[np.ndarray, int]:
    """``ms_prepare_step`` over CSR arrays (int32 num_new / num_cached / tables, int64
    table_offsets of length n + 1) into caller buffers (contiguous int64, e.g. pinned host
    memory).  Returns ``(flat_start int32, num_tokens)``."""
    lib = _capi.load()
    n = int(num_new.shape[0])
    for arr, dt, name in ((num_new, np.int32, "num_new"), (num_cached, np.int32, "num_cached"),
                          (table_offsets, np.int64, "table_offsets"), (tables, np.int32, "tables"),
                          (positions_out, np.int64, "positions_out"),
                          (slots_out, np.int64, "slots_out")):
        if arr.dtype != dt or not arr.flags.c_contiguous:
            raise ValueError(f"{name} must be a contiguous {np.dtype(dt).name} array")
    if num_cached.shape[0] != n or table_offsets.shape[0] != n + 1:
        raise ValueError("num_cached / table_offsets do not match num_new")
    tokens = int(num_new.sum(dtype=np.int64))
    if positions_out.shape[0] < tokens or slots_out.shape[0] < tokens:
        raise ValueError(f"positions_out / slots_out must be contiguous int64 arrays of >= {tokens} "
                         "elements")
    flat = np.empty(n, dtype=np.int32)
    got = C.c_int32(0)
    rc = lib.ms_prepare_step(
        n, num_new.ctypes.data, num_cached.ctypes.data, table_offsets.ctypes.data,
        tables.ctypes.data if tables.size else None, BLOCK_SIZE, flat.ctypes.data,
        positions_out.ctypes.data, slots_out.ctypes.data,
        min(positions_out.shape[0], slots_out.shape[0]), C.byref(got))
    _capi.check(rc, "prepare_step")
    return flat, got.value


def prepare_step(
    scheduled: list[tuple[int, int, list[int]]],
    *,
    positions_out: np.ndarray | None = None,
    slots_out: np.ndarray | None = None,
) -> tuple[list[SeqChunk], np.ndarray, np.ndarray]:
    """The attention inputs of ``ModelRunner.prepare`` (model_runner.py:162-205) in one native
    pass (``ms_prepare_step``).  ``scheduled`` holds ``(num_new, num_cached, block_table)`` per
    sequence in batch order; returns ``(chunks, positions, slot_mapping)`` with int64 positions
    and slots (``table[p // 16] * 16 + p % 16``) in flat-batch order.  Optional ``*_out`` arrays
    (int64, e.g. views of pinned host tensors) receive the results without new allocations."""
    n = len(scheduled)
    new = np.fromiter((s[0] for s in scheduled), dtype=np.int32, count=n)
    cached = np.fromiter((s[1] for s in scheduled), dtype=np.int32, count=n)
    lens = np.fromiter((len(s[2]) for s in scheduled), dtype=np.int64, count=n)
    offsets = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    total = int(offsets[-1])
    tables = np.fromiter(chain.from_iterable(s[2] for s in scheduled), dtype=np.int32, count=total)
    tokens = int(new.sum(dtype=np.int64))
    positions = positions_out if positions_out is not None else np.empty(tokens, dtype=np.int64)
    slots = slots_out if slots_out is not None else np.empty(tokens, dtype=np.int64)
    flat, got = prepare_arrays(new, cached, offsets, tables, positions, slots)
    chunks = [SeqChunk(int(flat[i]), int(new[i]), int(cached[i]), list(scheduled[i][2]))
              for i in range(n)]
    return chunks, positions[:got], slots[:got]


def build_attention_metadata(
    chunks: list[SeqChunk],
    slot_mapping: Tensor,
    block_size: int,
    *,
    pages_per_split: int = 0,
) -> AttentionMetadata:
    """Plan one step and upload it (one pinned H2D copy, no sync).  backends.py:80-98."""
    device = slot_mapping.device
    num_sms = _num_sms(device)  # raises for a non-CUDA device: there is no CPU path
    if block_size != BLOCK_SIZE:
        raise ValueError(f"block_size must be {BLOCK_SIZE}")
    num_tokens = int(slot_mapping.shape[0])
    packed, info = plan_batch(chunks, num_tokens, block_size, num_sms, pages_per_split)
    plan = _upload_plan(packed, device)
    slots = slot_mapping if slot_mapping.dtype == torch.int64 else slot_mapping.to(torch.int64)
    return AttentionMetadata(slots.contiguous(), plan, info, num_tokens,
                             _num_sms=num_sms, _pages_per_split=pages_per_split)


def same_launch_shape(a: _capi.MsPlanInfo, b: _capi.MsPlanInfo) -> bool:
    """Whether two plans launch the same kernels with the same arguments apart from the plan's
    contents: every field of the plan description is equal except the total page count (a
    statistic no launch reads)."""
    return all(getattr(a, name) == getattr(b, name)
               for name, _ in _capi.MsPlanInfo._fields_
               if name not in ("total_pages", "reserved"))


def _upload_plan(packed: np.ndarray, device: torch.device) -> Tensor:
    """The step's one host-to-device copy: the packed plan, through pinned memory, non-blocking
    (the reference's ``to_device``, utils.py:11-20)."""
    return torch.from_numpy(packed).pin_memory().to(device, non_blocking=True)


def _stream(device: torch.device) -> int:
    return int(torch.cuda.current_stream(device).cuda_stream)


def _rows(t: Tensor, name: str) -> int:
    """Row stride (elements) of a [T, heads, 128] tensor whose heads are packed in each row."""
    if t.dim() != 3 or t.shape[2] != HEAD_DIM or t.stride(2) != 1 or t.stride(1) != HEAD_DIM:
        raise ValueError(f"{name} must be [T, heads, {HEAD_DIM}] with contiguous heads")
    if t.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be bf16")
    return int(t.stride(0))


def kv_scatter(k: Tensor, v: Tensor, slot_mapping: Tensor, k_cache: Tensor, v_cache: Tensor) -> None:
    """Write this step's K/V rows into their slots (backends.py:159-160)."""
    nb, kvh = check_layer_views(k_cache, v_cache)
    t = int(k.shape[0])
    lib = _capi.load()
    rc = lib.ms_kv_scatter(
        k.data_ptr(), _rows(k, "k"), v.data_ptr(), _rows(v, "v"), t, kvh,
        slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), nb, _stream(k.device),
    )
    _capi.check(rc, "kv_scatter")


def attend(q: Tensor, k_cache: Tensor, v_cache: Tensor, meta: AttentionMetadata, scale: float,
           out: Tensor | None = None) -> Tensor:
    """Attention of every planned query row through the pool (backends.py:161-197).

    Rows not covered by ``meta`` are left untouched (undefined, like ``torch.empty_like``).
    """
    nb, kvh = check_layer_views(k_cache, v_cache)
    if out is None:
        out = torch.empty_like(q)
    h = int(q.shape[1])
    ws = meta.workspace(kvh, q.device)
    lib = _capi.load()
    rc = lib.ms_paged_attention(
        q.data_ptr(), _rows(q, "q"), out.data_ptr(), _rows(out, "out"), h, kvh,
        k_cache.data_ptr(), v_cache.data_ptr(), nb, meta.plan.data_ptr(), C.byref(meta.info),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0,
        float(scale), _stream(q.device),
    )
    _capi.check(rc, "paged_attention")
    return out


def paged_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    meta: AttentionMetadata,
    scale: float,
) -> Tensor:
    """Write this step's keys and values into the cache, then attend through it.

    q: [T, heads, 128]; k, v: [T, kv_heads, 128]; caches: layer views of the pool.
    Returns [T, heads, 128] (backends.py:145-158).
    """
    kv_scatter(k, v, meta.slot_mapping, k_cache, v_cache)
    return attend(q, k_cache, v_cache, meta, scale)
