"""The paged KV pool in the layout the sm_100a kernels read.

Replaces ``ModelRunner.allocate_kv_cache`` (src/miniserve/runner/model_runner.py:77-94).  The
reference pool is ``[layers, 2, slots, kv_heads, head_dim]``: one token's heads are contiguous,
so one KV head's 16-token block is 16 scattered 256-byte rows.  Here the pool is

    [layers, num_blocks, kv_heads, 2 (K, V), 2 (d // 64), 16 (token), 64 (d % 64)]  bf16

so that K and V of one (block, head) form one contiguous 8 KiB page pair that a single TMA box
moves into shared memory, already split into 128-byte rows for the swizzled layout the tensor
cores read.  Slot semantics are unchanged: slot = block * 16 + offset in the block.

Like the reference, the pool is zero-filled: masked-out keys of a partial last block are still
multiplied by a zero weight, and uninitialised memory could hold NaN bit patterns.
"""

from __future__ import annotations

import torch
from torch import Tensor

BLOCK_SIZE = 16
HEAD_DIM = 128


def kv_bytes_per_token(num_layers: int, num_kv_heads: int, head_dim: int = HEAD_DIM,
                       dtype_bytes: int = 2) -> int:
    """K and V of every layer for one token (qwen3.py:60-62): 112 KiB for Qwen3-0.6B in bf16."""
    return 2 * num_layers * num_kv_heads * head_dim * dtype_bytes


def allocate_kv_cache(
    num_layers: int,
    num_blocks: int,
    num_kv_heads: int,
    device: torch.device | str,
    dtype: torch.dtype = torch.bfloat16,
    zero: bool = True,
) -> tuple[Tensor, list[tuple[Tensor, Tensor]]]:
    """Allocate the pool and return ``(pool, [(k_cache, v_cache) per layer])``.

    Each per-layer view has shape ``[num_blocks, kv_heads, 2, 16, 64]``; ``v_cache`` starts
    4 KiB after ``k_cache`` inside every (block, head) page pair.
    """
    if dtype != torch.bfloat16:
        raise ValueError("the sm_100a kernels read a bf16 pool")
    shape = (num_layers, num_blocks, num_kv_heads, 2, 2, BLOCK_SIZE, HEAD_DIM // 2)
    pool = (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=device)
    views = [(pool[i, :, :, 0], pool[i, :, :, 1]) for i in range(num_layers)]
    return pool, views


def check_layer_views(k_cache: Tensor, v_cache: Tensor) -> tuple[int, int]:
    """Validate one layer's (k_cache, v_cache) views; return ``(num_blocks, num_kv_heads)``."""
    if k_cache.dtype != torch.bfloat16 or v_cache.dtype != torch.bfloat16:
        raise ValueError("KV pool views must be bf16")
    if k_cache.dim() != 5 or tuple(k_cache.shape[2:]) != (2, BLOCK_SIZE, HEAD_DIM // 2):
        raise ValueError(
            "k_cache must be a layer view of miniserve_b200.kv_pool.allocate_kv_cache "
            f"([blocks, kv_heads, 2, 16, 64]); got shape {tuple(k_cache.shape)}"
        )
    nb, kvh = int(k_cache.shape[0]), int(k_cache.shape[1])
    page = BLOCK_SIZE * HEAD_DIM  # elements of one K (or V) page
    want = (kvh * 2 * page, 2 * page, page // 2, HEAD_DIM // 2, 1)
    if tuple(k_cache.stride()) != want or tuple(v_cache.stride()) != want:
        raise ValueError(f"KV pool views have strides {tuple(k_cache.stride())}, expected {want}")
    if v_cache.shape != k_cache.shape or v_cache.data_ptr() != k_cache.data_ptr() + 2 * page:
        raise ValueError("v_cache must be the V half of the same pool as k_cache")
    return nb, kvh


def layer_as_slots(view: Tensor) -> Tensor:
    """A copy of one layer's K (or V) view in the reference layout ``[slots, kv_heads, 128]``."""
    nb, kvh = view.shape[0], view.shape[1]
    return view.permute(0, 3, 1, 2, 4).reshape(nb * BLOCK_SIZE, kvh, HEAD_DIM)


def slots_into_layer(view: Tensor, slots_layout: Tensor) -> None:
    """Fill one layer's K (or V) view from a reference-layout ``[slots, kv_heads, 128]`` tensor."""
    nb, kvh = view.shape[0], view.shape[1]
    src = slots_layout.reshape(nb, BLOCK_SIZE, kvh, 2, HEAD_DIM // 2).permute(0, 2, 3, 1, 4)
    view.copy_(src)
