"""KV pool layout helpers on the host: size formula (qwen3.py:60-62), view geometry and strides,
and the round trip between the reference's slot layout ([slots, kv_heads, 128]) and the pool."""

from __future__ import annotations

import pytest
import torch

from miniserve_b200.kv_pool import (allocate_kv_cache, check_layer_views, kv_bytes_per_token,
                                    layer_as_slots, slots_into_layer)


def test_kv_bytes_per_token_matches_the_reference_formula() -> None:
    # Qwen3-0.6B: 2 (K, V) x 28 layers x 8 KV heads x 128 dims x 2 bytes = 112 KiB.
    assert kv_bytes_per_token(28, 8) == 2 * 28 * 8 * 128 * 2 == 112 * 1024
    assert kv_bytes_per_token(28, 8, dtype_bytes=4) == 224 * 1024


def test_pool_views_geometry() -> None:
    pool, views = allocate_kv_cache(3, 5, 8, "cpu")
    assert pool.shape == (3, 5, 8, 2, 2, 16, 64) and pool.dtype == torch.bfloat16
    assert bool((pool == 0).all())  # zero-filled like the reference pool
    for k, v in views:
        assert check_layer_views(k, v) == (5, 8)
        # K and V of one (block, head) are one contiguous 8 KiB page pair, V 4 KiB after K.
        assert (v.data_ptr() - k.data_ptr()) == 16 * 128 * 2
    with pytest.raises(ValueError, match="bf16"):
        allocate_kv_cache(1, 1, 8, "cpu", dtype=torch.float16)


def test_check_layer_views_rejects_other_layouts() -> None:
    _, views = allocate_kv_cache(1, 4, 8, "cpu")
    k, v = views[0]
    with pytest.raises(ValueError, match="layer view"):
        check_layer_views(torch.zeros(64, 8, 128, dtype=torch.bfloat16), v)
    with pytest.raises(ValueError, match="V half"):
        check_layer_views(k, k)


def test_slot_layout_round_trip() -> None:
    g = torch.Generator().manual_seed(0)
    _, views = allocate_kv_cache(1, 6, 8, "cpu")
    k, _ = views[0]
    slots = torch.randn(6 * 16, 8, 128, generator=g).bfloat16()
    slots_into_layer(k, slots)
    assert torch.equal(layer_as_slots(k), slots)
    # slot s = block * 16 + offset: its head-h row sits in block s // 16, token s % 16, split in
    # two 64-dim halves.
    s, h = 37, 5
    blk, tok = divmod(s, 16)
    assert torch.equal(k[blk, h, 0, tok], slots[s, h, :64])
    assert torch.equal(k[blk, h, 1, tok], slots[s, h, 64:])
