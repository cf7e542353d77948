"""Run the CUDA path on a golden case (GPU test helper).

Everything here goes through the public Python API, which calls libmsattn.so through its C ABI.
"""

from __future__ import annotations

import torch

from golden.cases import EPS, H, THETA, CaseInputs
from miniserve_b200 import _capi
from miniserve_b200.attention import build_attention_metadata, paged_attention
from miniserve_b200.kv_pool import allocate_kv_cache, layer_as_slots, slots_into_layer
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter
from oracle import attention_oracle as orc


def setup_pool(inp: CaseInputs, device: torch.device):
    pool, views = allocate_kv_cache(1, inp.batch.num_blocks, 8, device)
    k_cache, v_cache = views[0]
    slots_into_layer(k_cache, inp.k_slots.to(device=device, dtype=torch.bfloat16))
    slots_into_layer(v_cache, inp.v_slots.to(device=device, dtype=torch.bfloat16))
    return pool, k_cache, v_cache


def run_layer(inp: CaseInputs, device: torch.device, pages_per_split: int = 0,
              fused: bool = True, positions_mode: bool = False) -> dict[str, torch.Tensor]:
    """Kernel A (+ scatter) then kernels B/C on one layer; returns GPU results."""
    b = inp.batch
    pool, k_cache, v_cache = setup_pool(inp, device)
    cos_t, sin_t = orc.rope_tables(128, inp.max_positions, THETA)
    positions = torch.from_numpy(b.positions).to(device)
    slot_mapping = torch.from_numpy(b.slots).to(device)
    qkv = inp.qkv.to(device=device, dtype=torch.bfloat16)
    qw = inp.q_weight.to(device=device, dtype=torch.bfloat16)
    kw = inp.k_weight.to(device=device, dtype=torch.bfloat16)
    meta = build_attention_metadata(b.chunks, slot_mapping, 16, pages_per_split=pages_per_split)
    if positions_mode:
        cos, sin = cos_t.to(device), sin_t.to(device)
        pos_arg = positions
    else:
        cos, sin = cos_t[positions.cpu()].to(device), sin_t[positions.cpu()].to(device)
        pos_arg = None
    if fused:
        q = qk_norm_rope_scatter(qkv, qw, kw, EPS, cos, sin, slot_mapping, k_cache, v_cache, H,
                                 positions=pos_arg)
        from miniserve_b200.attention import attend

        out = attend(q, k_cache, v_cache, meta, 128**-0.5)
    else:
        # The reference's call shape: q/k/v already normalised and rotated (here by kernel A on a
        # scratch pool), then paged_attention() scatters and attends.
        scratch_pool, sviews = allocate_kv_cache(1, b.num_blocks, 8, device)
        q = qk_norm_rope_scatter(qkv, qw, kw, EPS, cos, sin, slot_mapping, *sviews[0], H,
                                 positions=pos_arg)
        k_rot = layer_as_slots(sviews[0][0])[slot_mapping]
        v_new = layer_as_slots(sviews[0][1])[slot_mapping]
        out = paged_attention(q, k_rot, v_new, k_cache, v_cache, meta, 128**-0.5)
    status = _capi.device_status(int(torch.cuda.current_stream(device).cuda_stream))
    ks = layer_as_slots(k_cache)
    vs = layer_as_slots(v_cache)
    return {
        "q_rot": q,
        "k_at_slots": ks[slot_mapping],
        "v_at_slots": vs[slot_mapping],
        "out": out,
        "k_slots": ks,
        "v_slots": vs,
        "status": torch.tensor(status),
        "meta_info": meta.info,
    }


def covered_rows(inp: CaseInputs) -> torch.Tensor:
    rows = []
    for c in inp.batch.chunks:
        rows.extend(range(c.flat_start, c.flat_start + c.num_new))
    return torch.tensor(rows, dtype=torch.long)


def bf16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of bf16 ulps (ordered-integer distance of the bit patterns)."""
    def key(x: torch.Tensor) -> torch.Tensor:
        i = x.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -32768 - i, i)

    return (key(a) - key(b)).abs()
