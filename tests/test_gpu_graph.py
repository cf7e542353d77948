"""CUDA-graph capture of whole steps (every layer's kernel A + attention): decode, chunked
prefill on the tensor-core kernel, and a shared-prefix (cascade) group.

The C-ABI calls neither allocate nor synchronise, so once the first (eager) call on a device has
set kernel attributes, built the pool's tensor maps and allocated the step's workspace, the step
can be captured and replayed.  Replays must equal eager execution bit for bit, including after new
inputs are copied into the captured buffers.
"""

from __future__ import annotations

import pytest
import torch

from miniserve_b200.attention import attend, build_attention_metadata
from miniserve_b200.kv_pool import allocate_kv_cache
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter
from miniserve_b200.workloads import config2, config3, config4, rope_tables

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("workload", ["config2_32rows", "config3", "config4_64rows", "config4"])
def test_graph_replay_matches_eager(workload: str, cuda_device: torch.device) -> None:
    """Decode rows with forced splits (kernels A, B, C), config 3's chunks (kernel D beside the
    decode kernel), a 64-row cascade group (kernel D's prefix partials merged by the persistent
    decode kernel beside kernel D's one wave) and config 4's 512-row group (kernel D's small
    second wave: the decode grid leaves its SMs out, and consumer groups park their first unit)."""
    dev = cuda_device
    if workload == "config2_32rows":
        layers, batch, split = 28, config2(seed=5, num_seqs=32), 16
    elif workload == "config3":
        layers, batch, split = 4, config3(seed=5), 0
    elif workload == "config4":
        layers, batch, split = 2, config4(seed=5, num_seqs=512), 0
    else:
        layers, batch, split = 4, config4(seed=5, num_seqs=64), 0
    t = batch.num_tokens
    g = torch.Generator(device=dev).manual_seed(5)
    pool, views = allocate_kv_cache(layers, batch.num_blocks, 8, dev, zero=False)
    pool.normal_(generator=g)
    pool_copy = pool.clone()
    qkv = torch.randn(layers, t, 4096, generator=g, device=dev, dtype=torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(layers, 128, generator=g, device=dev)).bfloat16()
    kw = (1 + 0.1 * torch.randn(layers, 128, generator=g, device=dev)).bfloat16()
    cos_t, sin_t = rope_tables(128, batch.max_position + 8, 1e6, dev)
    pos = torch.from_numpy(batch.positions).to(dev)
    slots = torch.from_numpy(batch.slots).to(dev)
    cos, sin = cos_t[pos], sin_t[pos]
    meta = build_attention_metadata(batch.chunks, slots, 16, pages_per_split=split)
    if workload == "config2_32rows":
        assert meta.info.n_combine > 0
    elif workload == "config3":
        assert meta.info.n_tc_items > 0
    else:
        assert meta.info.n_cascade == 1
    q_buf = torch.empty(t, 16, 128, dtype=torch.bfloat16, device=dev)
    out = torch.empty(layers, t, 16, 128, dtype=torch.bfloat16, device=dev)

    def step() -> None:
        for i in range(layers):
            kc, vc = views[i]
            qk_norm_rope_scatter(qkv[i], qw[i], kw[i], 1e-6, cos, sin, slots, kc, vc, 16, q_out=q_buf)
            attend(q_buf, kc, vc, meta, 128**-0.5, out=out[i])

    step()  # eager warm-up on this device (attributes, tensor maps, workspace)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()

    for trial in range(2):
        new_qkv = torch.randn(layers, t, 4096, generator=g, device=dev, dtype=torch.bfloat16)
        qkv.copy_(new_qkv)
        pool.copy_(pool_copy)
        graph.replay()
        torch.cuda.synchronize(dev)
        replayed = out.clone()
        pool.copy_(pool_copy)
        step()
        torch.cuda.synchronize(dev)
        assert torch.equal(replayed, out), trial


def test_graph_replay_after_metadata_update(cuda_device: torch.device) -> None:
    """A step captured with one batch, replayed after ``AttentionMetadata.update`` has written a
    different batch of the same launch shape into its buffers (the same contexts, other pages:
    every block id remapped), equals an eager run of the new batch with freshly built metadata,
    bit for bit.  A batch of another shape is refused and leaves the metadata as it was."""
    from miniserve_b200.attention import SeqChunk

    dev = cuda_device
    layers, batch = 4, config2(seed=7, num_seqs=32)
    t = batch.num_tokens
    g = torch.Generator(device=dev).manual_seed(7)
    pool, views = allocate_kv_cache(layers, batch.num_blocks, 8, dev, zero=False)
    pool.normal_(generator=g)
    pool_copy = pool.clone()
    qkv = torch.randn(layers, t, 4096, generator=g, device=dev, dtype=torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(layers, 128, generator=g, device=dev)).bfloat16()
    kw = (1 + 0.1 * torch.randn(layers, 128, generator=g, device=dev)).bfloat16()
    cos_t, sin_t = rope_tables(128, batch.max_position + 8, 1e6, dev)
    pos = torch.from_numpy(batch.positions).to(dev)
    cos, sin = cos_t[pos], sin_t[pos]
    slots = torch.from_numpy(batch.slots).to(dev)
    meta = build_attention_metadata(batch.chunks, slots, 16, pages_per_split=16)
    assert meta.info.n_combine > 0
    q_buf = torch.empty(t, 16, 128, dtype=torch.bfloat16, device=dev)
    out = torch.empty(layers, t, 16, 128, dtype=torch.bfloat16, device=dev)

    def step(m) -> None:
        for i in range(layers):
            kc, vc = views[i]
            qk_norm_rope_scatter(qkv[i], qw[i], kw[i], 1e-6, cos, sin, m.slot_mapping, kc, vc, 16,
                                 q_out=q_buf)
            attend(q_buf, kc, vc, m, 128**-0.5, out=out[i])

    step(meta)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(meta)

    # The same contexts on other pages.
    perm = torch.randperm(batch.num_blocks, generator=torch.Generator().manual_seed(8))
    chunks_b = [SeqChunk(c.flat_start, c.num_new, c.num_cached, [int(perm[b]) for b in c.block_table])
                for c in batch.chunks]
    slots_cpu = torch.from_numpy(batch.slots)
    slots_b = (perm[slots_cpu // 16] * 16 + slots_cpu % 16).to(dev)
    assert meta.update(chunks_b, slots_b)
    qkv.copy_(torch.randn(layers, t, 4096, generator=g, device=dev, dtype=torch.bfloat16))
    pool.copy_(pool_copy)
    graph.replay()
    torch.cuda.synchronize(dev)
    replayed = out.clone()
    pool.copy_(pool_copy)
    step(build_attention_metadata(chunks_b, slots_b, 16, pages_per_split=16))
    torch.cuda.synchronize(dev)
    assert torch.equal(replayed, out)

    # Another shape (one context grows into a new page) is refused; nothing is written.
    plan_before = meta.plan.clone()
    grown = list(chunks_b)
    c0 = grown[0]
    pages = (c0.num_cached + 1 + 15) // 16
    extra = 16 * pages - c0.num_cached  # cached tokens that move the last token to a new page
    used = {b for c in chunks_b for b in c.block_table}
    free = next(b for b in range(batch.num_blocks) if b not in used)
    grown[0] = SeqChunk(c0.flat_start, 1, c0.num_cached + extra, c0.block_table[:pages] + [free])
    assert not meta.update(grown)
    torch.cuda.synchronize(dev)
    assert torch.equal(meta.plan, plan_before)
