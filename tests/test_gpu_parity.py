"""GPU parity: the CUDA path (through the C ABI) against the reference's golden outputs and the
CPU oracle, on the same seeded inputs.

Bars (from the path's contract):
  * slot placement and the V scatter are bit-exact; the scatter writes exactly the bits kernel A
    produced for K;
  * q/k after norm + RoPE equal the reference's bf16 op sequence except where the 128-term fp32
    sum of squares lands on a different ulp (a different summation order) -- at most one bf16 ulp
    on a tiny fraction of elements;
  * attention outputs agree with the reference's fp32 result within max-abs 2e-2.
"""

from __future__ import annotations

import pytest
import torch

from golden.cases import CASES, D, EPS, H, KVH, THETA, random_inputs
from golden_io import load_golden, make_inputs, run_oracle
from gpu_harness import bf16_ulp_diff, covered_rows, run_layer, setup_pool
from miniserve_b200 import _capi
from miniserve_b200.attention import attend, build_attention_metadata, kv_scatter
from miniserve_b200.kv_pool import allocate_kv_cache, layer_as_slots
from miniserve_b200.qwen3_attention import qk_norm_rope_scatter
from miniserve_b200.workloads import Batch, config2, config3, config4, custom
from oracle import attention_oracle as orc

pytestmark = pytest.mark.gpu

ATOL = 2e-2  # max-abs tolerance of bf16 attention outputs against the fp32 reference


def _fp32_reference_out(inp, q_rot_gpu: torch.Tensor, k_slots: torch.Tensor,
                        v_slots: torch.Tensor) -> torch.Tensor:
    """Oracle attention in fp32 over exactly the bf16 q and pool the kernels saw."""
    k_cache = k_slots.float().cpu()
    v_cache = v_slots.float().cpu()
    slots = torch.from_numpy(inp.batch.slots)
    meta = orc.build_metadata(
        [orc.SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table))
         for c in inp.batch.chunks], slots, 16)
    q = q_rot_gpu.float().cpu()
    return orc.paged_attention(q, k_cache[slots], v_cache[slots], k_cache, v_cache, meta, D**-0.5)


@pytest.mark.parametrize("name", [c for c in CASES if c.endswith("bf16")])
def test_kernel_a_matches_reference_bits(name: str, cuda_device: torch.device) -> None:
    """Against the reference's CPU results (the oracle reproduces them bit for bit, see
    test_oracle_golden.py, so its arrays stand in for cases stored as digests)."""
    inp = make_inputs(name)
    ref = run_oracle(inp)
    got = run_layer(inp, cuda_device)
    assert int(got["status"]) == 0
    # V rows are copied: bit-exact.  K rows in the pool are exactly what kernel A computed.
    assert torch.equal(got["v_at_slots"].cpu(), ref["v_at_slots"])
    for key in ("q_rot", "k_at_slots"):
        ulps = bf16_ulp_diff(got[key].cpu(), ref[key])
        assert int(ulps.max()) <= 1, key
        assert float((ulps > 0).float().mean()) <= 1e-3, key
    # The whole pool against the reference's pool after its index_copy_ (backends.py:159-160):
    # V everywhere and K in every slot this step does not write are bit-identical.
    written = torch.zeros(ref["k_cache"].shape[0], dtype=torch.bool)
    written[torch.from_numpy(inp.batch.slots)] = True
    assert torch.equal(got["v_slots"].cpu(), ref["v_cache"])
    assert torch.equal(got["k_slots"].cpu()[~written], ref["k_cache"][~written])


@pytest.mark.parametrize("name", [c for c in CASES if c.endswith("bf16")])
def test_kernel_a_matches_torch_cuda_sequence(name: str, cuda_device: torch.device) -> None:
    """The same op sequence run by PyTorch on the GPU (the reference on CUDA)."""
    inp = make_inputs(name)
    got = run_layer(inp, cuda_device)
    cos, sin = orc.rope_tables(D, inp.max_positions, THETA)
    pos = torch.from_numpy(inp.batch.positions)
    q, k, _ = orc.norm_rope(
        inp.qkv.to(cuda_device), inp.q_weight.to(cuda_device), inp.k_weight.to(cuda_device), EPS,
        cos[pos].to(cuda_device), sin[pos].to(cuda_device), H, KVH, D,
    )
    for ref, key in ((q, "q_rot"), (k, "k_at_slots")):
        ulps = bf16_ulp_diff(got[key], ref)
        assert int(ulps.max()) <= 1, key
        assert float((ulps > 0).float().mean()) <= 1e-3, key


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("pages_per_split", [0, 1, 3])
def test_attention_matches_reference(name: str, pages_per_split: int,
                                     cuda_device: torch.device) -> None:
    inp = make_inputs(name)
    gold = load_golden(name, inp.dtype)
    got = run_layer(inp, cuda_device, pages_per_split=pages_per_split)
    assert int(got["status"]) == 0
    rows = covered_rows(inp)
    out = got["out"].cpu()[rows].float()
    # Against the reference's own output (fp32 for cfg1, bf16 otherwise).
    err = (out - gold["out"][rows].float()).abs().max().item()
    assert err <= ATOL, err
    # Against the fp32 oracle on exactly the kernel's inputs: isolates kernel B/C error.
    ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows]
    err32 = (out - ref32).abs().max().item()
    assert err32 <= ATOL, err32


def _random_case_vs_fp32(batch, seed: int, pages_per_split: int, device: torch.device) -> float:
    inp = random_inputs(batch, seed)
    got = run_layer(inp, device, pages_per_split=pages_per_split)
    assert int(got["status"]) == 0
    rows = covered_rows(inp)
    ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows]
    return (got["out"].cpu()[rows].float() - ref32).abs().max().item()


@pytest.mark.parametrize("pages_per_split", [0, 8, 64])
def test_tensor_core_prefill_config3(pages_per_split: int, cuda_device: torch.device) -> None:
    """Config 3's geometry: 48 decode rows + two 1000-token chunks over 512 cached tokens
    (tcgen05 kernel for the chunks, decode kernel for the rest), against the fp32 oracle."""
    err = _random_case_vs_fp32(config3(seed=7), 7, pages_per_split, cuda_device)
    assert err <= ATOL, err


@pytest.mark.parametrize("rows", [
    [(65, 0)], [(128, 0)], [(129, 0)], [(200, 1)], [(64, 0), (65, 63)], [(300, 700), (1, 5)],
    [(1000, 0)],
], ids=["65", "128", "129", "200_over_1", "64_and_65", "300_over_700", "1000_fresh"])
def test_tensor_core_prefill_edges(rows, cuda_device: torch.device) -> None:
    """Tile and 128-key block boundaries of the tensor-core path (with forced splits too)."""
    for split in (0, 8):
        err = _random_case_vs_fp32(custom(rows, seed=len(rows)), 3, split, cuda_device)
        assert err <= ATOL, (split, err)


@pytest.mark.parametrize("rows", [
    [(9, 700), (16, 1500), (12, 40)], [(17, 300), (24, 2000), (32, 90)], [(33, 100), (64, 900)],
    [(16, 0), (32, 0), (9, 16)], [(10, 3000)] * 12,
], ids=["4_phases", "2_phases", "1_phase", "fresh", "many_4_phase"])
def test_tile_mode_page_phases(rows, cuda_device: torch.device) -> None:
    """Kernel B's tile mode (9-64-token chunks): tiles of <= 16 tokens split their pages over 4
    phases of warps, <= 32 tokens over 2, longer ones over 1; the phases merge at the end.  Whole
    and split items (whose partials the combine pass merges), against the fp32 oracle."""
    for split in (0, 8, 64):
        err = _random_case_vs_fp32(custom(rows, seed=len(rows) + 40), 5, split, cuda_device)
        assert err <= ATOL, (split, err)


def test_decode_outlier_rows_split(cuda_device: torch.device) -> None:
    """60 short decode rows and 4 long ones: the long rows are split (plan without tensor-core
    work) and merged by the combine pass; against the fp32 oracle."""
    rows = [(1, 100)] * 60 + [(1, 4000)] * 4
    err = _random_case_vs_fp32(custom(rows, seed=44), 44, 0, cuda_device)
    assert err <= ATOL, err


def test_config5_contexts_on_a_non_aliased_subset(cuda_device: torch.device) -> None:
    """Config 5's heavy-tailed contexts (logU[512, 32768]): its shortest, longest and quantile
    rows, each with its own blocks (no pool aliasing), against the fp32 oracle; automatic and
    forced splits."""
    import numpy as np

    from miniserve_b200.workloads import config5_contexts

    ctx = np.sort(config5_contexts(seed=0))
    pick = [ctx[0], ctx[-1]] + [ctx[int(q * (len(ctx) - 1))] for q in (0.1, 0.5, 0.9, 0.99)]
    rows = [(1, int(L) - 1) for L in pick] + [(5, int(pick[1]) - 5)]  # and one verify row
    for split in (0, 64):
        err = _random_case_vs_fp32(custom(rows, seed=21), 21, split, cuda_device)
        assert err <= ATOL, (split, err)


@pytest.mark.parametrize("pages_per_split", [0, 8])
def test_many_short_decode_rows(pages_per_split: int, cuda_device: torch.device) -> None:
    """80 decode and verify rows over 10-400 cached tokens: more decode CTAs than one resident
    wave and few pages each, which the persistent decode kernel serves (with forced splits, its
    partial-row path and the combine too).  Against the fp32 oracle."""
    import numpy as np

    rng = np.random.default_rng(31)
    rows = [(int(rng.choice([1, 1, 1, 5])), int(rng.integers(10, 400))) for _ in range(80)]
    err = _random_case_vs_fp32(custom(rows, seed=31), 31, pages_per_split, cuda_device)
    assert err <= ATOL, err


@pytest.mark.parametrize("num_seqs", [16, 64, 512], ids=["16_rows", "64_rows", "config4"])
def test_cascade_shared_prefix(num_seqs: int, cuda_device: torch.device) -> None:
    """Config 4's geometry (5-token verify rows sharing a 1024-token prefix, 64..256 own tokens):
    the prefix is attended once by the tensor-core kernel over all the rows' tokens, each row's
    own pages by the decode kernel, and the two merged; against the fp32 oracle."""
    batch = config4(seed=11, num_seqs=num_seqs)
    inp = random_inputs(batch, 11)
    got = run_layer(inp, cuda_device)
    assert int(got["status"]) == 0
    assert got["meta_info"].n_cascade == 1
    rows = covered_rows(inp)
    ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows]
    err = (got["out"].cpu()[rows].float() - ref32).abs().max().item()
    assert err <= ATOL, err


def test_cascade_group_beside_other_rows(cuda_device: torch.device) -> None:
    """A cascade group between a prefill chunk and unrelated decode rows, and a 15-row run that is
    too short to form a group: every row against the fp32 oracle."""
    g = config4(seed=12, num_seqs=20)
    short = config4(seed=13, num_seqs=15)
    rows = [(300, 40)] + [(c.num_new, c.num_cached) for c in g.chunks] + [(1, 900), (3, 77)]
    rows += [(c.num_new, c.num_cached) for c in short.chunks]
    batch = custom(rows, seed=14)
    # custom() gives every row its own blocks; share the first 64 blocks among rows 1..20 and,
    # separately, among the last 15 rows, as a prefix cache would.
    chunks = list(batch.chunks)
    for lo, hi in ((1, 21), (23, 38)):
        prefix = list(chunks[lo].block_table[:64])
        for i in range(lo, hi):
            c = chunks[i]
            chunks[i] = type(c)(c.flat_start, c.num_new, c.num_cached, prefix + list(c.block_table[64:]))
    shared = Batch(batch.name, chunks, batch.num_blocks, 0)
    inp = random_inputs(shared, 14)
    got = run_layer(inp, cuda_device)
    assert int(got["status"]) == 0
    assert got["meta_info"].n_cascade == 1
    rows_ = covered_rows(inp)
    ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows_]
    err = (got["out"].cpu()[rows_].float() - ref32).abs().max().item()
    assert err <= ATOL, err


def test_cascade_group_with_unrelated_rows_on_the_persistent_decode_kernel(
        cuda_device: torch.device) -> None:
    """Config 4's 512-row group (its prefix on 160 tensor-core CTAs: a small second wave, so the
    persistent decode kernel leaves those SMs out of its grid) between 64 unrelated decode and
    verify rows.  The decode kernel follows the tensor-core kernel and walks both kinds of unit;
    the unrelated rows have more pages, so they come first and many consumer groups start with a
    unit that merges no prefix before the unit they park.  Every row against the fp32 oracle."""
    import numpy as np

    rng = np.random.default_rng(16)
    g = config4(seed=16, num_seqs=512)
    other = [(int(rng.choice([1, 1, 5])), int(rng.integers(100, 600))) for _ in range(64)]
    rows = other[:32] + [(c.num_new, c.num_cached) for c in g.chunks] + other[32:]
    batch = custom(rows, seed=17)
    chunks = list(batch.chunks)
    lo, hi = 32, 32 + 512
    prefix = list(chunks[lo].block_table[:64])
    for i in range(lo, hi):
        c = chunks[i]
        chunks[i] = type(c)(c.flat_start, c.num_new, c.num_cached, prefix + list(c.block_table[64:]))
    shared = Batch(batch.name, chunks, batch.num_blocks, 0)
    inp = random_inputs(shared, 17)
    got = run_layer(inp, cuda_device)
    assert int(got["status"]) == 0
    info = got["meta_info"]
    assert info.n_cascade == 1
    assert 148 < info.n_tc_items * KVH <= 148 + 148 // 8  # a small second tensor-core wave
    assert info.n_decode_items * KVH > 2 * 148  # more than one resident decode wave
    assert info.decode_pages <= 32 * info.n_decode_items  # ... of short items: the units kernel
    rows_ = covered_rows(inp)
    ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows_]
    err = (got["out"].cpu()[rows_].float() - ref32).abs().max().item()
    assert err <= ATOL, err


@pytest.mark.parametrize("name", ["mixed_bf16", "prefix_verify_bf16", "prefill_bf16"])
def test_scatter_only_path_equals_fused(name: str, cuda_device: torch.device) -> None:
    """paged_attention(q, k, v, ...) (reference call shape) == the fused layer path."""
    inp = make_inputs(name)
    a = run_layer(inp, cuda_device, fused=True)
    b = run_layer(inp, cuda_device, fused=False)
    rows = covered_rows(inp).to(cuda_device)
    assert torch.equal(a["k_slots"], b["k_slots"])
    assert torch.equal(a["v_slots"], b["v_slots"])
    assert torch.equal(a["out"][rows], b["out"][rows])


def test_table_positions_mode_equals_gathered_rows(cuda_device: torch.device) -> None:
    inp = make_inputs("mixed_bf16")
    a = run_layer(inp, cuda_device, positions_mode=False)
    b = run_layer(inp, cuda_device, positions_mode=True)
    rows = covered_rows(inp).to(cuda_device)
    assert torch.equal(a["q_rot"], b["q_rot"])
    assert torch.equal(a["out"][rows], b["out"][rows])


@pytest.mark.parametrize("positions_mode", [False, True], ids=["rows", "table"])
def test_kernel_a_16_and_8_byte_forms_agree_bitwise(positions_mode: bool,
                                                    cuda_device: torch.device) -> None:
    """Kernel A has a 16-byte form (rows and norm weights 16-byte aligned) and an 8-byte form
    (rows only 8-byte aligned, e.g. a qkv row stride of width + 4): the same inputs give the same
    q and the same pool, bit for bit, through config 3's 2,048 tokens (gaussian values, so the
    norm's sums and RoPE's products cover many binades)."""
    from miniserve_b200.workloads import rope_tables

    dev = cuda_device
    batch = config3(seed=7)
    t = batch.num_tokens
    width = (H + 2 * KVH) * D
    g = torch.Generator(device=dev).manual_seed(7)
    qkv = torch.randn(t, width, generator=g, device=dev).mul_(3).bfloat16()
    padded = torch.zeros(t, width + 4, dtype=torch.bfloat16, device=dev)
    padded[:, :width] = qkv
    qkv_v8 = padded[:, :width]  # row stride width + 4: 8-byte aligned rows only
    assert qkv_v8.stride(0) % 8 == 4
    qw = (1 + 0.2 * torch.randn(D, generator=g, device=dev)).bfloat16()
    kw = (1 + 0.2 * torch.randn(D, generator=g, device=dev)).bfloat16()
    cos_t, sin_t = rope_tables(D, batch.max_position + 8, THETA, dev)
    pos = torch.from_numpy(batch.positions).to(dev)
    slots = torch.from_numpy(batch.slots).to(dev)
    if positions_mode:
        cos, sin, pos_arg = cos_t, sin_t, pos
    else:
        cos, sin, pos_arg = cos_t[pos], sin_t[pos], None
    res = []
    for x in (qkv, qkv_v8):
        pool, views = allocate_kv_cache(1, batch.num_blocks, KVH, dev)
        kc, vc = views[0]
        q = qk_norm_rope_scatter(x, qw, kw, EPS, cos, sin, slots, kc, vc, H, positions=pos_arg)
        torch.cuda.synchronize(dev)
        assert _capi.device_status(int(torch.cuda.current_stream(dev).cuda_stream)) == 0
        res.append((q, pool))
    assert torch.equal(res[0][0], res[1][0])
    assert torch.equal(res[0][1], res[1][1])


@pytest.mark.parametrize("strided", [False, True], ids=["contiguous", "qkv_views"])
@pytest.mark.parametrize("name", ["mixed_bf16", "prefix_verify_bf16", "groups_bf16", "prefill_bf16"])
def test_kv_scatter_whole_pool_bit_exact(name: str, strided: bool,
                                         cuda_device: torch.device) -> None:
    """ms_kv_scatter (the reference's scatter, backends.py:159-160) against index_copy_ on the
    reference-layout pool: every slot of the pool, written or not, is bit-identical.  With
    ``strided`` the K/V rows are views into a fused [T, 4096] projection output, as the
    reference's split (qwen3.py:94) hands them over."""
    inp = make_inputs(name)
    b = inp.batch
    _pool, k_cache, v_cache = setup_pool(inp, cuda_device)
    t = b.num_tokens
    g = torch.Generator().manual_seed(99)
    if strided:
        qkv = torch.randn(t, (H + 2 * KVH) * D, generator=g).bfloat16()
        k = qkv[:, H * D:(H + KVH) * D].view(t, KVH, D)
        v = qkv[:, (H + KVH) * D:].view(t, KVH, D)
        k_dev = qkv.to(cuda_device)[:, H * D:(H + KVH) * D].view(t, KVH, D)
        v_dev = qkv.to(cuda_device)[:, (H + KVH) * D:].view(t, KVH, D)
    else:
        k = torch.randn(t, KVH, D, generator=g).bfloat16()
        v = torch.randn(t, KVH, D, generator=g).bfloat16()
        k_dev, v_dev = k.to(cuda_device), v.to(cuda_device)
    slots = torch.from_numpy(b.slots)
    kv_scatter(k_dev, v_dev, slots.to(cuda_device), k_cache, v_cache)
    assert _capi.device_status(int(torch.cuda.current_stream(cuda_device).cuda_stream)) == 0
    ref_k = inp.k_slots.clone()
    ref_v = inp.v_slots.clone()
    ref_k.index_copy_(0, slots, k.contiguous())
    ref_v.index_copy_(0, slots, v.contiguous())
    assert torch.equal(layer_as_slots(k_cache).cpu(), ref_k)
    assert torch.equal(layer_as_slots(v_cache).cpu(), ref_v)


@torch.no_grad()
def test_config2_full_geometry_vs_fp32_oracle(cuda_device: torch.device) -> None:
    """Config 2 exactly as bench.py times it (256 decode rows, contexts U[256, 4096], a pool of
    1.1x the blocks needed with permuted tables, the automatic plan: one unsplit item per row)
    for one layer: kernel A then kernels B/C, against the oracle's attention in fp32 over the same
    bf16 queries and pool (run with PyTorch's plain fp32 math on the GPU; no TF32)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    dev = cuda_device
    batch = config2(seed=1000)
    nb, t = batch.num_blocks, batch.num_tokens
    g = torch.Generator(device=dev).manual_seed(2)
    pool, views = allocate_kv_cache(1, nb, KVH, dev, zero=False)
    pool.normal_(generator=g)
    k_cache, v_cache = views[0]
    qkv = torch.randn(t, (H + 2 * KVH) * D, generator=g, device=dev).bfloat16()
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).bfloat16()
    cos_t, sin_t = orc.rope_tables(D, batch.max_position + 8, THETA)
    positions = torch.from_numpy(batch.positions)
    slots = torch.from_numpy(batch.slots).to(dev)
    meta = build_attention_metadata(batch.chunks, slots, 16)
    assert meta.info.n_decode_items == 256 and meta.info.n_combine == 0
    assert meta.info.n_tc_items == 0 and meta.info.n_tile_items == 0
    q = qk_norm_rope_scatter(qkv, qw, kw, EPS, cos_t[positions].to(dev), sin_t[positions].to(dev),
                             slots, k_cache, v_cache, H)
    out = attend(q, k_cache, v_cache, meta, D**-0.5)
    assert _capi.device_status(int(torch.cuda.current_stream(dev).cuda_stream)) == 0

    ks = layer_as_slots(k_cache).float()
    vs = layer_as_slots(v_cache).float()
    chunks = [orc.SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table))
              for c in batch.chunks]
    ometa = orc.build_metadata(chunks, slots, 16)
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with sdpa_kernel(SDPBackend.MATH):
            ref = orc.paged_attention(q.float(), ks[slots], vs[slots], ks, vs, ometa, D**-0.5)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = allow
    err = (out.float() - ref).abs().max().item()
    print(f"config 2, {t} rows, {batch.kv_tokens_read()} context tokens: max-abs err {err:.3e}")
    assert err <= ATOL, err


def test_tensor_core_items_with_empty_tile_b_repeat_identically(cuda_device: torch.device) -> None:
    """Items whose tile B is empty (n_b = 0) run on the tensor-core kernel in every plan with an
    odd number of 64-token groups (the middle item of the zig-zag pairing) and for split-chunk
    tails.  Twenty chunks of 129-192 tokens (three groups each) plus decode rows, automatic and
    forced splits: 30 back-to-back calls give bit-identical outputs and a clean status, and the
    result matches the fp32 oracle."""
    from miniserve_b200.attention import plan_batch

    rows = [(129 + 3 * i, 40 * i) for i in range(20)] + [(1, 500), (5, 90)]
    batch = custom(rows, seed=71)
    inp = random_inputs(batch, 71)
    for split in (0, 8):
        _, info = plan_batch(batch.chunks, batch.num_tokens, 16, 148, split)
        assert info.n_tc_items > 0
        got = run_layer(inp, cuda_device, pages_per_split=split)
        assert int(got["status"]) == 0
        rows_ = covered_rows(inp)
        ref32 = _fp32_reference_out(inp, got["q_rot"], got["k_slots"], got["v_slots"])[rows_]
        err = (got["out"].cpu()[rows_].float() - ref32).abs().max().item()
        assert err <= ATOL, (split, err)
        # Repeat the attention alone on the same pool and queries.
        _pool, k_cache, v_cache = setup_pool(inp, cuda_device)
        from miniserve_b200.kv_pool import slots_into_layer

        slots_into_layer(k_cache, got["k_slots"])
        slots_into_layer(v_cache, got["v_slots"])
        slots = torch.from_numpy(batch.slots).to(cuda_device)
        meta = build_attention_metadata(batch.chunks, slots, 16, pages_per_split=split)
        first = attend(got["q_rot"], k_cache, v_cache, meta, D**-0.5)
        dev_rows = rows_.to(cuda_device)
        for _ in range(30):
            again = attend(got["q_rot"], k_cache, v_cache, meta, D**-0.5)
            assert torch.equal(again[dev_rows], first[dev_rows])
        assert _capi.device_status(int(torch.cuda.current_stream(cuda_device).cuda_stream)) == 0
        assert torch.equal(first[dev_rows], got["out"][dev_rows])
