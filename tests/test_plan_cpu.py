"""Host planner (ms_plan_build) properties: complete, disjoint page coverage; decode/tile split;
longest-first order; consistent split-KV partial rows; clear errors on bad batches."""

from __future__ import annotations

import numpy as np
import pytest

from miniserve_b200.attention import SeqChunk, plan_batch
from miniserve_b200.workloads import config1, config2, config3, config4, custom

REC = 8


def decode_plan(packed: np.ndarray, info):
    def recs(off: int, n: int) -> np.ndarray:
        return packed[off : off + n * REC].reshape(n, REC)

    return (recs(info.off_seqs, info.num_seqs + info.n_cascade), recs(info.off_decode, info.n_decode_items),
            recs(info.off_tile, info.n_tile_items), recs(info.off_tc, info.n_tc_items),
            recs(info.off_combine, info.n_combine))


def check_plan(chunks: list[SeqChunk], num_tokens: int, split: int = 0, num_sms: int = 148) -> None:
    packed, info = plan_batch(chunks, num_tokens, 16, num_sms, split)
    seqs, dec, til, tcv, comb = decode_plan(packed, info)
    assert info.num_seqs == len(chunks)
    flat_tables = packed[info.off_tables :]
    for i, c in enumerate(chunks):
        r = seqs[i]
        assert list(r[:4]) == [c.flat_start, c.num_new, c.num_cached, c.context_len]
        assert list(flat_tables[r[4] : r[4] + r[5]]) == list(c.block_table)
    # Cascade groups: records after the real sequences; members are consecutive decode / verify
    # rows, contiguous in the batch, whose tables start with the group's prefix blocks.
    cascade: dict[int, tuple[int, int]] = {}  # row -> (prefix pages, group index)
    group_of_vseq: dict[int, tuple[int, int, int]] = {}
    for g in range(info.n_cascade):
        flat, tokens, cached, ctx, toff, pages = (int(x) for x in seqs[len(chunks) + g][:6])
        assert cached == 16 * pages >= 256 and ctx == cached + tokens
        prefix = list(flat_tables[toff : toff + pages])
        members = [i for i, c in enumerate(chunks) if flat <= c.flat_start < flat + tokens]
        assert len(members) >= 16 and members == list(range(members[0], members[-1] + 1))
        assert sum(chunks[i].num_new for i in members) == tokens
        for i in members:
            c = chunks[i]
            assert c.num_new <= 8 and c.num_cached >= 16 * pages
            assert list(c.block_table[:pages]) == prefix
            assert i not in cascade
            cascade[i] = (pages, g)
        group_of_vseq[len(chunks) + g] = (tokens, pages, flat)
    vcover: dict[int, list[tuple[int, int, int, int]]] = {}
    # Every query tile's visible pages are covered exactly once by its items.  Tensor-core
    # records hold two 64-token tiles: A = (tok0, n_q), B = (fields 6, 7); unsplit chunks pair
    # groups g and G-1-g, split items keep A and B adjacent.
    cover: dict[tuple[int, int], list[tuple[int, int, int]]] = {}
    item_tokens: dict[tuple[int, int], int] = {}
    tc_groups: dict[tuple[int, int], int] = {}
    for kind, items in (("dec", dec), ("til", til), ("tc", tcv)):
        for it in items:
            seq, tok0, nq, pb, pe, part, tok_b, n_b = (int(x) for x in it[:8])
            if seq >= len(chunks):
                # a cascade group's shared prefix: adjacent 64-token tiles, pages [0, prefix)
                tokens, pages, _ = group_of_vseq[seq]
                assert kind == "tc" and pb == 0 and pe == pages and part >= 0 and tok0 % 128 == 0
                assert nq == min(64, tokens - tok0) and n_b == max(0, min(64, tokens - tok0 - 64))
                assert n_b == 0 or tok_b == tok0 + 64
                vcover.setdefault(seq, []).append((tok0, nq + n_b, part, pe))
                continue
            c = chunks[seq]
            if seq in cascade:
                # the row's own pages after the shared prefix: one unsplit decode item that
                # merges the row's prefix partials (fields 6, 7) into its output
                pages, g = cascade[seq]
                assert kind == "dec" and tok0 == 0 and nq == c.num_new and part == -1
                assert pb == pages and pe == -(-(c.num_cached + nq) // 16) and n_b == 1
                cover.setdefault((seq, tok0), []).append((pb, pe, tok_b))
                item_tokens[(seq, tok0)] = (nq, pe)
                continue
            assert 0 < nq and tok0 + nq <= c.num_new
            assert 0 <= pb < pe
            if kind == "dec":
                assert c.num_new <= 8 and tok0 == 0 and nq == c.num_new and tok_b == n_b == 0
                last = nq
            elif kind == "til":
                assert 8 < c.num_new <= 64 and tok0 == 0 and nq == c.num_new and tok_b == n_b == 0
                last = nq
            else:
                assert c.num_new > 64 and tok0 % 64 == 0 and nq == min(64, c.num_new - tok0)
                assert pb % 8 == 0, "tensor-core ranges start on 128-key blocks"
                for g0, gn in ((tok0, nq), (tok_b, n_b)):
                    if gn:
                        assert g0 % 64 == 0 and gn == min(64, c.num_new - g0)
                        key = (seq, g0)
                        tc_groups[key] = tc_groups.get(key, 0) + (1 if pb == 0 else 0)
                if n_b:
                    assert tok_b > tok0
                if part >= 0:
                    assert n_b == 0 or tok_b == tok0 + 64, "split items keep their tiles adjacent"
                last = tok_b + n_b if n_b else tok0 + nq
            assert pe <= -(-(c.num_cached + last) // 16)
            cover.setdefault((seq, tok0), []).append((pb, pe, part))
            item_tokens[(seq, tok0)] = (nq + n_b, -(-(c.num_cached + last) // 16))
        lens = [int(it[4] - it[3]) for it in items]
        assert lens == sorted(lens, reverse=True), "items must be longest first"
    for c_idx, c in enumerate(chunks):
        if c.num_new > 64:
            for g0 in range(0, c.num_new, 64):
                assert tc_groups.pop((c_idx, g0)) == 1, "each 64-token group in exactly one item"
    assert not tc_groups
    for vseq, parts in vcover.items():
        tokens, pages, _ = group_of_vseq[vseq]
        parts.sort()
        assert [p[0] for p in parts] == list(range(0, tokens, 128))
        base = parts[0][2]
        assert all(p[2] == base + 2 * p[0] for p in parts), "prefix partial rows in token order"
        group_of_vseq[vseq] = (tokens, pages, base)
    assert len(vcover) == info.n_cascade
    combos = {(int(r[0]), int(r[1])): r for r in comb}
    for key, spans in list(cover.items()):
        if key[0] not in cascade:
            continue
        pages, g = cascade[key[0]]
        _, _, base = group_of_vseq[len(chunks) + g]
        (pb, pe, merge_row), = spans
        assert key not in combos, "cascade rows merge in the decode kernel, no combine record"
        prefix_row = base + 2 * (chunks[key[0]].flat_start - int(seqs[len(chunks) + g][0]))
        assert merge_row == prefix_row
        del cover[key]
    for key, spans in cover.items():
        spans = sorted(spans)
        n_tokens, pages = item_tokens[key]
        assert spans[0][0] == 0 and spans[-1][1] == pages
        for a, b in zip(spans, spans[1:]):
            assert a[1] == b[0]
        if len(spans) == 1:
            assert spans[0][2] == -1 and key not in combos
        else:
            r = combos.pop(key)
            assert int(r[2]) == n_tokens and int(r[4]) == len(spans) and int(r[5]) == 0
            parts = sorted(s[2] for s in spans)
            assert parts == [int(r[3]) + k * 2 * n_tokens for k in range(len(spans))]
    assert not combos
    for c_idx, c in enumerate(chunks):
        if c.num_new <= 64 and c_idx not in cascade:
            assert (c_idx, 0) in cover
    assert info.workspace_bytes_per_kv_head == info.part_rows * 129 * 4
    # decode_pages: the pages the decode / verify items read (it picks the decode kernel form)
    assert info.decode_pages == int(sum(int(it[4] - it[3]) for it in dec))
    # combine_tokens_max: the most query tokens of one combine record (it sizes the combine grid)
    assert info.combine_tokens_max == max((int(c[2]) for c in comb), default=0)


@pytest.mark.parametrize("make", [config1, config2, config3, config4])
@pytest.mark.parametrize("split", [0, 1, 7, 64])
def test_plan_covers_benchmark_batches(make, split: int) -> None:
    b = make(seed=3)
    check_plan(b.chunks, b.num_tokens, split)


@pytest.mark.parametrize("seed", range(5))
def test_plan_random_ragged_batches(seed: int) -> None:
    rng = np.random.default_rng(seed)
    rows = []
    for _ in range(int(rng.integers(1, 40))):
        kind = rng.integers(0, 4)
        n = 1 if kind == 0 else int(rng.integers(2, 9)) if kind == 1 else int(rng.integers(9, 300))
        rows.append((n, int(rng.integers(0, 3000))))
    b = custom(rows, seed=seed)
    check_plan(b.chunks, b.num_tokens, int(rng.integers(0, 20)))


@pytest.mark.parametrize("rows", [
    [(1024, 8192)], [(512, 8192)], [(2048, 16384)], [(1024, 4096)], [(768, 12000)],
    [(1024, 8192), (1024, 8192)], [(128, 32768)], [(300, 20000), (90, 5000)],
])
def test_tc_split_fits_one_wave(rows) -> None:
    """Prefill chunks over long caches, with fewer tensor-core tiles x KV heads than SMs, are
    split into more items but never beyond one wave of CTAs (one per SM); split ranges start on
    whole 128-key blocks, and the plan stays a complete cover."""
    b = custom(rows, seed=2)
    check_plan(b.chunks, b.num_tokens)
    packed, info = plan_batch(b.chunks, b.num_tokens, 16, 148, 0)
    tiles = sum((c.num_new + 127) // 128 for c in b.chunks)
    assert tiles * 8 < 148
    assert tiles < info.n_tc_items and info.n_tc_items * 8 <= 148
    _, _, _, tcv, _ = decode_plan(packed, info)
    assert all(int(it[3]) % 8 == 0 for it in tcv)


def test_decode_outliers_split_only_without_tensor_core_work() -> None:
    """Decode rows beyond a wave stay whole, except that in a plan without tensor-core work the
    rows longer than the pages per item-slot are split into pieces of about that size."""
    rows = [(1, 100)] * 60 + [(1, 4000)] * 4
    b = custom(rows, seed=4)
    check_plan(b.chunks, b.num_tokens)
    packed, info = plan_batch(b.chunks, b.num_tokens, 16, 148, 0)
    _, dec, _, _, comb = decode_plan(packed, info)
    assert info.pages_per_split < 512 and info.n_combine == 4
    assert max(int(it[4] - it[3]) for it in dec) <= info.pages_per_split
    assert all(int(it[4] - it[3]) == 7 for it in dec if int(it[0]) < 60)  # short rows whole
    # The same rows beside a tensor-core chunk: nothing is split.
    b2 = custom(rows + [(300, 0)], seed=4)
    check_plan(b2.chunks, b2.num_tokens)
    _, info2 = plan_batch(b2.chunks, b2.num_tokens, 16, 148, 0)
    assert info2.n_combine == 0 and info2.n_decode_items == 64


@pytest.mark.parametrize("num_sms", [1, 7, 132, 148, 296])
@pytest.mark.parametrize("seed", range(4))
def test_plan_cover_for_other_sm_counts(num_sms: int, seed: int) -> None:
    """The automatic splits (decode, tile, tensor-core, outlier rows) depend on the SM count; the
    plan must stay a complete, disjoint cover for any of them, mixed batches and cascade groups
    included."""
    rng = np.random.default_rng(100 + seed)
    rows = []
    for _ in range(int(rng.integers(1, 60))):
        kind = rng.integers(0, 5)
        n = (1 if kind <= 1 else int(rng.integers(2, 9)) if kind == 2
             else int(rng.integers(9, 65)) if kind == 3 else int(rng.integers(65, 700)))
        rows.append((n, int(rng.integers(0, 6000))))
    b = custom(rows, seed=seed)
    check_plan(b.chunks, b.num_tokens, 0, num_sms)
    c4 = config4(seed=seed, num_seqs=40)
    check_plan(c4.chunks, c4.num_tokens, 0, num_sms)


def test_empty_batch() -> None:
    packed, info = plan_batch([], 0)
    assert info.n_decode_items == info.n_tile_items == info.n_combine == 0


def test_plan_rejects_short_table() -> None:
    with pytest.raises(ValueError, match="blocks but its table has"):
        plan_batch([SeqChunk(0, 1, 40, [0, 1])], 1)


def test_plan_rejects_zero_new_tokens() -> None:
    with pytest.raises(ValueError, match="invalid"):
        plan_batch([SeqChunk(0, 0, 4, [0])], 1)


def test_plan_rejects_rows_outside_batch() -> None:
    with pytest.raises(ValueError, match="invalid"):
        plan_batch([SeqChunk(5, 4, 0, [0])], 6)


def test_plan_rejects_other_block_sizes() -> None:
    with pytest.raises(ValueError, match="block_size"):
        plan_batch([SeqChunk(0, 1, 0, [0])], 1, block_size=32)


@pytest.mark.parametrize("world", [1, 8])
def test_config5_shard_plans(world: int) -> None:
    from miniserve_b200.workloads import config5, config5_contexts

    ctx = config5_contexts(seed=0)
    total_rows = 0
    for rank in sorted({0, world - 1}):
        b = config5(rank, world, seed=0, pool_bytes=20e9)
        assert all(0 <= x < b.num_blocks for c in b.chunks[:50] for x in c.block_table)
        assert all(len(c.block_table) * 16 >= c.context_len for c in b.chunks)
        total_rows += len(b.chunks)
        if world == 1:
            assert len(b.chunks) == len(ctx) and b.aliased
    packed, info = plan_batch(config5(0, world, seed=0, pool_bytes=20e9).chunks,
                              len(config5(0, world, seed=0, pool_bytes=20e9).chunks), 16, 148, 0)
    assert info.n_decode_items >= len(ctx) // world - 1
