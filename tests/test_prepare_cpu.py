"""Native runner preparation (ms_prepare_step) against the restated reference loop
(model_runner.py:162-205): flat offsets, positions and slot mappings in flat-batch order."""

from __future__ import annotations

import numpy as np
import pytest

from miniserve_b200.attention import prepare_step
from miniserve_b200.workloads import config1, config2, config3, config4
from oracle import attention_oracle as orc


def _check(scheduled: list[tuple[int, int, list[int]]]) -> None:
    chunks, pos, slots = prepare_step(scheduled)
    ref_chunks, ref_pos, ref_slots = orc.prepare_step(scheduled, 16)
    assert pos.dtype == np.int64 and slots.dtype == np.int64
    assert pos.tolist() == ref_pos and slots.tolist() == ref_slots
    assert [(c.flat_start, c.num_new, c.num_cached, c.block_table) for c in chunks] == [
        (c.flat_start, c.num_new, c.num_cached, c.block_table) for c in ref_chunks]


def test_reference_docstring_example() -> None:
    # model_runner.py:165-170: A decoding at 7, B decoding at 3, C prefilling 5 tokens.
    chunks, pos, slots = prepare_step([(1, 7, [5]), (1, 3, [9]), (5, 0, [2])])
    assert pos.tolist() == [7, 3, 0, 1, 2, 3, 4]
    assert slots.tolist() == [5 * 16 + 7, 9 * 16 + 3, 32, 33, 34, 35, 36]
    assert [c.flat_start for c in chunks] == [0, 1, 2]


@pytest.mark.parametrize("make", [config1, config2, config3, config4])
def test_benchmark_batches(make) -> None:
    b = make(seed=5)
    scheduled = [(c.num_new, c.num_cached, list(c.block_table)) for c in b.chunks]
    _check(scheduled)
    chunks, pos, slots = prepare_step(scheduled)
    assert np.array_equal(pos, b.positions) and np.array_equal(slots, b.slots)


@pytest.mark.parametrize("seed", range(6))
def test_random_batches_and_block_boundaries(seed: int) -> None:
    rng = np.random.default_rng(seed)
    scheduled = []
    for _ in range(int(rng.integers(1, 60))):
        n = int(rng.choice([1, 2, 5, 8, 15, 16, 17, 64, 200]))
        c = int(rng.integers(0, 3000))
        need = -(-(n + c) // 16) + int(rng.integers(0, 3))
        scheduled.append((n, c, rng.integers(0, 100_000, size=need).tolist()))
    _check(scheduled)


def test_into_preallocated_buffers() -> None:
    scheduled = [(3, 14, [4, 6]), (1, 0, [8])]
    pos = np.full(16, -1, dtype=np.int64)
    slots = np.full(16, -1, dtype=np.int64)
    _, p, s = prepare_step(scheduled, positions_out=pos, slots_out=slots)
    assert p.tolist() == [14, 15, 16, 0] and s.tolist() == [78, 79, 96, 128]
    assert pos[4:].tolist() == [-1] * 12  # nothing written past the batch


def test_empty_batch() -> None:
    chunks, pos, slots = prepare_step([])
    assert chunks == [] and pos.size == 0 and slots.size == 0


def test_errors() -> None:
    with pytest.raises(ValueError, match="blocks but its table has"):
        prepare_step([(1, 40, [0, 1])])
    with pytest.raises(ValueError, match="invalid"):
        prepare_step([(0, 4, [0])])
    with pytest.raises(ValueError, match="contiguous int64"):
        prepare_step([(5, 0, [0])], positions_out=np.zeros(4, dtype=np.int64),
                     slots_out=np.zeros(8, dtype=np.int64))
    with pytest.raises(ValueError, match="contiguous int64"):
        prepare_step([(2, 0, [0])], positions_out=np.zeros(4, dtype=np.int32))


def test_capacity_error_from_the_library() -> None:
    import ctypes as C

    from miniserve_b200 import _capi

    lib = _capi.load()
    new = np.array([5], dtype=np.int32)
    cached = np.array([0], dtype=np.int32)
    offsets = np.array([0, 1], dtype=np.int64)
    tables = np.array([3], dtype=np.int32)
    flat = np.zeros(1, dtype=np.int32)
    pos = np.zeros(4, dtype=np.int64)
    slots = np.zeros(4, dtype=np.int64)
    got = C.c_int32(-1)
    rc = lib.ms_prepare_step(1, new.ctypes.data, cached.ctypes.data, offsets.ctypes.data,
                             tables.ctypes.data, 16, flat.ctypes.data, pos.ctypes.data,
                             slots.ctypes.data, 4, C.byref(got))
    assert rc == _capi.MS_ERR_CAPACITY and got.value == 0
    assert "tokens scheduled" in lib.ms_last_error().decode()
