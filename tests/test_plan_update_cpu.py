"""When a new step's plan can be written into a captured step's buffers
(``AttentionMetadata.update``): the launch-shape rule, checked on the host planner.

A CUDA graph captured over the attention calls keeps the grid sizes and section offsets that
the plan description gave at capture time; the kernels read the plan's contents at run time.
So a new plan may replace the captured one exactly when ``same_launch_shape`` holds.
"""

from __future__ import annotations

import numpy as np

from miniserve_b200.attention import SeqChunk, plan_batch, same_launch_shape


def _decode_batch(contexts: list[int], seed: int = 0) -> list[SeqChunk]:
    rng = np.random.default_rng(seed)
    perm = rng.permutation(4096).tolist()
    chunks, cur = [], 0
    for i, L in enumerate(contexts):
        pages = (L + 15) // 16
        chunks.append(SeqChunk(i, 1, L - 1, perm[cur:cur + pages]))
        cur += pages
    return chunks


def _info(chunks: list[SeqChunk]):
    return plan_batch(chunks, sum(c.num_new for c in chunks), 16, 148)[1]


def test_same_batch_has_the_same_shape() -> None:
    ctx = [300, 1000, 77, 4000, 16, 2049]
    assert same_launch_shape(_info(_decode_batch(ctx)), _info(_decode_batch(ctx)))


def test_contexts_growing_inside_their_last_page_keep_the_shape() -> None:
    # 300 -> 301 and 1000 -> 1001 stay inside page 19 / 63; other pages are remapped freely.
    a = _info(_decode_batch([300, 1000, 77], seed=1))
    b = _info(_decode_batch([301, 1001, 78], seed=2))
    assert same_launch_shape(a, b)


def test_a_new_page_changes_the_shape() -> None:
    # 320 -> 321 needs a 21st page: the block tables grow, every later section moves.
    a = _info(_decode_batch([320, 1000]))
    b = _info(_decode_batch([321, 1000]))
    assert not same_launch_shape(a, b)


def test_a_different_mix_changes_the_shape() -> None:
    # The same sequences, the second prefilling 200 tokens instead of decoding one.
    a = _info([SeqChunk(0, 1, 299, list(range(19))), SeqChunk(1, 200, 0, list(range(19, 32)))])
    b = _info([SeqChunk(0, 1, 299, list(range(19))), SeqChunk(1, 1, 199, list(range(19, 32)))])
    assert not same_launch_shape(a, b)
