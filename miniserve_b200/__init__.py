"""MiniServe's per-step paged-attention path, rebuilt for B200 (sm_100a).

Public surface (mirrors src/miniserve/attention/backends.py and model/qwen3.py):

* ``attention``: ``SeqChunk``, ``build_attention_metadata``, ``paged_attention``, ``attend``,
  ``kv_scatter``, ``SHORT_QUERY``, ``MAX_GATHER_TOKENS``
* ``qwen3_attention``: ``Qwen3Attention`` (drop-in module), ``qk_norm_rope_scatter`` (kernel A)
* ``kv_pool``: ``allocate_kv_cache`` in the pool layout the kernels read
* ``sharding``: sequence sharding over ranks

The compute runs in ``_lib/libmsattn.so`` (C ABI in ``include/msattn.h``); build it with
``python -m miniserve_b200.build``.
"""

from .attention import (
    MAX_GATHER_TOKENS,
    SHORT_QUERY,
    AttentionMetadata,
    SeqChunk,
    attend,
    build_attention_metadata,
    kv_scatter,
    paged_attention,
)
from .kv_pool import allocate_kv_cache

__all__ = [
    "MAX_GATHER_TOKENS",
    "SHORT_QUERY",
    "AttentionMetadata",
    "SeqChunk",
    "allocate_kv_cache",
    "attend",
    "build_attention_metadata",
    "kv_scatter",
    "paged_attention",
]
