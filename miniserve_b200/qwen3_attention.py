"""Drop-in ``Qwen3Attention`` whose per-head norm, RoPE, K/V scatter and attention are the
sm_100a kernels (src/miniserve/model/qwen3.py:65-100).

The module keeps the reference's parameter names (``qkv_proj``, ``o_proj``, ``q_norm.weight``,
``k_norm.weight``) so the reference loader (``load_weights``, model/loader.py:51-79) fills it
unchanged, and the same ``forward(x, cos, sin, k_cache, v_cache, meta)`` signature, so
``Qwen3DecoderLayer`` calls it unchanged.  The o_proj GEMM stays a library call (cuBLAS); the qkv
projection is cuBLAS followed by kernel A, or, with ``fused_qkv``, kernel E (both in one launch).
"""

from __future__ import annotations

from typing import Any

import torch
from torch import Tensor, nn

from . import _capi
from .attention import AttentionMetadata, _rows, _stream, attend
from .kv_pool import HEAD_DIM, check_layer_views

# Smallest step (tokens) for which ``fused_qkv="auto"`` takes kernel E: measured on a B200 against
# cuBLAS + kernel A (its 16-byte form) over 28 layers, kernel E is 0.74-0.93x from 64 to 1536
# tokens, 1.01x at 2048 and 1.12-1.26x from 4096 tokens up.
FUSED_QKV_MIN_TOKENS = 2048


class HeadNorm(nn.Module):
    """Holds an RMSNorm's weight and eps (layers.py:10-22); applied inside kernel A."""

    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


def qk_norm_rope_scatter(
    qkv: Tensor,
    q_weight: Tensor,
    k_weight: Tensor,
    eps: float,
    cos: Tensor,
    sin: Tensor,
    slot_mapping: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    num_heads: int,
    positions: Tensor | None = None,
    q_out: Tensor | None = None,
) -> Tensor:
    """Kernel A: returns normalised, rotated q ``[T, H, 128]``; writes k (normalised, rotated)
    and v into their pool slots.  ``cos``/``sin`` are per-token rows ``[T, 128]`` fp32, or the
    whole table when ``positions`` is given (qwen3.py:94-98 + backends.py:159-160)."""
    nb, kvh = check_layer_views(k_cache, v_cache)
    t = int(qkv.shape[0])
    width = (num_heads + 2 * kvh) * HEAD_DIM
    if qkv.dim() != 2 or qkv.shape[1] != width or qkv.stride(1) != 1 or qkv.dtype != torch.bfloat16:
        raise ValueError(f"qkv must be bf16 [T, {width}] with unit column stride")
    if q_weight.dtype != torch.bfloat16 or k_weight.dtype != torch.bfloat16:
        raise ValueError("q_norm / k_norm weights must be bf16")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or cos.stride(-1) != 1:
        raise ValueError("cos/sin must be fp32 with unit column stride")
    if sin.stride(0) != cos.stride(0):
        raise ValueError("cos and sin must share a row stride")
    if positions is None and cos.shape[0] < t:
        raise ValueError("per-token cos/sin rows must cover every token")
    if q_out is None:
        q_out = torch.empty((t, num_heads, HEAD_DIM), dtype=torch.bfloat16, device=qkv.device)
    pos_ptr, max_pos = None, 0
    if positions is not None:
        if positions.dtype != torch.int64:
            raise ValueError("positions must be int64")
        pos_ptr, max_pos = positions.data_ptr(), int(cos.shape[0])
    lib = _capi.load()
    rc = lib.ms_qk_norm_rope_scatter(
        qkv.data_ptr(), int(qkv.stride(0)), t, num_heads, kvh, q_weight.data_ptr(),
        k_weight.data_ptr(), float(eps), cos.data_ptr(), sin.data_ptr(), int(cos.stride(0)),
        pos_ptr, max_pos, slot_mapping.data_ptr(), q_out.data_ptr(), _rows(q_out, "q_out"),
        k_cache.data_ptr(), v_cache.data_ptr(), nb, _stream(qkv.device),
    )
    _capi.check(rc, "qk_norm_rope_scatter")
    return q_out


def qkv_proj_norm_rope_scatter(
    x: Tensor,
    w_qkv: Tensor,
    q_weight: Tensor,
    k_weight: Tensor,
    eps: float,
    cos: Tensor,
    sin: Tensor,
    slot_mapping: Tensor,
    k_cache: Tensor,
    v_cache: Tensor,
    num_heads: int,
    positions: Tensor | None = None,
    q_out: Tensor | None = None,
) -> Tensor:
    """Kernel E: ``qkv_proj`` (``x @ w_qkv.T``, qwen3.py:94) with kernel A as its epilogue, in one
    tensor-core launch.  Same outputs as ``qk_norm_rope_scatter(x @ w_qkv.T, ...)`` up to the
    GEMM's fp32 accumulation order (a projection output may differ by one bf16 ulp)."""
    nb, kvh = check_layer_views(k_cache, v_cache)
    t = int(x.shape[0])
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype != torch.bfloat16:
        raise ValueError("x must be bf16 [T, hidden] with unit column stride")
    hidden = int(x.shape[1])
    width = (num_heads + 2 * kvh) * HEAD_DIM
    if (w_qkv.dim() != 2 or tuple(w_qkv.shape) != (width, hidden) or w_qkv.stride(1) != 1
            or w_qkv.dtype != torch.bfloat16):
        raise ValueError(f"w_qkv must be bf16 [{width}, {hidden}] with unit column stride")
    if q_weight.dtype != torch.bfloat16 or k_weight.dtype != torch.bfloat16:
        raise ValueError("q_norm / k_norm weights must be bf16")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32 or cos.stride(-1) != 1:
        raise ValueError("cos/sin must be fp32 with unit column stride")
    if sin.stride(0) != cos.stride(0):
        raise ValueError("cos and sin must share a row stride")
    if positions is None and cos.shape[0] < t:
        raise ValueError("per-token cos/sin rows must cover every token")
    if q_out is None:
        q_out = torch.empty((t, num_heads, HEAD_DIM), dtype=torch.bfloat16, device=x.device)
    pos_ptr, max_pos = None, 0
    if positions is not None:
        if positions.dtype != torch.int64:
            raise ValueError("positions must be int64")
        pos_ptr, max_pos = positions.data_ptr(), int(cos.shape[0])
    lib = _capi.load()
    rc = lib.ms_qkv_proj_norm_rope_scatter(
        x.data_ptr(), int(x.stride(0)), t, hidden, w_qkv.data_ptr(), int(w_qkv.stride(0)),
        num_heads, kvh, q_weight.data_ptr(), k_weight.data_ptr(), float(eps), cos.data_ptr(),
        sin.data_ptr(), int(cos.stride(0)), pos_ptr, max_pos, slot_mapping.data_ptr(),
        q_out.data_ptr(), _rows(q_out, "q_out"), k_cache.data_ptr(), v_cache.data_ptr(), nb,
        _stream(x.device),
    )
    _capi.check(rc, "qkv_proj_norm_rope_scatter")
    return q_out


class Qwen3Attention(nn.Module):
    """Same constructor and forward as the reference module (qwen3.py:65-100)."""

    def __init__(self, cfg: Any) -> None:
        super().__init__()
        self.num_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.head_dim = cfg.head_dim
        if self.head_dim != HEAD_DIM or self.num_heads != 2 * self.num_kv_heads:
            raise ValueError("the sm_100a path serves head_dim 128 with two query heads per KV head")
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scale = self.head_dim**-0.5
        self.qkv_proj: nn.Module = nn.Linear(cfg.hidden_size, self.q_size + 2 * self.kv_size,
                                             bias=False)
        self.o_proj: nn.Module = nn.Linear(self.q_size, cfg.hidden_size, bias=False)
        self.q_norm = HeadNorm(self.head_dim, cfg.rms_norm_eps)
        self.k_norm = HeadNorm(self.head_dim, cfg.rms_norm_eps)
        # True: kernel E computes the projection and the norm/RoPE/scatter in one launch (faster
        # from about a thousand tokens per step; a projection output can differ from cuBLAS's by
        # one bf16 ulp, from the GEMM's accumulation order).  False: cuBLAS, then kernel A.
        # "auto": kernel E for steps of at least FUSED_QKV_MIN_TOKENS tokens, else cuBLAS + A.
        fused = getattr(cfg, "fused_qkv", False)
        if fused != "auto" and not isinstance(fused, (bool, int)):
            raise ValueError(f"fused_qkv must be True, False or 'auto', not {fused!r}")
        self.fused_qkv: bool | str = fused if fused == "auto" else bool(fused)

    def forward(
        self,
        x: Tensor,
        cos: Tensor,
        sin: Tensor,
        k_cache: Tensor,
        v_cache: Tensor,
        meta: AttentionMetadata,
    ) -> Tensor:
        t = x.shape[0]
        fused = self.fused_qkv is True or (self.fused_qkv == "auto" and t >= FUSED_QKV_MIN_TOKENS)
        if fused and isinstance(self.qkv_proj, nn.Linear):
            q = qkv_proj_norm_rope_scatter(
                x, self.qkv_proj.weight, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
                cos, sin, meta.slot_mapping, k_cache, v_cache, self.num_heads,
            )
        else:
            qkv = self.qkv_proj(x)
            q = qk_norm_rope_scatter(
                qkv, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps, cos, sin,
                meta.slot_mapping, k_cache, v_cache, self.num_heads,
            )
        out = attend(q, k_cache, v_cache, meta, self.scale)
        result: Tensor = self.o_proj(out.reshape(t, self.q_size))
        return result
