"""A minimal Qwen3 forward with a pluggable attention step (test harness).

Mirrors the reference model's op order (src/miniserve/model/qwen3.py:104-158 and layers.py):
embedding -> per layer [RMSNorm -> fused qkv -> attention -> o_proj -> residual -> RMSNorm ->
SwiGLU -> residual] -> final RMSNorm -> tied/untied LM head.  The attention step receives the
layer index and the fused qkv rows and returns the attention output [T, H*D] (before o_proj), so
the same weights run through the CPU oracle or through the CUDA path.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor

from oracle import attention_oracle as orc


@dataclass
class Shapes:
    vocab: int
    hidden: int
    inter: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float
    theta: float


QWEN3_06B = Shapes(151936, 1024, 3072, 28, 16, 8, 128, 1e-6, 1e6)


class Qwen3Weights:
    def __init__(self, shapes: Shapes, tensors: dict[str, Tensor]) -> None:
        self.s = shapes
        self.t = tensors

    @classmethod
    def from_hf_state_dict(cls, shapes: Shapes, sd: dict[str, Tensor], dtype, device) -> Qwen3Weights:
        """Fuse q/k/v and gate/up the way the reference loader does (model/loader.py:41-79)."""
        t: dict[str, Tensor] = {}
        g = lambda k: sd[k].to(device=device, dtype=dtype)  # noqa: E731
        t["embed"] = g("model.embed_tokens.weight")
        t["norm"] = g("model.norm.weight")
        t["lm_head"] = g("lm_head.weight") if "lm_head.weight" in sd else t["embed"]
        for i in range(shapes.layers):
            p = f"model.layers.{i}."
            t[f"{i}.ln1"] = g(p + "input_layernorm.weight")
            t[f"{i}.ln2"] = g(p + "post_attention_layernorm.weight")
            t[f"{i}.qkv"] = torch.cat([g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight"),
                                       g(p + "self_attn.v_proj.weight")])
            t[f"{i}.o"] = g(p + "self_attn.o_proj.weight")
            t[f"{i}.qn"] = g(p + "self_attn.q_norm.weight")
            t[f"{i}.kn"] = g(p + "self_attn.k_norm.weight")
            t[f"{i}.gu"] = torch.cat([g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")])
            t[f"{i}.down"] = g(p + "mlp.down_proj.weight")
        return cls(shapes, t)

    @classmethod
    def random(cls, shapes: Shapes, seed: int, dtype, device, std: float = 0.02) -> Qwen3Weights:
        gen = torch.Generator(device=device).manual_seed(seed)
        s = shapes

        def rnd(*shape: int) -> Tensor:
            return (torch.randn(*shape, generator=gen, device=device) * std).to(dtype)

        def ones_ish(n: int) -> Tensor:
            return (1 + 0.1 * torch.randn(n, generator=gen, device=device)).to(dtype)

        qkv_rows = (s.heads + 2 * s.kv_heads) * s.head_dim
        t: dict[str, Tensor] = {"embed": rnd(s.vocab, s.hidden), "norm": ones_ish(s.hidden)}
        t["lm_head"] = t["embed"]
        for i in range(s.layers):
            t[f"{i}.ln1"] = ones_ish(s.hidden)
            t[f"{i}.ln2"] = ones_ish(s.hidden)
            t[f"{i}.qkv"] = rnd(qkv_rows, s.hidden)
            t[f"{i}.o"] = rnd(s.hidden, s.heads * s.head_dim)
            t[f"{i}.qn"] = ones_ish(s.head_dim)
            t[f"{i}.kn"] = ones_ish(s.head_dim)
            t[f"{i}.gu"] = rnd(2 * s.inter, s.hidden)
            t[f"{i}.down"] = rnd(s.hidden, s.inter)
        return cls(s, t)


AttentionStep = Callable[[int, Tensor], Tensor]  # (layer, qkv [T, (H+2KVH)*D]) -> [T, H*D]


def forward(w: Qwen3Weights, input_ids: Tensor, attention: AttentionStep,
            from_hidden: bool = False) -> Tensor:
    """Final hidden states [T, hidden] (qwen3.py:140-153).  from_hidden: `attention` receives the
    normalised hidden states and does the qkv projection itself (a fused projection kernel)."""
    s, t = w.s, w.t
    x = t["embed"][input_ids]
    for i in range(s.layers):
        h = orc.rms_norm(x, t[f"{i}.ln1"], s.eps)
        att_in = h if from_hidden else F.linear(h, t[f"{i}.qkv"])
        x = x + F.linear(attention(i, att_in), t[f"{i}.o"])
        h = orc.rms_norm(x, t[f"{i}.ln2"], s.eps)
        gate, up = F.linear(h, t[f"{i}.gu"]).chunk(2, dim=-1)
        x = x + F.linear(F.silu(gate) * up, t[f"{i}.down"])
    return orc.rms_norm(x, t["norm"], s.eps)


def logits(w: Qwen3Weights, hidden: Tensor) -> Tensor:
    return F.linear(hidden, w.t["lm_head"]).float()


def oracle_attention(w: Qwen3Weights, caches: list[tuple[Tensor, Tensor]], meta: orc.OracleMeta,
                     cos_rows: Tensor, sin_rows: Tensor) -> AttentionStep:
    """The reference's attention step (qwen3.py:94-99) through the oracle, on any device."""
    s = w.s

    def step(i: int, qkv: Tensor) -> Tensor:
        q, k, v = orc.norm_rope(qkv, w.t[f"{i}.qn"], w.t[f"{i}.kn"], s.eps, cos_rows, sin_rows,
                                s.heads, s.kv_heads, s.head_dim)
        out = orc.paged_attention(q, k, v, caches[i][0], caches[i][1], meta, s.head_dim**-0.5)
        return out.reshape(qkv.shape[0], s.heads * s.head_dim)

    return step
