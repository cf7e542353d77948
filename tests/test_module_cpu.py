"""Host logic of the drop-in ``Qwen3Attention`` (no GPU): which projection path ``forward`` takes
for each ``fused_qkv`` setting, and the setting's validation.  The CUDA entry points are replaced
by recorders, so nothing here launches a kernel.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from miniserve_b200 import qwen3_attention as qa

HIDDEN = 64


def _cfg(fused):
    return SimpleNamespace(num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                           hidden_size=HIDDEN, rms_norm_eps=1e-6, fused_qkv=fused)


def _run(monkeypatch, fused, tokens: int) -> list[str]:
    calls: list[str] = []

    def fused_path(x, *args, **kwargs):
        calls.append("kernel_e")
        return torch.zeros(x.shape[0], 16, 128)

    def split_path(qkv, *args, **kwargs):
        assert qkv.shape == (tokens, 16 * 128 + 2 * 8 * 128)
        calls.append("cublas+kernel_a")
        return torch.zeros(qkv.shape[0], 16, 128)

    monkeypatch.setattr(qa, "qkv_proj_norm_rope_scatter", fused_path)
    monkeypatch.setattr(qa, "qk_norm_rope_scatter", split_path)
    monkeypatch.setattr(qa, "attend", lambda q, *a, **k: torch.zeros_like(q))
    mod = qa.Qwen3Attention(_cfg(fused))
    x = torch.zeros(tokens, HIDDEN)
    out = mod(x, None, None, None, None, SimpleNamespace(slot_mapping=None))
    assert out.shape == (tokens, HIDDEN)
    return calls


@pytest.mark.parametrize("tokens", [1, 256, qa.FUSED_QKV_MIN_TOKENS - 1, qa.FUSED_QKV_MIN_TOKENS,
                                    4096])
def test_fused_qkv_dispatch(monkeypatch, tokens: int) -> None:
    assert _run(monkeypatch, False, tokens) == ["cublas+kernel_a"]
    assert _run(monkeypatch, True, tokens) == ["kernel_e"]
    expect = "kernel_e" if tokens >= qa.FUSED_QKV_MIN_TOKENS else "cublas+kernel_a"
    assert _run(monkeypatch, "auto", tokens) == [expect]


def test_fused_qkv_default_is_off(monkeypatch) -> None:
    cfg = _cfg(False)
    del cfg.fused_qkv
    assert qa.Qwen3Attention(cfg).fused_qkv is False


@pytest.mark.parametrize("bad", ["yes", "on", 1.5, None])
def test_fused_qkv_rejects_unknown_settings(bad) -> None:
    with pytest.raises(ValueError):
        qa.Qwen3Attention(_cfg(bad))
