"""The drop-in inside MiniServe itself, on the CPU.

INTEGRATION.md gives the three edits a maintainer makes in MiniServe: the runner imports
``build_attention_metadata`` / ``MAX_GATHER_TOKENS`` / ``SeqChunk`` from ``miniserve_b200.attention``
(src/miniserve/runner/model_runner.py:20-25), ``ModelRunner.allocate_kv_cache``
(model_runner.py:77-94) allocates the pool with ``miniserve_b200.kv_pool.allocate_kv_cache``, and
the model uses ``miniserve_b200.qwen3_attention.Qwen3Attention`` in place of its own class
(src/miniserve/model/qwen3.py:65-100).  These tests apply exactly those edits to the reference's
unmodified source tree (by monkeypatching its modules) and drive its own ``LLMEngine`` and
``ModelRunner`` through them.

There is no GPU here, so libmsattn.so's device entry points are served by ``capi_emulator``,
which does the reference's own math (through the oracle) on the memory behind the pointers each
call receives; the planner and the rest of the host code are the real library.  What is checked
is the wiring: the greedy tokens the engine generates with the edits equal the unmodified
engine's exactly (bf16 on the CPU, the same ops), the KV pool in the new layout holds exactly the
reference pool's contents, every C-ABI call gets the shapes and strides the reference's tensors
have, the plans cover every kernel family, and ``profile_num_blocks`` sizes the new pool
correctly through the swapped path.  The kernels themselves are checked on a B200 by the ``gpu``
tests.

Skipped where the reference's source tree is absent (set MINISERVE_SRC to its ``src`` folder).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
_SRC = Path(os.environ.get("MINISERVE_SRC", ROOT.parent / "reference" / "src"))
if not (_SRC / "miniserve" / "__init__.py").exists():
    pytest.skip("MiniServe's source tree is not available", allow_module_level=True)
if str(_SRC) not in sys.path:
    sys.path.insert(0, str(_SRC))
transformers = pytest.importorskip("transformers")

import miniserve.model.qwen3 as ref_qwen3  # noqa: E402
import miniserve.runner.model_runner as ref_runner  # noqa: E402
from miniserve.config import EngineConfig  # noqa: E402
from miniserve.engine.engine import LLMEngine  # noqa: E402
from miniserve.engine.scheduler import ScheduledSeq  # noqa: E402
from miniserve.engine.sequence import SamplingParams, Sequence  # noqa: E402
from miniserve.model.loader import from_hf_model  # noqa: E402

import miniserve_b200.attention as ms_attention  # noqa: E402
import miniserve_b200.qwen3_attention as ms_qwen3  # noqa: E402
from capi_emulator import EmulatedLib  # noqa: E402
from miniserve_b200 import _capi, kv_pool  # noqa: E402

# Reference-style tiny model, but with the head geometry the sm_100a path serves (head_dim 128,
# two query heads per KV head) and 16-token blocks.
TINY = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
            num_attention_heads=4, num_key_value_heads=2, head_dim=128,
            max_position_embeddings=2048, rms_norm_eps=1e-6, tie_word_embeddings=True)
EOS_ID = 3
N_OUT = 12
GREEDY = SamplingParams(max_tokens=N_OUT, temperature=0.0, ignore_eos=True)


def _hf_model():
    torch.manual_seed(0)
    model = transformers.Qwen3ForCausalLM(transformers.Qwen3Config(**TINY))
    return model.to(torch.bfloat16).eval()


def allocate_kv_cache_edit(self, num_blocks: int) -> None:
    """``ModelRunner.allocate_kv_cache`` as INTEGRATION.md edits it."""
    c = self.model_cfg
    self.kv_cache, self.kv_caches = None, []
    self.kv_cache, self.kv_caches = kv_pool.allocate_kv_cache(
        c.num_hidden_layers, num_blocks, c.num_key_value_heads, self.device, self.dtype)
    self.num_blocks = num_blocks


@pytest.fixture
def swapped(monkeypatch: pytest.MonkeyPatch) -> EmulatedLib:
    """Apply the three edits to the reference's modules; route device calls to the emulator."""
    lib = EmulatedLib()
    monkeypatch.setattr(ref_qwen3, "Qwen3Attention", ms_qwen3.Qwen3Attention)
    monkeypatch.setattr(ref_runner, "build_attention_metadata", ms_attention.build_attention_metadata)
    monkeypatch.setattr(ref_runner, "MAX_GATHER_TOKENS", ms_attention.MAX_GATHER_TOKENS)
    monkeypatch.setattr(ref_runner, "SeqChunk", ms_attention.SeqChunk)
    monkeypatch.setattr(ref_runner.ModelRunner, "allocate_kv_cache", allocate_kv_cache_edit)
    # No GPU: the emulator stands in for the device entry points, the plan stays in host memory
    # and streams are a placeholder.
    monkeypatch.setattr(_capi, "load", lambda path=None: lib)
    monkeypatch.setattr(ms_attention, "_num_sms", lambda device: 148)
    monkeypatch.setattr(ms_attention, "_upload_plan", lambda packed, device: torch.from_numpy(packed))
    monkeypatch.setattr(ms_attention, "_stream", lambda device: 0)
    monkeypatch.setattr(ms_qwen3, "_stream", lambda device: 0)
    return lib


def _engine(hf, **over) -> LLMEngine:
    settings = dict(model="tiny-qwen3-d128", device="cpu", dtype="bfloat16", block_size=16,
                    max_model_len=1024, num_gpu_blocks=640, max_num_seqs=80,
                    max_num_batched_tokens=512)
    settings.update(over)
    cfg = EngineConfig(**settings)
    max_positions = cfg.max_model_len + cfg.num_speculative_tokens + 1
    model = from_hf_model(hf, torch.device("cpu"), torch.bfloat16, max_positions)
    return LLMEngine(cfg, model=model, eos_token_ids=[EOS_ID])


def _prompts() -> list[list[int]]:
    g = torch.Generator().manual_seed(1)
    # > 64 tokens (tensor-core items), 9-64 (tile items), <= 8 (decode items) ...
    solo = [torch.randint(4, 512, (n,), generator=g).tolist() for n in (300, 150, 40, 17, 5)]
    # ... and 70 prompts sharing a 272-token prefix (17 cached blocks under prefix caching), whose
    # decode rows form a shared-prefix (cascade) group (a group needs more than 64 query tokens).
    prefix = torch.randint(4, 512, (272,), generator=g).tolist()
    shared = [prefix + torch.randint(4, 512, (3 + n % 17,), generator=g).tolist()
              for n in range(70)]
    return solo + shared


@pytest.mark.parametrize("over", [{}, {"speculative": "ngram", "num_speculative_tokens": 4},
                                  {"max_num_batched_tokens": 96}],
                         ids=["default", "spec-ngram", "chunked-prefill"])
def test_engine_generates_the_reference_tokens(over, swapped: EmulatedLib) -> None:
    hf = _hf_model()
    prompts = _prompts()
    ours_engine = _engine(hf, **over)
    assert isinstance(ours_engine.model.layers[0].self_attn, ms_qwen3.Qwen3Attention)
    ours = ours_engine.generate(prompts, GREEDY)

    with pytest.MonkeyPatch.context() as undo:  # the unmodified reference, same weights
        undo.setattr(ref_qwen3, "Qwen3Attention", _ORIG_ATTENTION)
        undo.setattr(ref_runner, "build_attention_metadata", _ORIG_BUILD)
        undo.setattr(ref_runner, "MAX_GATHER_TOKENS", _ORIG_MAX_GATHER)
        undo.setattr(ref_runner, "SeqChunk", _ORIG_SEQCHUNK)
        undo.setattr(ref_runner.ModelRunner, "allocate_kv_cache", _ORIG_ALLOC)
        ref_engine = _engine(hf, **over)
        assert isinstance(ref_engine.model.layers[0].self_attn, _ORIG_ATTENTION)
        ref = ref_engine.generate(prompts, GREEDY)
    assert ours == ref

    # The new pool holds exactly what the reference's pool holds, slot for slot.
    c = ours_engine.model.cfg
    for layer in range(c.num_hidden_layers):
        k_view, v_view = ours_engine.runner.kv_caches[layer]
        assert torch.equal(kv_pool.layer_as_slots(k_view), ref_engine.runner.kv_cache[layer, 0])
        assert torch.equal(kv_pool.layer_as_slots(v_view), ref_engine.runner.kv_cache[layer, 1])

    # Every call got the reference tensors' geometry; the plans reached every kernel family.
    kinds = [k for k, _ in swapped.calls]
    steps = kinds.count("ms_plan_build")
    assert steps > 0
    assert kinds.count("ms_qk_norm_rope_scatter") == steps * c.num_hidden_layers
    assert kinds.count("ms_paged_attention") == steps * c.num_hidden_layers
    width = (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim
    for kind, a in swapped.calls:
        if kind == "ms_qk_norm_rope_scatter":
            assert a["num_heads"] == c.num_attention_heads and a["num_kv_heads"] == c.num_key_value_heads
            assert a["qkv_row_stride"] == width  # the qkv_proj output, split in place
            assert a["q_out_row_stride"] == c.num_attention_heads * c.head_dim
            assert a["cs_row_stride"] == c.head_dim and not a["positions"]  # gathered rows
            assert a["eps"] == pytest.approx(c.rms_norm_eps)
        if kind == "ms_paged_attention":
            assert a["scale"] == pytest.approx(c.head_dim**-0.5)
    attn = [a for k, a in swapped.calls if k == "ms_paged_attention"]
    assert any(a["n_tc_items"] for a in attn) and any(a["n_tile_items"] for a in attn)
    assert any(a["n_decode_items"] for a in attn)
    if not over:
        assert any(a["n_cascade"] for a in attn), "no step formed a shared-prefix group"
    if "speculative" in over:
        assert any(any(1 < ch.num_new <= 8 for ch in a["chunks"]) for a in attn), \
            "no speculative verify query reached the attention"


def test_profile_num_blocks_through_the_drop_in(swapped: EmulatedLib,
                                                monkeypatch: pytest.MonkeyPatch) -> None:
    """``ModelRunner.profile_num_blocks`` (model_runner.py:97-155) with the edits: its two dummy
    steps (the biggest prefill; ``max_num_seqs`` decodes sized by ``MAX_GATHER_TOKENS``) run
    through the drop-in, and its pool size matches the new layout's real bytes per block.  The
    CUDA memory counters are faked (no GPU here): a fixed weight and activation footprint plus
    the live pool's actual size."""
    hf = _hf_model()
    cfg = EngineConfig(model="tiny-qwen3-d128", device="cpu", dtype="bfloat16", block_size=16,
                       max_model_len=1024, num_gpu_blocks=320, max_num_seqs=24,
                       max_num_batched_tokens=512)
    model = from_hf_model(hf, torch.device("cpu"), torch.bfloat16, cfg.max_model_len + 1)
    runner = ref_runner.ModelRunner(cfg, model.cfg, model, torch.device("cuda"), torch.bfloat16)

    weights, activations, total = 1 << 30, 3 << 28, 180 << 30

    def pool_bytes() -> int:
        return 0 if runner.kv_cache is None else runner.kv_cache.numel() * 2

    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(torch.cuda, "reset_peak_memory_stats", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "memory_allocated", lambda *a, **k: weights + pool_bytes())
    monkeypatch.setattr(torch.cuda, "max_memory_allocated",
                        lambda *a, **k: weights + pool_bytes() + activations)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda *a, **k: (total - weights, total))
    monkeypatch.setattr(ref_runner, "to_device",
                        lambda data, device, dtype=torch.long: torch.tensor(data, dtype=dtype))
    sizes = []

    def alloc_on_host(self, num_blocks: int) -> None:
        c = self.model_cfg
        self.kv_cache, self.kv_caches = kv_pool.allocate_kv_cache(
            c.num_hidden_layers, num_blocks, c.num_key_value_heads, "cpu", self.dtype)
        self.num_blocks = num_blocks
        sizes.append((num_blocks, self.kv_cache.numel() * 2))

    monkeypatch.setattr(ref_runner.ModelRunner, "allocate_kv_cache", alloc_on_host)
    num_blocks = runner.profile_num_blocks()

    # The pool profile_num_blocks allocated: its real bytes per block are the runner's figure.
    (pool_blocks, nbytes), = sizes
    assert nbytes == pool_blocks * runner.bytes_per_block
    budget = total * cfg.gpu_memory_utilization - weights - activations
    assert num_blocks == int(budget // runner.bytes_per_block)
    # Both dummy steps went through the drop-in's planner and kernels.
    plans = [a for k, a in swapped.calls if k == "ms_plan_build"]
    prefill_len = min(cfg.max_num_batched_tokens, cfg.max_model_len - 1)
    assert plans[0]["num_seqs"] == 1 and plans[0]["num_tokens"] == prefill_len
    assert plans[1]["num_seqs"] == cfg.max_num_seqs and plans[1]["num_tokens"] == cfg.max_num_seqs
    attn = [a for k, a in swapped.calls if k == "ms_paged_attention"]
    ctx = ms_attention.MAX_GATHER_TOKENS // cfg.max_num_seqs - 1
    assert all(ch.context_len == ctx + 1 for ch in attn[-1]["chunks"])


def test_runner_prepare_feeds_the_drop_in(swapped: EmulatedLib) -> None:
    """``ModelRunner.prepare`` (model_runner.py:162-205) hands the reference's own SeqChunk
    objects and int64 slot mapping to the drop-in ``build_attention_metadata``, whose plan
    records each sequence exactly as the chunk describes it."""
    hf = _hf_model()
    eng = _engine(hf)
    runner = eng.runner
    seqs = []
    for i, (n, cached) in enumerate([(70, 0), (1, 300), (5, 64), (20, 33)]):
        s = Sequence(f"s{i}", list(range(4, 4 + cached + n)), SamplingParams())
        s.block_table = list(range(20 * i, 20 * i + -(-(cached + n) // 16)))
        s.num_computed = cached
        seqs.append(ScheduledSeq(s, n))
    inp = runner.prepare(seqs)
    meta = inp.attn
    assert isinstance(meta, ms_attention.AttentionMetadata)
    assert meta.slot_mapping.dtype == torch.int64 and meta.num_tokens == 96
    plan = meta.plan.numpy()
    info = meta.info
    for i, sch in enumerate(seqs):
        rec = plan[info.off_seqs + 8 * i : info.off_seqs + 8 * i + 6].tolist()
        flat = sum(x.num_new_tokens for x in seqs[:i])
        n, c = sch.num_new_tokens, sch.seq.num_computed
        assert rec[:4] == [flat, n, c, c + n]
        table = plan[info.off_tables + rec[4] : info.off_tables + rec[4] + rec[5]].tolist()
        assert table == sch.seq.block_table
    expect = [t[p // 16] * 16 + p % 16 for s in seqs
              for t in [s.seq.block_table] for p in range(s.seq.num_computed,
                                                          s.seq.num_computed + s.num_new_tokens)]
    assert meta.slot_mapping.tolist() == expect


_ORIG_ATTENTION = ref_qwen3.Qwen3Attention
_ORIG_BUILD = ref_runner.build_attention_metadata
_ORIG_MAX_GATHER = ref_runner.MAX_GATHER_TOKENS
_ORIG_SEQCHUNK = ref_runner.SeqChunk
_ORIG_ALLOC = ref_runner.ModelRunner.allocate_kv_cache
