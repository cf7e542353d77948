"""Benchmark of MiniServe's per-step paged-attention path on B200.

Headline workload (config 2 of the path's benchmark set): one decode step of Qwen3-0.6B's
attention path over all 28 layers for 256 sequences per GPU with context lengths U[256, 4096]
(one new token each), 16 query / 8 KV heads, head_dim 128, 16-token blocks, a KV pool of 1.1x
the blocks needed per layer with randomly permuted block tables, N(0,1) bf16 values (synthetic;
no model weights are involved on this path).  A "step" = for each of the 28 layers: kernel A
(q/k RMSNorm + RoPE + K/V scatter) and the attention kernels (paged split-KV attention + combine).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (launched by torchrun) the global batch is N x 256 rows -- N copies of the single-GPU
batch's context lengths -- sharded over the ranks by context tokens (greedy LPT), so every GPU
streams the same bytes as at N = 1 (weak scaling) with no data-path collective; the time is the
max over ranks.  The same line also reports, as extra keys, config 3 (mixed prefill, the
tensor-core kernel), config 4 (shared prefix + speculative verify, the cascade path) and config 5
(box scale: 8,192 rows sharded over the N GPUs, strong scaling), each with its own roofline.
``--impl reference`` times the reference algorithm (the CPU oracle restating MiniServe's torch
code) on the host cores on the same batch.

Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS = 28
H, KVH, D = 16, 8, 128
METRIC = "decode tok/s (paged-attn path, 28 layers, config 2)"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
SEED = 1000  # every workload's batch geometry (config 5: its own seed 0)


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seqs", type=int, default=256)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--pages-per-split", type=int, default=0)
    p.add_argument("--no-graph", action="store_true",
                   help="time eager launches instead of replaying the captured step")
    p.add_argument("--layers", type=int, default=LAYERS,
                   help="layers per step (28 for the headline; fewer only for small profiles)")
    p.add_argument("--tokens", type=int, default=4096,
                   help="--workload qkv: tokens per step")
    p.add_argument("--workload", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "qkv", "prefill"],
                   default="cfg2",
                   help="cfg2 is the headline; cfg1 (8 short decode rows), cfg3 (mixed prefill), "
                        "cfg4 (prefix + verify) and cfg5 (box scale: 8192 rows sharded over the "
                        "ranks) alone; qkv times kernel E (qkv projection + norm/RoPE/scatter) "
                        "beside cuBLAS + kernel A at --tokens tokens; prefill times the tensor-core "
                        "kernel alone on config 3's chunks and on fresh prompts")
    p.add_argument("--no-extras", action="store_true",
                   help="headline only: skip the config 3 / 4 / 5 keys")
    p.add_argument("--no-qkv-part", action="store_true",
                   help="skip timing kernel E (qkv projection + norm/RoPE/scatter) beside "
                        "cuBLAS + kernel A")
    p.add_argument("--pool-gb", type=float, default=150.0,
                   help="cfg5: per-GPU pool shared by all layers")
    return p.parse_args()


def peaks() -> tuple[dict, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return json.loads(f.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def traffic_per_unit(key: str) -> dict | None:
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    return json.loads(f.read_text()).get(key)


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen | None = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------------------------


def make_batch(name: str, rank: int, world: int, seqs: int = 256, pool_gb: float = 150.0):
    """This rank's batch of a workload.  Configs 1, 3 and 4 are single-GPU configurations: every
    rank runs the same batch.  Config 2 shards N copies of the single-GPU batch, config 5 its
    8,192 rows, by context tokens."""
    from miniserve_b200.workloads import config1, config2, config3, config4, config5

    if name == "cfg1":
        return config1(seed=SEED)
    if name == "cfg2":
        return config2(seed=SEED, num_seqs=seqs, rank=rank, world=world)
    if name == "cfg3":
        return config3(seed=SEED)
    if name == "cfg4":
        return config4(seed=SEED)
    return config5(rank, world, seed=0, pool_bytes=pool_gb * 1e9)


def workload_label(name: str, world: int, seqs: int = 256, layers: int = LAYERS,
                   pool_gb: float = 150.0) -> str:
    return {
        "cfg1": "config1: 8 decode seqs, ctx U[1,512], pool 1070 blocks",
        "cfg2": (f"config2: {seqs} decode seqs/GPU (global batch {seqs * world}, LPT-sharded by "
                 f"context tokens), ctx U[256,4096], 16q/8kv heads, d128, block 16, {layers} layers"),
        "cfg3": "config3: 48 decode rows ctx U[128,2048] + 2 chunks x 1000 tokens over 512 cached",
        "cfg4": ("config4: 512 rows sharing a 1024-token prefix (64 blocks), U[64,256] own tokens, "
                 "5-token verify queries"),
        "cfg5": (f"config5: 8192 decode seqs in total, ctx logU[512,32768], LPT-sharded by tokens "
                 f"over {world} GPU(s), one {pool_gb:.0f} GB pool per GPU shared by the 28 layers"),
    }[name]


def headline_config(world: int, seqs: int, layers: int) -> dict:
    """The `config` object of the headline line, identical in both arms."""
    return {
        "workload": workload_label("cfg2", world, seqs, layers),
        "layers": layers,
        "l2": "inputs larger than L2 (KV read per layer-step ~2.2 GB >> 126 MB)",
        "parallelism": f"sequence-sharded x{world}, no data-path collective",
    }


def attention_bytes(batch) -> tuple[int, int, int]:
    """Algorithmic bytes of one attention launch (kernels B+C/D), of one kernel-A launch, and the
    attention FLOPs (causal pairs only).

    Attention bytes: every distinct physical KV block's K and V of each KV head once (bf16; a
    shared prefix block counts once), the queries in and the outputs out, and the block-table
    entries.  Kernel A: the qkv row read, q written, K and V written to the pool, cos/sin rows and
    the slot/position indices.  FLOPs: 4 * 128 * 16 heads per (query token, visible key).
    """
    # A pool shared by all layers (config 5) still streams every context token from HBM, since
    # the pool is far larger than L2: count the logical tokens there.
    kv_tokens = batch.kv_tokens_read() if getattr(batch, "aliased", False) else batch.unique_kv_tokens()
    t = batch.num_tokens
    tables = sum(-(-c.context_len // 16) for c in batch.chunks)
    attn = kv_tokens * KVH * D * 2 * 2 + t * H * D * 2 * 2 + tables * 4
    kern_a = t * (H + 2 * KVH) * D * 2 + t * H * D * 2 + t * 2 * KVH * D * 2 + t * D * 4 * 2 + t * 8
    pairs = sum(c.num_new * c.num_cached + c.num_new * (c.num_new + 1) // 2 for c in batch.chunks)
    return attn, kern_a, 4 * D * H * pairs


class DeviceStep:
    """One workload's step on this GPU: ``layers`` x (kernel A, attention), every input resident
    in HBM, the plan built and uploaded once (it is per step, shared by the layers)."""

    def __init__(self, batch, layers: int, device: torch.device, pages_per_split: int = 0,
                 seed: int = 1234) -> None:
        from miniserve_b200.attention import build_attention_metadata
        from miniserve_b200.kv_pool import allocate_kv_cache
        from miniserve_b200.workloads import rope_tables

        self.batch, self.layers, self.device = batch, layers, device
        self.alias = bool(getattr(batch, "aliased", False)) or batch.name.startswith("cfg5")
        t = batch.num_tokens
        g = torch.Generator(device=device).manual_seed(seed)
        self.pool, views = allocate_kv_cache(1 if self.alias else layers, batch.num_blocks, KVH,
                                             device, zero=False)
        for layer in range(self.pool.shape[0]):
            self.pool[layer].normal_(generator=g)
        # Config 5: one pool shared by all layers (it cannot hold 28 separate ones).
        self.views = views * layers if self.alias else views
        self.qkv_all = torch.randn(layers, t, (H + 2 * KVH) * D, generator=g, device=device,
                                   dtype=torch.bfloat16)
        self.qw = (1 + 0.1 * torch.randn(layers, D, generator=g, device=device)).bfloat16()
        self.kw = (1 + 0.1 * torch.randn(layers, D, generator=g, device=device)).bfloat16()
        self.cos_t, self.sin_t = rope_tables(D, batch.max_position + 8, 1e6, device)
        positions = torch.from_numpy(batch.positions).to(device)
        self.slot_mapping = torch.from_numpy(batch.slots).to(device)
        self.cos, self.sin = self.cos_t[positions], self.sin_t[positions]
        self.pages_per_split = pages_per_split
        self.meta = build_attention_metadata(batch.chunks, self.slot_mapping, 16,
                                             pages_per_split=pages_per_split)
        self.q_buf = torch.empty(t, H, D, dtype=torch.bfloat16, device=device)
        self.out_all = torch.empty(layers, t, H, D, dtype=torch.bfloat16, device=device)
        self.stream = torch.cuda.current_stream(device)
        info = self.meta.info
        self.launches_per_layer = (1 + (info.n_decode_items > 0) + (info.n_tile_items > 0)
                                   + (info.n_tc_items > 0) + (info.n_combine > 0))
        self.ev_attn = [[torch.cuda.Event(enable_timing=True) for _ in range(2)]
                        for _ in range(layers)]
        self.graph: torch.cuda.CUDAGraph | None = None

    def step(self, timed_kernels: bool = False) -> None:
        from miniserve_b200.attention import attend
        from miniserve_b200.qwen3_attention import qk_norm_rope_scatter

        for layer in range(self.layers):
            k_cache, v_cache = self.views[layer]
            qk_norm_rope_scatter(self.qkv_all[layer], self.qw[layer], self.kw[layer], 1e-6,
                                 self.cos, self.sin, self.slot_mapping, k_cache, v_cache, H,
                                 q_out=self.q_buf)
            if timed_kernels:
                self.ev_attn[layer][0].record(self.stream)
            attend(self.q_buf, k_cache, v_cache, self.meta, D**-0.5, out=self.out_all[layer])
            if timed_kernels:
                self.ev_attn[layer][1].record(self.stream)

    def check_status(self, when: str) -> None:
        from miniserve_b200 import _capi

        status = _capi.device_status(int(self.stream.cuda_stream))
        if status:
            raise RuntimeError(f"device status {status:#x} {when}")

    def capture(self) -> None:
        """The whole step as one CUDA graph (the C-ABI calls neither allocate nor synchronise)."""
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()
        for _ in range(2):
            self.graph.replay()
        torch.cuda.synchronize(self.device)

    def timed(self, fn, steps: int, world: int) -> float:
        """Milliseconds for ``steps`` calls of ``fn``: barrier + synchronize on both sides, CUDA
        events on the launching stream."""
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(self.device)
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(self.stream)
        for _ in range(steps):
            fn()
        stop.record(self.stream)
        torch.cuda.synchronize(self.device)
        return start.elapsed_time(stop)

    def attention_launch_ms(self, reps: int) -> float:
        """Mean CUDA-event duration of the attention launches (events around each layer's
        attention call, on the stream it launches on)."""
        ms: list[float] = []
        for _ in range(max(1, reps)):
            self.step(timed_kernels=True)
            torch.cuda.synchronize(self.device)
            ms.extend(self.ev_attn[layer][0].elapsed_time(self.ev_attn[layer][1])
                      for layer in range(self.layers))
        return float(np.mean(ms))

    def part_us(self, chunks, reps: int = 10) -> float:
        """One attention call over a subset of the rows, alone: CUDA-graph replay of ``reps``
        calls on layer 0's pool, microseconds per call."""
        from miniserve_b200.attention import attend, build_attention_metadata

        k_cache, v_cache = self.views[0]
        sub_meta = build_attention_metadata(chunks, self.slot_mapping, 16,
                                            pages_per_split=self.pages_per_split)
        attend(self.q_buf, k_cache, v_cache, sub_meta, D**-0.5, out=self.out_all[0])
        torch.cuda.synchronize(self.device)
        g_sub = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_sub):
            for _ in range(reps):
                attend(self.q_buf, k_cache, v_cache, sub_meta, D**-0.5, out=self.out_all[0])
        g_sub.replay()
        torch.cuda.synchronize(self.device)
        best = float("inf")
        for _ in range(3):
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(self.stream)
            g_sub.replay()
            p1.record(self.stream)
            torch.cuda.synchronize(self.device)
            best = min(best, p0.elapsed_time(p1) * 1e3 / reps)
        del g_sub
        return best

    def release(self) -> None:
        self.graph = None
        for name in ("pool", "views", "qkv_all", "out_all", "q_buf", "meta", "cos", "sin"):
            setattr(self, name, None)
        torch.cuda.synchronize(self.device)
        torch.cuda.empty_cache()


def roofline_hbm(kernel: str, nbytes: float, us: float, traffic: float | None) -> dict:
    pk, src = peaks()
    hbm = float(pk["hbm_gbs"])
    achieved = nbytes / (us * 1e-6) / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": hbm,
            "peak_source": f"{src} (hbm_gbs: copy bandwidth)", "unit": "GB/s",
            "frac": achieved / hbm, "traffic": traffic, "algorithmic_bytes_per_launch": nbytes}


def roofline_tensor(kernel: str, flops: float, us: float, traffic: float | None) -> dict:
    pk, src = peaks()
    burst = float(pk["bf16_tflops"])
    sustained = float(pk.get("bf16_tflops_sustained", burst))
    achieved = flops / (us * 1e-6) / 1e12
    return {"kernel": kernel, "bound": "tensor", "achieved": achieved, "peak": burst,
            "peak_source": f"{src} (bf16_tflops: cuBLAS GEMM burst; timed alone)",
            "unit": "TFLOP/s", "frac": achieved / burst,
            "frac_of_sustained": achieved / sustained, "peak_sustained": sustained,
            "traffic": traffic, "algorithmic_flops_per_launch": flops}


def scaled_traffic(key: str, units: float) -> float | None:
    """ncu's DRAM bytes for a kernel, per unit of its work (from profiles/traffic.json), times
    the units this launch processes."""
    t = traffic_per_unit(key)
    if not t:
        return None
    return float(t["bytes_per_unit"]) * units


# ---------------------------------------------------------------------------------------------
# our implementation: the headline
# ---------------------------------------------------------------------------------------------


def time_qkv_projection(t: int, views, qw, kw, cos, sin, slot_mapping, layers: int,
                        device: torch.device, stream) -> dict:
    """Kernel E (the qkv projection with kernel A as its epilogue, qwen3.py:94-98 +
    backends.py:159-160) beside what it replaces, cuBLAS + kernel A, on this workload's tokens.
    Each layer has its own x [T, 1024] and W [4096, 1024] (28 x 8 MiB of weights > L2); both
    forms are captured as one CUDA graph over the layers and replayed."""
    from miniserve_b200.qwen3_attention import qk_norm_rope_scatter, qkv_proj_norm_rope_scatter

    hidden, width = 1024, (H + 2 * KVH) * D
    g = torch.Generator(device=device).manual_seed(4321)
    x = torch.randn(layers, t, hidden, generator=g, device=device, dtype=torch.bfloat16)
    w = (torch.randn(layers, width, hidden, generator=g, device=device) / 32).bfloat16()
    qkv = torch.empty(t, width, dtype=torch.bfloat16, device=device)
    q_buf = torch.empty(t, H, D, dtype=torch.bfloat16, device=device)

    def fused() -> None:
        for layer in range(layers):
            qkv_proj_norm_rope_scatter(x[layer], w[layer], qw[layer], kw[layer], 1e-6, cos, sin,
                                       slot_mapping, *views[layer], H, q_out=q_buf)

    def unfused() -> None:
        for layer in range(layers):
            torch.matmul(x[layer], w[layer].t(), out=qkv)
            qk_norm_rope_scatter(qkv, qw[layer], kw[layer], 1e-6, cos, sin, slot_mapping,
                                 *views[layer], H, q_out=q_buf)

    res = {}
    for name, fn in (("fused_kernel_e", fused), ("cublas_plus_kernel_a", unfused)):
        fn()
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize(device)
        res[name] = e0.elapsed_time(e1) * 1e3 / (5 * layers)
        del graph
    pk, src = peaks()
    flops = 2.0 * t * hidden * width
    # W and x read once, q and the K/V rows written once (the projection output is not stored).
    nbytes = 2.0 * (width * hidden + t * hidden + t * width)
    us = res["fused_kernel_e"]
    floor_us = max(flops / (float(pk["bf16_tflops"]) * 1e12),
                   nbytes / (float(pk["hbm_gbs"]) * 1e9)) * 1e6
    # Back-to-back tensor-core launches run at the power-capped clock: the sustained GEMM figure
    # is the matching denominator for the large-token cases.
    sustained = float(pk.get("bf16_tflops_sustained", pk["bf16_tflops"]))
    floor_sustained_us = max(flops / (sustained * 1e12),
                             nbytes / (float(pk["hbm_gbs"]) * 1e9)) * 1e6
    return {
        "tokens": t,
        "hidden": hidden,
        "us_per_layer": {k: round(v, 2) for k, v in res.items()},
        "speedup_vs_cublas_plus_a": res["cublas_plus_kernel_a"] / us,
        "fused_TFLOPS": flops / (us * 1e-6) / 1e12,
        "fused_GBps_algorithmic": nbytes / (us * 1e-6) / 1e9,
        "roofline_floor_us": floor_us,
        "frac_of_roofline": floor_us / us,
        "frac_of_sustained_roofline": floor_sustained_us / us,
        "peak_source": src,
        "timing": f"CUDA-graph replay of {layers} layers x 5, per layer; distinct W per layer",
    }


def run_qkv_only(args: argparse.Namespace, rank: int, device: torch.device) -> None:
    """--workload qkv: kernel E beside cuBLAS + kernel A on --tokens tokens (one sequence's
    prefill positions, a permuted pool), --layers distinct layers per timed pass."""
    from miniserve_b200 import _capi
    from miniserve_b200.kv_pool import allocate_kv_cache
    from miniserve_b200.workloads import rope_tables

    if rank != 0:
        return
    t, layers = args.tokens, args.layers
    nb = (t + 15) // 16 + 8
    _pool, views = allocate_kv_cache(layers, nb, KVH, device)
    g = torch.Generator(device=device).manual_seed(7)
    qw = (1 + 0.1 * torch.randn(layers, D, generator=g, device=device)).bfloat16()
    kw = (1 + 0.1 * torch.randn(layers, D, generator=g, device=device)).bfloat16()
    cos_t, sin_t = rope_tables(D, t + 8, 1e6, device)
    positions = torch.arange(t, device=device)
    cos, sin = cos_t[positions], sin_t[positions]
    slots = torch.randperm(nb * 16, generator=g, device=device)[:t]
    stream = torch.cuda.current_stream(device)
    r = time_qkv_projection(t, views, qw, kw, cos, sin, slots, layers, device, stream)
    status = _capi.device_status(int(stream.cuda_stream))
    if status:
        raise RuntimeError(f"device status {status:#x}")
    print(json.dumps({"metric": "qkv projection + q/k norm + RoPE + K/V scatter (us per layer)",
                      "value": r["us_per_layer"]["fused_kernel_e"], "unit": "us",
                      "higher_is_better": False, "n_gpus": 1, "dtype": "bf16",
                      "data": "synthetic", "config": {"workload": f"qkv: {t} tokens, hidden "
                                                      f"1024, 16q/8kv heads, {layers} layers"},
                      "qkv_projection": r}), flush=True)


def run_prefill_only(rank: int, device: torch.device) -> None:
    """--workload prefill: the attention call alone on prefill-only batches (the tensor-core
    kernel, plus the combine pass where a plan splits tiles): config 3's two chunks, fresh prompts
    of 2048 / 4096 / 8192 tokens and 1024 new tokens over 8192 cached.  CUDA-graph replay of 10
    calls, best of 5 replays; causal FLOPs against the measured bf16 peak."""
    from miniserve_b200 import _capi
    from miniserve_b200.attention import attend, build_attention_metadata
    from miniserve_b200.kv_pool import allocate_kv_cache
    from miniserve_b200.workloads import config3, custom

    if rank != 0:
        return
    pk, src = peaks()
    burst = float(pk["bf16_tflops"])
    sustained = float(pk.get("bf16_tflops_sustained", burst))
    cases = {
        "config3_chunks": [c for c in config3(seed=SEED).chunks if c.num_new > 64],
        "fresh_2048": custom([(2048, 0)], seed=1).chunks,
        "fresh_4096": custom([(4096, 0)], seed=1).chunks,
        "fresh_8192": custom([(8192, 0)], seed=1).chunks,
        "1024_over_8192": custom([(1024, 8192)], seed=1).chunks,
    }
    stream = torch.cuda.current_stream(device)
    res = {}
    for name, chunks in cases.items():
        nb = max(b for c in chunks for b in c.block_table) + 1
        t = max(c.flat_start + c.num_new for c in chunks)
        g = torch.Generator(device=device).manual_seed(3)
        pool, views = allocate_kv_cache(1, nb, KVH, device, zero=False)
        pool.normal_(generator=g)
        kc, vc = views[0]
        q = torch.randn(t, H, D, generator=g, device=device).bfloat16()
        out = torch.empty_like(q)
        meta = build_attention_metadata(chunks, torch.zeros(t, dtype=torch.int64, device=device), 16)
        attend(q, kc, vc, meta, D**-0.5, out=out)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(10):
                attend(q, kc, vc, meta, D**-0.5, out=out)
        graph.replay()
        torch.cuda.synchronize(device)
        best = float("inf")
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(device)
            best = min(best, e0.elapsed_time(e1) * 1e3 / 10)
        del graph
        status = _capi.device_status(int(stream.cuda_stream))
        if status:
            raise RuntimeError(f"device status {status:#x} ({name})")
        pairs = sum(c.num_new * c.num_cached + c.num_new * (c.num_new + 1) // 2 for c in chunks)
        tflops = 4 * D * H * pairs / (best * 1e-6) / 1e12
        res[name] = {"us": round(best, 2), "TFLOPS_causal": round(tflops, 1),
                     "frac_of_burst": round(tflops / burst, 3),
                     "frac_of_sustained": round(tflops / sustained, 3),
                     "tc_items": int(meta.info.n_tc_items), "combine": int(meta.info.n_combine)}
    head = res["config3_chunks"]
    print(json.dumps({"metric": "prefill attention TFLOP/s (tensor-core kernel, config 3's chunks)",
                      "value": head["TFLOPS_causal"], "unit": "TFLOP/s", "higher_is_better": True,
                      "n_gpus": 1, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": "prefill-only attention calls"},
                      "peak_source": src, "cases": res,
                      "timing": "CUDA-graph replay of 10 calls, best of 5, per call"}), flush=True)


def run_e2e(ws: DeviceStep, args: argparse.Namespace, world: int
            ) -> tuple[float, float, int, int]:
    """The same step through the public Python API with host buffers: each step prepares its
    positions and slot mapping from the block tables (ms_prepare_step), plans (ms_plan_build)
    and uploads the plan, copies every layer's qkv up from pinned host memory and every layer's
    output back.  Two forms: eager (every layer's calls made from Python each step) and replayed
    (the device part of a step -- cos/sin rows, every layer's copies and kernels -- captured once
    as a CUDA graph; each step prepares and plans on the host, writes positions, slots and plan
    into the captured buffers with AttentionMetadata.update, and replays).  Returns (ms of the
    replayed form and of the eager form for args.steps steps, H2D bytes per step, D2H bytes per
    step)."""
    from miniserve_b200.attention import attend, build_attention_metadata, prepare_arrays
    from miniserve_b200.qwen3_attention import qk_norm_rope_scatter

    device, stream, batch = ws.device, ws.stream, ws.batch
    layers, t = ws.layers, batch.num_tokens
    qkv_host = ws.qkv_all.cpu().pin_memory()
    out_host = torch.empty(layers, t, H, D, dtype=torch.bfloat16).pin_memory()
    qkv_dev = torch.empty_like(ws.qkv_all)
    n_seq = len(batch.chunks)
    new_np = np.fromiter((c.num_new for c in batch.chunks), dtype=np.int32, count=n_seq)
    cached_np = np.fromiter((c.num_cached for c in batch.chunks), dtype=np.int32, count=n_seq)
    offsets_np = np.zeros(n_seq + 1, dtype=np.int64)
    np.cumsum([len(c.block_table) for c in batch.chunks], out=offsets_np[1:])
    tables_np = np.concatenate([np.asarray(c.block_table, dtype=np.int32) for c in batch.chunks])
    pos_bufs = [torch.empty(t, dtype=torch.int64).pin_memory() for _ in range(2)]
    slot_bufs = [torch.empty(t, dtype=torch.int64).pin_memory() for _ in range(2)]
    copies_done: list = [None, None]
    step_no = [0]
    copy_stream = torch.cuda.Stream(device)
    qkv_arrived = [torch.cuda.Event() for _ in range(layers)]
    qkv_consumed = [torch.cuda.Event() for _ in range(layers)]
    out_written = [torch.cuda.Event() for _ in range(layers)]
    first_step = [True]
    step_started = torch.cuda.Event()
    overlap_copies = qkv_host[0].numel() * 2 >= (1 << 20)  # per-layer copies of >= 1 MiB

    def e2e_step() -> None:
        k = step_no[0] & 1
        step_no[0] += 1
        if copies_done[k] is not None:
            copies_done[k].synchronize()  # the copy that read this buffer two steps ago is done
        prepare_arrays(new_np, cached_np, offsets_np, tables_np, pos_bufs[k].numpy(),
                       slot_bufs[k].numpy())
        slots_d = slot_bufs[k].to(device, non_blocking=True)
        pos_d = pos_bufs[k].to(device, non_blocking=True)
        done = torch.cuda.Event()
        done.record(stream)
        copies_done[k] = done
        m = build_attention_metadata(batch.chunks, slots_d, 16, pages_per_split=ws.pages_per_split)
        c, s = ws.cos_t[pos_d], ws.sin_t[pos_d]
        if not overlap_copies:
            # Small steps: two bulk copies cost less host time than per-layer stream choreography.
            qkv_dev.copy_(qkv_host, non_blocking=True)
            for layer in range(layers):
                k_cache, v_cache = ws.views[layer]
                q = qk_norm_rope_scatter(qkv_dev[layer], ws.qw[layer], ws.kw[layer], 1e-6, c, s,
                                         slots_d, k_cache, v_cache, H, q_out=ws.q_buf)
                attend(q, k_cache, v_cache, m, D**-0.5, out=ws.out_all[layer])
            out_host.copy_(ws.out_all, non_blocking=True)
            return
        # Each layer's qkv goes up, and its output comes back, on a copy stream, overlapped with
        # the other layers' kernels (as a serving engine pipelines them); the step ends when the
        # last output is on the host.
        step_started.record(stream)  # no copy of this step may run before the step begins
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(step_started)
            for layer in range(layers):
                if not first_step[0]:
                    copy_stream.wait_event(qkv_consumed[layer])
                qkv_dev[layer].copy_(qkv_host[layer], non_blocking=True)
                qkv_arrived[layer].record(copy_stream)
        for layer in range(layers):
            k_cache, v_cache = ws.views[layer]
            stream.wait_event(qkv_arrived[layer])
            q = qk_norm_rope_scatter(qkv_dev[layer], ws.qw[layer], ws.kw[layer], 1e-6, c, s,
                                     slots_d, k_cache, v_cache, H, q_out=ws.q_buf)
            qkv_consumed[layer].record(stream)
            attend(q, k_cache, v_cache, m, D**-0.5, out=ws.out_all[layer])
            out_written[layer].record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(out_written[layer])
                out_host[layer].copy_(ws.out_all[layer], non_blocking=True)
        stream.wait_stream(copy_stream)
        first_step[0] = False

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize(device)
    eager_ms = ws.timed(e2e_step, args.steps, world)

    # Replayed form.  Positions, slots and plan live in buffers the graph captured; the host
    # writes each step's values into them on the stream (after the previous replay's kernels).
    pos_dev = torch.empty(t, dtype=torch.int64, device=device)
    slot_dev = torch.empty(t, dtype=torch.int64, device=device)
    prepare_arrays(new_np, cached_np, offsets_np, tables_np, pos_bufs[0].numpy(),
                   slot_bufs[0].numpy())
    pos_dev.copy_(pos_bufs[0])
    slot_dev.copy_(slot_bufs[0])
    meta_g = build_attention_metadata(batch.chunks, slot_dev, 16, pages_per_split=ws.pages_per_split)

    def device_part() -> None:
        cur = torch.cuda.current_stream(device)
        c, s = ws.cos_t[pos_dev], ws.sin_t[pos_dev]
        if not overlap_copies:
            qkv_dev.copy_(qkv_host, non_blocking=True)
            for layer in range(layers):
                k_cache, v_cache = ws.views[layer]
                q = qk_norm_rope_scatter(qkv_dev[layer], ws.qw[layer], ws.kw[layer], 1e-6, c, s,
                                         slot_dev, k_cache, v_cache, H, q_out=ws.q_buf)
                attend(q, k_cache, v_cache, meta_g, D**-0.5, out=ws.out_all[layer])
            out_host.copy_(ws.out_all, non_blocking=True)
            return
        step_started.record(cur)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(step_started)
            for layer in range(layers):
                qkv_dev[layer].copy_(qkv_host[layer], non_blocking=True)
                qkv_arrived[layer].record(copy_stream)
        for layer in range(layers):
            k_cache, v_cache = ws.views[layer]
            cur.wait_event(qkv_arrived[layer])
            q = qk_norm_rope_scatter(qkv_dev[layer], ws.qw[layer], ws.kw[layer], 1e-6, c, s,
                                     slot_dev, k_cache, v_cache, H, q_out=ws.q_buf)
            attend(q, k_cache, v_cache, meta_g, D**-0.5, out=ws.out_all[layer])
            out_written[layer].record(cur)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(out_written[layer])
                out_host[layer].copy_(ws.out_all[layer], non_blocking=True)
        cur.wait_stream(copy_stream)

    device_part()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        device_part()
    torch.cuda.synchronize(device)

    def replay_step() -> None:
        k = step_no[0] & 1
        step_no[0] += 1
        if copies_done[k] is not None:
            copies_done[k].synchronize()
        prepare_arrays(new_np, cached_np, offsets_np, tables_np, pos_bufs[k].numpy(),
                       slot_bufs[k].numpy())
        pos_dev.copy_(pos_bufs[k], non_blocking=True)
        slot_dev.copy_(slot_bufs[k], non_blocking=True)
        done = torch.cuda.Event()
        done.record(stream)
        copies_done[k] = done
        if not meta_g.update(batch.chunks):
            raise RuntimeError("the step's plan no longer matches the captured launch shape")
        graph.replay()

    for _ in range(max(1, args.warmup)):
        replay_step()
    torch.cuda.synchronize(device)
    graph_ms = ws.timed(replay_step, args.steps, world)
    torch.cuda.synchronize(device)
    del graph
    h2d = qkv_host.numel() * 2 + pos_bufs[0].numel() * 8 + slot_bufs[0].numel() * 8 \
        + int(ws.meta.info.total_ints) * 4
    d2h = out_host.numel() * 2
    return graph_ms, eager_ms, h2d, d2h


def run_headline(args: argparse.Namespace, rank: int, world: int, device: torch.device) -> dict:
    batch = make_batch(args.workload, rank, world, args.seqs, args.pool_gb)
    ws = DeviceStep(batch, args.layers, device, args.pages_per_split, seed=1234 + rank)
    for _ in range(args.warmup):
        ws.step()
    torch.cuda.synchronize(device)
    ws.check_status("after warm-up")
    if not args.no_graph:
        ws.capture()

    # ---- timed region: device-resident inputs ----
    sampler = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if sampler:
        sampler.start()
    eager_ms = ws.timed(ws.step, args.steps, world)
    total_ms = ws.timed(ws.graph.replay, args.steps, world) if ws.graph is not None else eager_ms
    attn_ms = ws.attention_launch_ms(min(args.steps, 5))
    clocks = sampler.stop() if sampler else None
    if world > 1:
        torch.distributed.barrier()
    ws.check_status("after timing")

    # ---- a mixed batch's two parts, timed apart (decode rows; prefill chunks) ----
    parts = None
    dec_chunks = [c for c in batch.chunks if c.num_new <= 64]
    pre_chunks = [c for c in batch.chunks if c.num_new > 64]
    if dec_chunks and pre_chunks:
        parts = {}
        for name, sub in (("decode_rows", dec_chunks), ("prefill_chunks", pre_chunks)):
            us = ws.part_us(sub)
            sub_bytes, _, sub_flops = attention_bytes(type(batch)(batch.name, sub, batch.num_blocks))
            parts[name] = {"us_per_layer": us, "GB/s": sub_bytes / (us * 1e-6) / 1e9,
                           "TFLOPS_causal": sub_flops / (us * 1e-6) / 1e12,
                           "timing": "CUDA-graph replay of 10 calls, this part alone"}

    qkv_part = None
    if not args.no_qkv_part and rank == 0:
        qkv_part = time_qkv_projection(batch.num_tokens, ws.views, ws.qw, ws.kw, ws.cos, ws.sin,
                                       ws.slot_mapping, ws.layers, device, ws.stream)
        ws.check_status("after the qkv projection timing")

    e2e_ms, e2e_eager_ms, h2d, d2h = run_e2e(ws, args, world)
    attn_bytes, a_bytes, attn_flops = attention_bytes(batch)
    info = ws.meta.info
    res = {
        "total_ms": total_ms, "eager_ms": eager_ms, "graph": ws.graph is not None,
        "e2e_ms": e2e_ms, "e2e_eager_ms": e2e_eager_ms, "attn_ms": attn_ms, "attn_bytes": attn_bytes,
        "attn_flops": attn_flops, "logical_kv_tokens": batch.kv_tokens_read(),
        "kernel_a_bytes": a_bytes, "tokens": batch.num_tokens,
        "kv_tokens": (batch.kv_tokens_read() if ws.alias else batch.unique_kv_tokens()),
        "pool_shared_by_layers": ws.alias, "num_blocks": batch.num_blocks, "clocks": clocks,
        "launches_per_step": ws.layers * ws.launches_per_layer, "h2d": h2d, "d2h": d2h,
        "parts": parts, "qkv_projection": qkv_part,
        "plan": {"decode_items": info.n_decode_items, "tile_items": info.n_tile_items,
                 "tc_items": info.n_tc_items, "combine": info.n_combine,
                 "cascade_groups": info.n_cascade, "pages_per_split": info.pages_per_split},
    }
    ws.release()
    return res


# ---------------------------------------------------------------------------------------------
# our implementation: the other configurations, reported beside the headline
# ---------------------------------------------------------------------------------------------


def run_single_gpu_config(name: str, args: argparse.Namespace, device: torch.device) -> dict:
    """Config 3 or 4 on this GPU: the 28-layer step (CUDA-graph replay) and its attention
    launches, each with the roofline of the kernel that dominates it."""
    steps, warmup = max(3, min(args.steps, 20)), max(3, args.warmup)
    batch = make_batch(name, 0, 1)
    ws = DeviceStep(batch, LAYERS, device, 0, seed=77)
    for _ in range(warmup):
        ws.step()
    torch.cuda.synchronize(device)
    ws.check_status(f"after the {name} warm-up")
    ws.capture()
    total_ms = ws.timed(ws.graph.replay, steps, 1)
    attn_ms = ws.attention_launch_ms(3)
    ws.check_status(f"after the {name} timing")
    attn_bytes, _, attn_flops = attention_bytes(batch)
    info = ws.meta.info
    out = {
        "workload": workload_label(name, 1),
        "us_per_layer_step": total_ms * 1e3 / (steps * LAYERS),
        "tokens_per_s": batch.num_tokens * steps / (total_ms * 1e-3),
        "attn_us_per_layer": attn_ms * 1e3,
        "timing": f"CUDA-graph replay of the 28-layer step x {steps} after {warmup} warm-up steps; "
                  "attention launches timed with CUDA events around each layer's call",
        "plan": {"decode_items": info.n_decode_items, "tile_items": info.n_tile_items,
                 "tc_items": info.n_tc_items, "combine": info.n_combine,
                 "cascade_groups": info.n_cascade},
    }
    if name == "cfg3":
        dec = [c for c in batch.chunks if c.num_new <= 64]
        pre = [c for c in batch.chunks if c.num_new > 64]
        pre_us, dec_us = ws.part_us(pre), ws.part_us(dec)
        pre_batch = type(batch)(batch.name, pre, batch.num_blocks)
        dec_batch = type(batch)(batch.name, dec, batch.num_blocks)
        _, _, pre_flops = attention_bytes(pre_batch)
        dec_bytes, _, _ = attention_bytes(dec_batch)
        pre_q = sum(c.num_new for c in pre)
        out["prefill_part"] = {
            "us_per_layer": pre_us,
            "roofline": roofline_tensor("prefill_tc_kernel (kernel D, tcgen05/TMEM): the two "
                                        "1000-token chunks", pre_flops, pre_us,
                                        scaled_traffic("prefill_tc_cfg3", pre_q)),
            "timing": "CUDA-graph replay of 10 attention calls over the prefill chunks alone",
        }
        out["decode_part"] = {
            "us_per_layer": dec_us,
            "roofline": roofline_hbm("paged_attn_kernel decode mode: the 48 decode rows",
                                     dec_bytes, dec_us, None),
            "timing": "CUDA-graph replay of 10 attention calls over the decode rows alone",
        }
        out["roofline"] = out["prefill_part"]["roofline"]
    else:
        # Cascade: the shared prefix once on the tensor-core kernel, every row's own pages on the
        # persistent decode kernel; bytes count each physical block once (logical bytes beside).
        logical = (batch.kv_tokens_read() * KVH * D * 2 * 2 + batch.num_tokens * H * D * 2 * 2)
        out["roofline"] = roofline_hbm(
            "cascade attention: prefill_tc_kernel (shared prefix once) + "
            "paged_decode_units_kernel (own pages, merged)", attn_bytes, attn_ms * 1e3,
            scaled_traffic("cascade_cfg4", batch.num_tokens))
        out["roofline"]["logical_bytes_per_launch"] = logical
        out["roofline"]["logical_GBps"] = logical / (attn_ms * 1e-3) / 1e9
    ws.release()
    return out


def run_config5(args: argparse.Namespace, rank: int, world: int, device: torch.device) -> dict:
    """Config 5 (box scale) at this N: the 8,192 rows sharded over the ranks by context tokens
    (strong scaling), a pool of about 150 GB per GPU shared by the 28 layers.  Time = max over
    ranks of the 28-layer step; per-rank roofline from each rank's own bytes and time."""
    steps, warmup = max(3, min(args.steps, 5)), 3
    batch = make_batch("cfg5", rank, world, pool_gb=args.pool_gb)
    ws = DeviceStep(batch, LAYERS, device, 0, seed=55 + rank)
    for _ in range(warmup):
        ws.step()
    torch.cuda.synchronize(device)
    ws.check_status("after the config-5 warm-up")
    ws.capture()
    sampler = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if sampler:
        sampler.start()
    total_ms = ws.timed(ws.graph.replay, steps, world)
    clocks = sampler.stop() if sampler else None
    attn_ms = ws.attention_launch_ms(1)
    ws.check_status("after the config-5 timing")
    attn_bytes, _, _ = attention_bytes(batch)
    mine = torch.tensor([total_ms / steps, attn_ms, attn_bytes / (attn_ms * 1e-3) / 1e9,
                         batch.num_tokens, batch.kv_tokens_read()], dtype=torch.float64,
                        device=device)
    every = [torch.zeros_like(mine) for _ in range(world)]
    if world > 1:
        torch.distributed.all_gather(every, mine)
    else:
        every = [mine]
    rows = [x.cpu().tolist() for x in every]
    ws.release()
    step_ms = max(r[0] for r in rows)
    hbm = float(peaks()[0]["hbm_gbs"])
    per_rank = [{"rank": i, "ms_per_step": r[0], "attn_us_per_layer": r[1] * 1e3,
                 "achieved_GBps": r[2], "frac": r[2] / hbm, "rows": int(r[3]),
                 "kv_tokens_per_layer": int(r[4])} for i, r in enumerate(rows)]
    slowest = min(per_rank, key=lambda r: r["achieved_GBps"])
    return {
        "workload": workload_label("cfg5", world, pool_gb=args.pool_gb),
        "scaling": "strong",
        "value": 8192 / (step_ms * 1e-3),
        "unit": "tok/s",
        "ms_per_step": step_ms,
        "us_per_layer_step": step_ms * 1e3 / LAYERS,
        "timing": f"CUDA-graph replay of the 28-layer step x {steps} after {warmup} warm-up "
                  "steps; max over ranks",
        "roofline": {**roofline_hbm("paged_attn_kernel decode mode + combine (each rank's "
                                    "share; logical bytes, the shared pool is >> L2)",
                                    slowest["achieved_GBps"] * 1.0, 1e6, None),
                     "achieved": slowest["achieved_GBps"], "frac": slowest["frac"],
                     "algorithmic_bytes_per_launch": None,
                     "note": "slowest rank's attention launches: its bytes / its CUDA-event time"},
        "per_rank": per_rank,
        "clocks": clocks,
    }


# ---------------------------------------------------------------------------------------------
# the reference's CPU path (oracle restatement of MiniServe's torch code)
# ---------------------------------------------------------------------------------------------


def cpu_reference_layer_setup(batch, seed: int = 0):
    """One layer of a batch in the reference's own layout and dtype, on the host: the same
    geometry, pool size and block tables as the GPU arm."""
    from oracle import attention_oracle as orc

    chunks = [orc.SeqChunk(c.flat_start, c.num_new, c.num_cached, list(c.block_table))
              for c in batch.chunks]
    g = torch.Generator().manual_seed(seed)
    nslots = batch.num_blocks * 16
    t = batch.num_tokens
    k_cache = torch.randn(nslots, KVH, D, generator=g).bfloat16()
    v_cache = torch.randn(nslots, KVH, D, generator=g).bfloat16()
    qkv = torch.randn(t, (H + 2 * KVH) * D, generator=g).bfloat16()
    qw = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16()
    kw = (1 + 0.1 * torch.randn(D, generator=g)).bfloat16()
    cos, sin = orc.rope_tables(D, batch.max_position + 8, 1e6)
    slots = torch.from_numpy(batch.slots)
    positions = torch.from_numpy(batch.positions)

    def layer() -> None:
        meta = orc.build_metadata(chunks, slots, 16)
        orc.attention_layer(qkv, qw, kw, 1e-6, cos, sin, positions, k_cache, v_cache, meta)

    return layer, t


def run_cpu_layers(batch, warmup: int, iters: int) -> tuple[float, int, int, int]:
    """Median seconds of one layer of the reference's CPU path (all host threads), after
    ``warmup`` untimed runs; the same policy serves the reference arm and the cpu_baseline."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layer, t = cpu_reference_layer_setup(batch)
    for _ in range(warmup):
        layer()
    times = []
    for _ in range(iters):
        t0 = time.perf_counter()
        layer()
        times.append(time.perf_counter() - t0)
    return float(statistics.median(times)), t, threads, len(times)


CPU_SAMPLE = ("each sample = 1 of the 28 layers of this rank-0 batch (norm + RoPE + scatter + "
              "metadata + gathered SDPA, the oracle restating MiniServe's torch path) on the "
              "host CPU; median of the samples; tok/s = tokens / (28 x median)")


# ---------------------------------------------------------------------------------------------


def main() -> None:
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        batch = make_batch("cfg2", 0, max(world, args.gpus), args.seqs)
        t_layer, t, threads, n = run_cpu_layers(batch, max(3, args.warmup), args.steps)
        value = t / (LAYERS * t_layer)
        line = {
            "impl": "reference",
            "metric": METRIC,
            "value": value,
            "unit": "tok/s",
            "n_gpus": args.gpus,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": t_layer * 1e3,
            "step": "one bounded sample: 1 of the 28 layers of the batch",
            "ms_per_layer": t_layer * 1e3,
            "ms_per_28_layers_extrapolated": t_layer * LAYERS * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": headline_config(max(world, args.gpus), args.seqs, LAYERS),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": CPU_SAMPLE + f"; {n} samples"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=device)
    from miniserve_b200.build import build

    if rank == 0:
        build()
    if world > 1:
        torch.distributed.barrier()

    if args.workload in ("qkv", "prefill"):
        if args.workload == "qkv":
            run_qkv_only(args, rank, device)
        else:
            run_prefill_only(rank, device)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return

    r = run_headline(args, rank, world, device)
    hbm = float(peaks()[0]["hbm_gbs"])
    my_achieved = r["attn_bytes"] / (r["attn_ms"] * 1e-3) / 1e9
    ms = torch.tensor([r["total_ms"], r["e2e_ms"], r["attn_ms"], r["eager_ms"], r["e2e_eager_ms"]],
                      dtype=torch.float64, device=device)
    toks = torch.tensor([r["tokens"]], dtype=torch.float64, device=device)
    mine = torch.tensor([my_achieved, r["attn_ms"], r["attn_bytes"]], dtype=torch.float64,
                        device=device)
    every = [torch.zeros_like(mine) for _ in range(world)]
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(toks, op=torch.distributed.ReduceOp.SUM)
        torch.distributed.all_gather(every, mine)
    else:
        every = [mine]
    per_rank = [x.cpu().tolist() for x in every]
    total_ms, e2e_ms, attn_ms_max, eager_ms, e2e_eager_ms = (float(x) for x in ms.cpu())
    ms_per_step = total_ms / args.steps
    e2e_per_step = e2e_ms / args.steps
    tokens_all = int(toks.item())

    headline = args.workload == "cfg2" and args.layers == LAYERS
    extras: dict = {}
    if headline and not args.no_extras:
        # Configs 3 and 4 are single-GPU configurations: rank 0 runs them while the others wait.
        if rank == 0:
            extras["config3"] = run_single_gpu_config("cfg3", args, device)
            extras["config4"] = run_single_gpu_config("cfg4", args, device)
        if world > 1:
            torch.distributed.barrier()
        extras["config5"] = run_config5(args, rank, world, device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and headline:
        batch0 = make_batch("cfg2", 0, 1, args.seqs)
        t_layer, t, threads, n = run_cpu_layers(batch0, 3, 20)
        cpu = {"value": t / (LAYERS * t_layer), "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": CPU_SAMPLE + f"; {n} samples after 3 warm-up runs"}

    if rank == 0:
        slowest = min(range(world), key=lambda i: per_rank[i][0])
        achieved = per_rank[slowest][0]
        if args.workload == "cfg2":
            kernel = "paged_attn_kernel decode mode (kernel B; + combine C when a plan splits)"
            units = r["kv_tokens"]
            traffic = scaled_traffic("paged_attn_decode_cfg2", units)
        else:
            kernel, traffic = f"attention launches of {args.workload}", None
        line = {
            "metric": METRIC if args.workload == "cfg2" else METRIC.replace("config 2", args.workload),
            "value": tokens_all / (ms_per_step * 1e-3),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong" if args.workload == "cfg5" else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": (headline_config(world, args.seqs, args.layers) if args.workload == "cfg2"
                       else {"workload": workload_label(args.workload, world, args.seqs,
                                                        args.layers, args.pool_gb),
                             "layers": args.layers,
                             "parallelism": f"sequence-sharded x{world}"}),
            "workload_stats": {"kv_tokens_per_layer": r["kv_tokens"],
                               "logical_kv_tokens_per_layer": r["logical_kv_tokens"],
                               "pool_blocks_per_layer": r["num_blocks"],
                               "tokens_per_rank": r["tokens"]},
            "us_per_layer_step": ms_per_step * 1e3 / args.layers,
            "step_timing": "CUDA-graph replay of the captured step" if r["graph"] else "eager",
            "eager_ms_per_step": eager_ms / args.steps,
            "attn_us_per_layer": attn_ms_max * 1e3,
            "roofline": {
                **roofline_hbm(kernel, per_rank[slowest][2], per_rank[slowest][1] * 1e3, traffic),
                "achieved": achieved,
                "frac": achieved / hbm,
                "per_rank_achieved": [x[0] for x in per_rank],
                "note": "achieved = the slowest rank's algorithmic bytes / its mean attention "
                        "launch time (CUDA events)",
                "attn_tflops": r["attn_flops"] / (r["attn_ms"] * 1e-3) / 1e12,
            },
            "cpu_baseline": cpu,
            "e2e": {"value": tokens_all / (e2e_per_step * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                    "eager_value": tokens_all / (e2e_eager_ms / args.steps * 1e-3),
                    "host_work_per_step": "ms_prepare_step (positions, slots) + ms_plan_build "
                                          "+ the plan written into the captured step's buffers "
                                          "(AttentionMetadata.update) + one CUDA-graph replay of "
                                          "the step's device part: qkv of all layers in, outputs "
                                          "of all layers out (per layer on a copy stream, "
                                          "overlapped with the other layers' kernels, when a "
                                          "layer's input is >= 1 MiB), cos/sin rows, every "
                                          "layer's kernels; eager_value: the same with every "
                                          "layer's calls made from Python each step"},
            "gpu_launches": r["launches_per_step"] * args.steps,
            "clocks": r["clocks"],
            "plan": r["plan"],
        }
        if r["parts"] is not None:
            line["parts"] = r["parts"]
        if r["qkv_projection"] is not None:
            line["qkv_projection"] = r["qkv_projection"]
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
