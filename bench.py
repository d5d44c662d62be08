#!/usr/bin/env python
"""Benchmark of the exact segmented decode-attention path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode128k_bf16|decode8k_fp16]

Workload (default ``decode128k_bf16``): one layer, batch 1, 32 query heads /
8 KV heads, head_dim 128, bf16 K/V; context 132,120 tokens = 127 archived
blocks of 1,000 + a 1,024-token tail block + a full 4,096-token hot ring;
q, K, V ~ N(0, 1) (seeded). One "call" is one decode-attention call (1 new
token, all heads, whole context); a step is ``calls_per_step`` back-to-back
calls. The metric unit is calls/s (= decoded tokens/s for this layer).

With N GPUs (torchrun, one process per GPU) the archived blocks are
partitioned contiguously over the ranks, balancing tokens with the hot ring on
the last rank; each call attends locally and the ranks' (output, LSE) pairs
are merged inside the attention kernel over NVLink (``--merge p2p``, default)
or with an NCCL all-gather + LSE-merge kernel (``--merge nccl``). Strong
scaling: the context is fixed.

Reported (rank 0, one JSON line): device throughput with inputs resident in
HBM (CUDA-graph-captured calls timed with CUDA events, max over ranks),
``e2e`` through the public API with the new token's q/k/v taken from pinned
host memory and the output returned to pinned host memory every call (the
kernels read and write those buffers across the bus), the decode kernel's
roofline against the measured HBM copy bandwidth, NVML clock samples taken
during the timed region, and (N = 1) a CPU baseline: the reference algorithm
restated in numpy, on the host's cores. ``--impl reference`` prints that CPU
arm alone.

At N = 1 the line also carries ``secondary`` (the 8K fp16 decode workload)
and ``prefill``: one layer of a 32K-token prompt prefilled in 2048-token
chunks on the tcgen05 tensor-core kernel, against the measured bf16 peak.

``--shard-of N`` times rank 0's shard of the N-way partition alone on one GPU
(the per-rank kernel of a sharded run, for profiling).

Other workloads (one GPU, one JSON line each): ``prefill32k_chunk2048_bf16``,
``warm_reload_bf16`` (decode steps that reload cold blocks), and the whole
models ``model8b_e2e_bf16`` (Llama-3-8B shape) and
``model7b_prefill32k_warm_bf16`` (Mistral-7B shape, 32K prompt, half the
archived blocks in the pinned host tier; ``--decode-steps N``, default 128).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "rfsn-mlx_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode attn tokens/s & HBM GB/s (%roofline) at 8K/128K ctx, 1/2/4/8 B200"

WORKLOADS = {
    "decode128k_bf16": dict(
        dtype="bfloat16", q_heads=32, kv_heads=8, head_dim=128, blocks=[1000] * 127 + [1024], hot=4096,
        block_size=1000, seed=3,
        desc="1 layer, batch 1, 32 q / 8 kv heads, head_dim 128, bf16; 132,120-token context = 127 x 1000 + 1 x 1024 "
             "archived blocks + 4,096-token hot ring",
    ),
    "decode8k_fp16": dict(
        dtype="float16", q_heads=32, kv_heads=8, head_dim=128, blocks=[256] * 24, hot=2048, block_size=256, seed=2,
        desc="1 layer, batch 1, 32 q / 8 kv heads, head_dim 128, fp16; 8,192-token context = 24 x 256 archived "
             "blocks + 2,048-token hot ring",
    ),
}


def algorithmic_bytes(w: dict, tokens: int) -> int:
    """K and V read once (GQA shared) + q read + output written (float32)."""
    es = 2
    return 2 * tokens * w["kv_heads"] * w["head_dim"] * es + 2 * w["q_heads"] * w["head_dim"] * 4


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


# ------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """NVML samples of SM clock and clock-event reasons while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int, period_s: float = 0.01) -> None:
        self.index, self.period = index, period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def start(self) -> "ClockSampler":
        try:
            import pynvml

            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception as exc:  # no NVML: report it, keep running
            self.error = f"nvml unavailable: {exc}"
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self) -> None:
        n = self._nvml
        get_reasons = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM), int(get_reasons(self._h))))
            except Exception as exc:
                self.error = str(exc)
                return
            time.sleep(self.period)

    def stop(self) -> dict:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "note": self.error}
        reasons = set()
        for _, mask in self.samples:
            for bit, name in self.REASONS.items():
                if mask & bit and name != "gpu_idle":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(s for s, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(reasons),
            "samples": len(self.samples),
        }


# ------------------------------------------------------------------------------------ setup
def _extra(fn):
    """Result of an optional part of the JSON line, or {"error": ...} if it raised."""
    try:
        return fn()
    except Exception as exc:  # noqa: BLE001 - reported in the line
        return {"error": f"{type(exc).__name__}: {exc}"}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def build_shard(w: dict, rank: int, world: int, device, extra_tokens: int):
    """This rank's LayerKVCache: its contiguous block range, plus the hot ring on the last rank."""
    import torch

    from rfsn_b200 import LayerKVCache, RFSNConfig
    from rfsn_b200.sharded import balanced_shards

    blocks = w["blocks"]
    lo, hi = balanced_shards(blocks, w["hot"], world)[rank]
    starts = [sum(blocks[:i]) for i in range(len(blocks))]
    archived_total = sum(blocks)
    local_tokens = sum(blocks[lo:hi])
    owns_hot = rank == world - 1
    cfg = RFSNConfig(
        hidden_dim=w["q_heads"] * w["head_dim"], num_heads=w["q_heads"], num_kv_heads=w["kv_heads"],
        head_dim=w["head_dim"], num_layers=1, vocab_size=128, hot_capacity=w["hot"],
        warm_capacity=archived_total + w["hot"] + extra_tokens + 4 * w["block_size"],
        cold_capacity=archived_total + w["hot"] + extra_tokens + 4 * w["block_size"],
        block_size_seq=w["block_size"], model_dtype=w["dtype"], disk_cache_dir=tempfile.mkdtemp(prefix="rfsn_bench_"),
    )
    pool = local_tokens + (extra_tokens + 2 * max(w["block_size"], w["hot"]) if owns_hot else 0) + 64
    cache = LayerKVCache(cfg, batch_size=1, num_heads=w["q_heads"], num_kv_heads=w["kv_heads"], layer_id=0,
                         session_id=f"bench-r{rank}", device=device, pool_tokens=pool)
    dt = cache.dtype
    gen = torch.Generator(device=device)
    for i in range(lo, hi):
        gen.manual_seed(w["seed"] * 100003 + i)
        shape = (1, w["kv_heads"], blocks[i], w["head_dim"])
        k = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt)
        v = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt)
        cache.import_block(k, v, starts[i])
    cache.hot_start = archived_total
    if owns_hot:
        gen.manual_seed(w["seed"] * 100003 + 99991)
        shape = (1, w["kv_heads"], w["hot"], w["head_dim"])
        k = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt)
        v = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt)
        cache.evict_for_append(w["hot"])
        cache.append_exact(k, v)
    return cache, owns_hot, local_tokens + (w["hot"] if owns_hot else 0), archived_total + w["hot"]


def barrier(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


PARITY_TOL = 2e-3  # max-abs bar for attention outputs (fp16/bf16 K/V, float32 accumulation)


def _parity_q(w, device):
    """The query of the parity calls: the same seeded tensor on every rank."""
    import torch

    gen = torch.Generator(device=device).manual_seed(w["seed"] * 7919 + 17)
    return torch.randn((1, w["q_heads"], 1, w["head_dim"]), generator=gen, device=device, dtype=torch.float32)


def _dense_context(w, device):
    """The whole context's K/V in logical order, regenerated from the per-block
    seeds ``build_shard`` uses (archived blocks, then the hot ring), float64."""
    import torch

    dt = {"bfloat16": torch.bfloat16, "float16": torch.float16}[w["dtype"]]
    ks, vs = [], []
    gen = torch.Generator(device=device)
    for i, n in enumerate(w["blocks"]):
        gen.manual_seed(w["seed"] * 100003 + i)
        shape = (w["kv_heads"], n, w["head_dim"])
        ks.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt).double())
        vs.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt).double())
    gen.manual_seed(w["seed"] * 100003 + 99991)
    shape = (w["kv_heads"], w["hot"], w["head_dim"])
    ks.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt).double())
    vs.append(torch.randn(shape, generator=gen, device=device, dtype=torch.float32).to(dt).double())
    return torch.cat(ks, dim=1), torch.cat(vs, dim=1)


def _dense_attention(q, k, v):
    """softmax(q k^T / sqrt(D)) v over every key (the query is the last token),
    query head h on KV head h // G; float64."""
    import torch

    Hq, D = q.shape[1], q.shape[3]
    G = Hq // k.shape[0]
    qh = q[0, :, 0, :].double().view(k.shape[0], G, D)                   # [Hkv, G, D]
    p = (torch.bmm(qh, k.transpose(1, 2)) / (D ** 0.5)).softmax(dim=-1)  # [Hkv, G, T]
    return torch.bmm(p, v).reshape(1, Hq, 1, D)                          # [1, Hq, 1, D]


E2E_EXTRA = [0]  # extra ring tokens a full-context replay cache must hold (set by run_ours)


def static_parity(cache, w, world, rank, device, total_tokens, peers):
    """Correctness of the timed call: every rank makes one more call of the
    timed kind (local attention + the cross-GPU merge at N > 1) with a fixed
    query; rank 0 compares the merged output with (a) the single-GPU kernel
    over the whole context (rank 0 rebuilds it from the per-block seeds; at
    N = 1 that is the timed kernel itself, so only (b) is reported) and (b) a
    dense float64 softmax over the same keys. Returns (rank 0) the figures and
    a fresh full-context cache for the end-to-end check."""
    import torch

    from rfsn_b200.cache import paged_attention
    from rfsn_b200.sharded import merge_across_ranks

    q = _parity_q(w, device)
    pos = total_tokens - 1
    segs = cache.get_attention_segments()
    if world > 1 and peers is not None:
        got = paged_attention(cache, q, pos, segs, peers=peers)
    elif world > 1:
        if len(segs) == 0:
            out = torch.zeros_like(q)
            lse = torch.full(q.shape[:3], float("-inf"), device=device)
        else:
            out, lse = paged_attention(cache, q, pos, segs, want_lse=True)
        got = merge_across_ranks(out, lse)
    else:
        got = paged_attention(cache, q, pos, segs)
    torch.cuda.synchronize()
    res = None
    if rank == 0:
        def figures():
            r = {}
            full = build_shard(w, 0, 1, device, E2E_EXTRA[0])[0]
            if world > 1:
                ref1 = paged_attention(full, q, pos, full.get_attention_segments())
                r["max_abs_vs_1gpu"] = float((got - ref1).abs().max())
            k64, v64 = _dense_context(w, device)
            dense = _dense_attention(q, k64, v64)
            del k64, v64
            r["max_abs_vs_dense_fp64"] = float((got.double() - dense).abs().max())
            r["query_position"] = pos
            return r, full
        try:
            res = figures()
        except Exception as exc:  # noqa: BLE001 - reported in the line
            res = ({"error": f"{type(exc).__name__}: {exc}"}, None)
    barrier(world)
    return res


def e2e_parity(full, w, e2e_info):
    """Rank 0: the last output of the end-to-end loop against the same token
    sequence replayed through ``attention_step`` (op by op, public API) on the
    single-GPU full-context cache."""
    import torch

    from rfsn_b200.layer import attention_step

    pos0, n_calls, q_h, k_h, v_h, last = e2e_info
    q, k, v = (t.to(full.device) for t in (q_h, k_h, v_h))
    out = None
    for i in range(n_calls):
        out = attention_step(q, k, v, full, pos0 + i)
    torch.cuda.synchronize()
    return {"max_abs_vs_1gpu_replay": float((out.cpu() - last).abs().max()), "calls_replayed": n_calls}


# ------------------------------------------------------------------------------------ measurements
L2_ROTATION_BYTES = 256e6  # more than twice the 126 MB L2: rotated shard copies are read from HBM every call


def shard_copies(w, world: int, total_tokens: int) -> int:
    """Copies of a rank's shard the calls rotate through, so that consecutive
    calls of a rank never find its K/V in L2 (a decode step runs every other
    layer's attention between two calls of one layer). The same on every rank."""
    if world == 1:
        return 1
    per_rank = algorithmic_bytes(w, total_tokens) / world
    return max(1, int(-(-L2_ROTATION_BYTES // per_rank)))


def device_throughput(caches, w, world, steps, warmup, calls_per_step, *, collective: bool, peers=None):
    """calls/s with inputs resident: CUDA-graph-captured calls, CUDA events.
    Call i uses shard copy i % len(caches)."""
    import torch

    from rfsn_b200 import _native as native
    from rfsn_b200.cache import paged_attention
    from rfsn_b200.sharded import merge_across_ranks

    cache = caches[0]
    total = cache.hot_start + cache.hot_seq_len
    q = torch.randn((1, w["q_heads"], 1, w["head_dim"]), device=cache.device, dtype=torch.float32)
    pos = total - 1
    segs = [c.get_attention_segments() for c in caches]
    use_coll = collective and world > 1

    def one_call(i):
        c, sg = caches[i % len(caches)], segs[i % len(caches)]
        if use_coll and peers is not None:
            return paged_attention(c, q, pos, sg, peers=peers)
        if use_coll:
            out, lse = paged_attention(c, q, pos, sg, want_lse=True)
            return merge_across_ranks(out, lse)
        return paged_attention(c, q, pos, sg, want_lse=world > 1)

    for i in range(3 * len(caches)):  # eager warm-up: sizes the workspace, sets kernel attributes
        one_call(i)
    torch.cuda.synchronize()
    before = native.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(calls_per_step):
            one_call(i)
    launches_per_step = native.launch_count() - before
    torch.cuda.synchronize()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    end.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    del graph
    return ms, launches_per_step * steps


def e2e_throughput(caches, w, world, owns_hot, steps, calls_per_step, peers=None):
    """calls/s through the public API with pinned host inputs and a host
    read-back every call. With several shard copies they act as layers: every
    token is stepped through each copy in turn at the same position."""
    import torch

    from rfsn_b200 import _native as native
    from rfsn_b200.layer import GraphedDecodeStep
    from rfsn_b200.sharded import GraphedShardedDecodeStep, sharded_decode_step

    cache = caches[0]
    ncopy = len(caches)
    dt = cache.dtype
    H, Hkv, D = w["q_heads"], w["kv_heads"], w["head_dim"]
    gen = torch.Generator().manual_seed(7)
    q_h = torch.randn((1, H, 1, D), generator=gen).to(dt).pin_memory()
    k_h = torch.randn((1, Hkv, 1, D), generator=gen).to(dt).pin_memory()
    v_h = torch.randn((1, Hkv, 1, D), generator=gen).to(dt).pin_memory()
    out_h = torch.empty((1, H, 1, D), dtype=torch.float32).pin_memory()
    pos = cache.hot_start + cache.hot_seq_len if owns_hot else None
    # every rank needs the global position: the hot owner broadcasts it
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([pos if owns_hot else 0], device=cache.device)
        dist.all_reduce(t)
        pos = int(t.item())

    graphed = []
    if world == 1 or peers is not None:
        # one graph replay per call: H2D of the token's q (and k/v on the hot-window
        # owner), RoPE + append, paged attention (merged over NVLink when sharded),
        # D2H of the output (rfsn_b200.layer.GraphedDecodeStep /
        # rfsn_b200.sharded.GraphedShardedDecodeStep)
        for c in caches:
            g = GraphedDecodeStep(c, H) if world == 1 else GraphedShardedDecodeStep(c, H, owns_hot=owns_hot,
                                                                                     peers=peers)
            g.q_host.copy_(q_h)
            g.k_host.copy_(k_h)
            g.v_host.copy_(v_h)
            graphed.append(g)

    def call(i, p):
        if graphed:
            graphed[i % ncopy].step(p)
            return
        c = caches[i % ncopy]
        q = q_h.to(c.device, non_blocking=True)
        k = k_h.to(c.device, non_blocking=True)
        v = v_h.to(c.device, non_blocking=True)
        out = sharded_decode_step(c, q, k if owns_hot else None, v if owns_hot else None, p, owns_hot=owns_hot,
                                  peers=peers)
        out_h.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for t in range(3):  # warm-up tokens
        for j in range(ncopy):
            call(j, pos + t)
    pos += 3
    barrier(world)
    before = native.launch_count()
    replays0 = sum(g.replays for g in graphed)
    tokens = -(-steps * calls_per_step // ncopy)
    n = tokens * ncopy
    t0 = time.perf_counter()
    for i in range(n):
        call(i, pos + i // ncopy)
    elapsed = time.perf_counter() - t0
    launches = native.launch_count() - before
    if graphed:  # kernels replayed inside the graph are not host launches
        launches += graphed[0].graph_kernels * (sum(g.replays for g in graphed) - replays0)
    barrier(world)
    if graphed:  # the replay copies the whole packed staging buffer (step state + q/k/v)
        h2d = graphed[0].stage_host.numel() * graphed[0].stage_host.element_size()
    else:
        h2d = q_h.numel() * q_h.element_size() + (k_h.numel() * k_h.element_size() * 2 if owns_hot else 0)
    d2h = out_h.numel() * out_h.element_size()
    last = (graphed[-1].out_host if graphed else out_h).clone()
    info = (pos - 3, tokens + 3, q_h, k_h, v_h, last)  # every token appended, for a replay check
    return elapsed, n, launches, h2d, d2h, info


def cpu_baseline_sample(w, budget_s=20.0):
    from oracle.cpu_baseline import synthetic_decode_inputs, time_calls

    q, segs, qpos = synthetic_decode_inputs(w["blocks"], w["hot"], w["kv_heads"], w["q_heads"], w["head_dim"],
                                            w["dtype"], w["seed"])
    sec, n, threads = time_calls(q, segs, qpos, calls=3, warmup=1, budget_s=budget_s)
    return sec, n, threads


# ------------------------------------------------------------------------------------ arms
def run_reference(args, w):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    per_step = []
    threads = len(os.sched_getaffinity(0)) or os.cpu_count() or 1
    from oracle.cpu_baseline import attention_all_cores, synthetic_decode_inputs, time_calls

    q, segs, qpos = synthetic_decode_inputs(w["blocks"], w["hot"], w["kv_heads"], w["q_heads"], w["head_dim"],
                                            w["dtype"], w["seed"])
    for _ in range(max(1, min(args.warmup, 2))):
        attention_all_cores(q, segs, qpos, threads)
    for _ in range(args.steps):
        s, n_, threads = time_calls(q, segs, qpos, calls=1, warmup=0)
        per_step.append(s)
    total = sum(per_step)
    value = args.steps / total
    tokens = sum(w["blocks"]) + w["hot"]
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": f"synthetic N(0,1) q/K/V, seed {w['seed']}",
        "config": {"workload": args.workload, "desc": w["desc"], "context_tokens": tokens, "calls_per_step": 1},
        "cpu_baseline": {
            "value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{args.steps} full decode-attention calls over the {tokens}-token context; the reference "
                      "algorithm (float32 upcast, GQA repeat, two passes) restated in numpy, (KV head, segment run) items on a thread pool with one BLAS thread per worker",
        },
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args, w):
    import torch

    world, rank, local = dist_env()
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())
    e2e_calls = max(1, min(args.calls_per_step, 50))
    extra = args.steps * e2e_calls + 8
    E2E_EXTRA[0] = extra
    cache, owns_hot, local_tokens, total_tokens = build_shard(w, rank, world, device, extra)
    # a shard smaller than L2 is rotated with copies of itself (same data)
    caches = [cache] + [build_shard(w, rank, world, device, extra)[0]
                        for _ in range(shard_copies(w, world, sum(w["blocks"]) + w["hot"]) - 1)]
    torch.cuda.synchronize()

    peers = None
    if world > 1 and args.merge == "p2p":
        from rfsn_b200.sharded import PeerGroup

        peers = PeerGroup(w["kv_heads"], w["head_dim"])
    peak, peak_kind = measured_peaks()
    sampler = ClockSampler(device.index).start()
    # kernel-only (local attention, no collective): roofline of the decode kernel
    k_ms, _ = device_throughput(caches, w, world, args.steps, args.warmup, args.calls_per_step, collective=False)
    # full call (local attention + all-gather + merge when N > 1)
    ms, launches = device_throughput(caches, w, world, args.steps, args.warmup, args.calls_per_step, collective=True,
                                     peers=peers)
    clocks = sampler.stop()
    ms = max_over_ranks(ms, world)
    k_ms_max = max_over_ranks(k_ms, world)
    # correctness of what was timed (outside the timed region)
    static = static_parity(cache, w, world, rank, device, total_tokens, peers)

    calls = args.steps * args.calls_per_step
    value = calls / (ms / 1e3)
    per_call_ms = ms / calls
    local_bytes = algorithmic_bytes(w, local_tokens)
    # the slowest rank's kernel (ranks hold the same bytes within a block)
    k_call_s = k_ms_max / 1e3 / calls
    achieved = local_bytes / k_call_s / 1e9

    # e2e through the public API (appends the new token each call)
    e_elapsed, e_n, e_launches, h2d, d2h, e2e_info = e2e_throughput(caches, w, world, owns_hot, args.steps, e2e_calls,
                                                                     peers)
    e_elapsed = max_over_ranks(e_elapsed, world)
    parity = None
    if rank == 0:
        figs, full = static
        parity = {"tol": PARITY_TOL, "timed_call": figs}
        if full is not None:
            parity["e2e_call"] = _extra(lambda: e2e_parity(full, w, e2e_info))
        vals = [v for d in (parity["timed_call"], parity.get("e2e_call", {})) for k_, v in d.items()
                if k_.startswith("max_abs")]
        parity["ok"] = (bool(vals) and all(v <= PARITY_TOL for v in vals)
                        and "error" not in parity["timed_call"] and "error" not in parity.get("e2e_call", {}))
        del full
    barrier(world)

    traffic = None
    prof = ROOT / "profiles" / f"{args.workload}_traffic.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    if world > 1:
        # the committed capture is of the whole context on one GPU; a shard's launch
        # (which also runs the cross-GPU merge) has no capture of its own
        traffic = None

    secondary = None
    prefill = None
    cpu = None
    if world == 1 and rank == 0:
        # The headline is measured by now: a failing extra is reported in the
        # line instead of taking the line with it.
        if args.workload == "decode128k_bf16" and not args.no_secondary:
            secondary = _extra(lambda: secondary_8k(args, device, peak))
        if not args.no_prefill:
            prefill = _extra(lambda: prefill_32k(args, device))
        if not args.no_cpu_baseline:
            def cpu_line():
                sec, n, threads = cpu_baseline_sample(w)
                return {
                    "value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": "port",
                    "sample": f"median of {n} full decode-attention calls over the {total_tokens}-token context "
                              "after 1 warm-up; the reference algorithm (float32 upcast, GQA repeat, two passes) "
                              "restated in numpy, (KV head, segment run) items on a thread pool with one BLAS thread per worker",
                }

            cpu = _extra(cpu_line)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16" if w["dtype"] == "bfloat16" else "fp16",
            "data": f"synthetic N(0,1) q/K/V (seeded); K/V resident in HBM",
            "config": {
                "workload": args.workload,
                "desc": w["desc"],
                "context_tokens": total_tokens,
                "calls_per_step": args.calls_per_step,
                "l2": (f"inputs larger than L2: {algorithmic_bytes(w, total_tokens) / 1e6:.0f} MB of K/V per call"
                       if len(caches) == 1 else
                       f"each rank rotates {len(caches)} copies of its {local_bytes / 1e6:.0f} MB shard "
                       f"({len(caches) * local_bytes / 1e6:.0f} MB > L2); the end-to-end loop steps every token "
                       "through the copies like layers"),
                "parallelism": (f"context-sharded over {world} GPUs by archived block; LSE merge "
                                + ("fused into the attention kernel over NVLink (CUDA IPC mailboxes)"
                                   if args.merge == "p2p" else "via NCCL all-gather + merge kernel"))
                if world > 1 else "1 GPU",
            },
            "us_per_call": per_call_ms * 1e3,
            "hbm_gbs": algorithmic_bytes(w, total_tokens) / (per_call_ms / 1e3) / 1e9,
            "context_tokens_per_s": total_tokens * value,
            "kernel_only_us_per_call_max_rank": k_ms_max / calls * 1e3,
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": local_bytes,
                "kernel": "rfsn::fast::paged_decode_kernel (rank 0's shard bytes over the slowest rank's kernel time; "
                          "the cross-GPU merge is outside this figure, in us_per_call)",
            },
            "e2e": {
                "value": e_n / e_elapsed,
                "unit": "tokens/s",
                "h2d_bytes_per_step": h2d * e2e_calls,
                "d2h_bytes_per_step": d2h * e2e_calls,
                "calls_per_step": e2e_calls,
                "api": "rfsn_b200.layer.GraphedDecodeStep (host buffers in/out, one graph replay per call)"
                if world == 1 else ("rfsn_b200.sharded.GraphedShardedDecodeStep (host buffers in/out, one graph "
                                    "replay per call, merge over NVLink in the kernel)" if peers is not None
                                    else "rfsn_b200.sharded.sharded_decode_step (NCCL merge)"),
            },
            "gpu_launches": launches,
            "e2e_gpu_launches": e_launches,
            "clocks": clocks,
            "parity": parity,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if secondary is not None:
            line["secondary"] = secondary
        if prefill is not None:
            line["prefill"] = prefill
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        import gc

        dist.barrier()
        torch.cuda.synchronize()
        gc.collect()
        dist.destroy_process_group()
    if rank == 0 and parity is not None and not parity["ok"]:
        print(f"parity check failed (max-abs bar {PARITY_TOL}): {json.dumps(parity)}", file=sys.stderr, flush=True)
        return 3
    return 0


def run_shard(args, w):
    """``--shard-of N``: one rank's share of the N-way partition of the
    workload (rank 0's archived blocks) on one GPU, the decode kernel alone,
    the shard rotated with copies of itself so every call reads HBM. Used to
    profile the per-rank kernel of a sharded run on one GPU."""
    import torch

    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    n = args.shard_of
    cache, _, local_tokens, total_tokens = build_shard(w, 0, n, device, 0)
    caches = [cache] + [build_shard(w, 0, n, device, 0)[0] for _ in range(shard_copies(w, n, total_tokens) - 1)]
    ms, launches = device_throughput(caches, w, 1, args.steps, args.warmup, args.calls_per_step, collective=False)
    calls = args.steps * args.calls_per_step
    us = ms * 1e3 / calls
    nbytes = algorithmic_bytes(w, local_tokens)
    peak, kind = measured_peaks()
    print(json.dumps({
        "metric": "decode-attention kernel time of one rank's shard (us/call)", "workload": args.workload,
        "shard": f"rank 0 of {n}", "shard_tokens": local_tokens, "shard_copies": len(caches), "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "value": us, "unit": "us/call",
        "gbs": nbytes / us / 1e3, "frac_of_measured_hbm": nbytes / us / 1e3 / peak, "peak_kind": kind,
        "gpu_launches": launches,
    }), flush=True)
    return 0


def secondary_8k(args, device, peak):
    """The 8K fp16 workload at N = 1, rotating 8 copies of the context so that
    consecutive calls miss L2 (8 x 33.6 MB > 126 MB)."""
    import torch

    w = WORKLOADS["decode8k_fp16"]
    caches = [build_shard(w, 0, 1, device, 0)[0] for _ in range(8)]
    from rfsn_b200.cache import paged_attention

    q = torch.randn((1, w["q_heads"], 1, w["head_dim"]), device=device)
    segs = [c.get_attention_segments() for c in caches]
    tokens = caches[0].hot_start + caches[0].hot_seq_len
    for c, s in zip(caches, segs):
        paged_attention(c, q, tokens - 1, s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    reps = 25
    with torch.cuda.graph(graph):
        for _ in range(reps):
            for c, s in zip(caches, segs):
                paged_attention(c, q, tokens - 1, s)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_rep = max(4, args.steps)
    start.record()
    for _ in range(n_rep):
        graph.replay()
    end.record()
    end.synchronize()
    calls = n_rep * reps * len(caches)
    us = start.elapsed_time(end) * 1e3 / calls
    bytes_ = algorithmic_bytes(w, tokens)
    return {
        "workload": "decode8k_fp16",
        "desc": w["desc"],
        "value": 1e6 / us,
        "unit": "tokens/s",
        "us_per_call": us,
        "hbm_gbs": bytes_ / (us / 1e6) / 1e9,
        "frac_of_measured_hbm": bytes_ / (us / 1e6) / 1e9 / peak,
        "l2": "8 rotating copies of the context (269 MB > L2)",
    }


PREFILL_WORKLOAD = "prefill32k_chunk2048_bf16"
PREFILL_DESC = ("one layer of a 32,768-token prompt prefilled in 16 chunks of 2,048 tokens, 32 q / 8 kv heads, head_dim "
                "128, bf16 K/V; hot ring 4,096 tokens, so chunk c attends to c-1 archived 2,048-token blocks plus the "
                "hot window (the previous chunk and itself), causally")


def bf16_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
        except Exception:
            pass
    return 1590.0, "fallback"


def prefill_32k(args, device):
    """Chunked-prefill attention on the tcgen05 kernel: the 16 chunk calls of one
    layer, K/V resident in HBM, timed with CUDA events. q holds bf16 values, as
    the projection and RoPE of a bf16 model deliver it; the same layer with
    float32 q (random values with residuals) is timed too. Useful FLOPs count
    the causal products once (4 * heads * head_dim per query-key pair); the
    kernel issues 1.5x that on the tensor cores for 16-bit q (q K^T, and the
    16-bit high + residual parts of P in P V) and 2x for float32 q."""
    import ctypes

    import torch

    from rfsn_b200 import _native as native

    H, Hkv, D, chunk, cap, n_chunks = 32, 8, 128, 2048, 4096, 16
    n_blocks_max = n_chunks - 2
    rows = cap + n_blocks_max * chunk
    gen = torch.Generator(device=device).manual_seed(5)
    k = torch.randn((Hkv, rows, D), generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn((Hkv, rows, D), generator=gen, device=device).to(torch.bfloat16)
    q32 = torch.randn((1, H, chunk, D), generator=gen, device=device)
    q = q32.to(torch.bfloat16).float()
    out = torch.empty_like(q)
    lse = torch.empty((1, H, chunk), device=device)
    arena = native.Arena(k, v)
    recs = torch.zeros((n_blocks_max + 1, 4), dtype=torch.int32)
    tile = 0
    for i in range(n_blocks_max):
        recs[i] = torch.tensor([cap + i * chunk, i * chunk, chunk, tile], dtype=torch.int32)
        tile += chunk // 64
    recs_d = recs.to(device)
    nbytes = native.workspace_bytes(1, H, Hkv, chunk, D, 0)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    calls, flops = [], 0.0
    for c in range(n_chunks):
        nb = max(0, c - 1)
        hot_start = nb * chunk
        hot_len = min(c + 1, 2) * chunk
        table = native.PageTableC(recs_d.data_ptr(), nb, nb * chunk, nb * (chunk // 64), 0)
        hot = native.HotWindowC(0, cap, hot_start % cap, hot_len, hot_start)
        calls.append((table, hot, c * chunk))
        flops += 4.0 * H * D * (chunk * c * chunk + chunk * (chunk + 1) / 2)
    lib = native.lib()

    def run_layer(qt):
        for table, hot, pos in calls:
            native.check(lib.rfsn_paged_attention(arena.handle, qt.data_ptr(), 1, H, Hkv, chunk, pos, ctypes.byref(table),
                                                  ctypes.byref(hot), out.data_ptr(), lse.data_ptr(), ws.data_ptr(),
                                                  nbytes, 0, native.stream_ptr()), "prefill")

    reps = max(3, min(args.steps, 10))

    def time_layer(qt):
        for _ in range(2):
            run_layer(qt)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            run_layer(qt)
        end.record()
        end.synchronize()
        native.check(lib.rfsn_workspace_check(ws.data_ptr(), native.stream_ptr(), 30_000_000), "prefill workspace")
        return start.elapsed_time(end) / reps

    ms_fp32_q = time_layer(q32)
    ms = time_layer(q)  # last: `out` holds the 16-bit q layer's last chunk
    # correctness of the last chunk (its output is what `out` holds now): the first
    # and last query row of every (query block, KV head) unit against a dense
    # float64 softmax over the keys in logical order (archived blocks, then the ring)
    rows = sorted({r for qb in range(chunk // 32) for r in (32 * qb, 32 * qb + 31)})
    q_pos0 = (n_chunks - 1) * chunk
    keys_k = torch.cat([k[:, cap:cap + n_blocks_max * chunk], k[:, :cap]], dim=1).double()  # [Hkv, 32768, D]
    keys_v = torch.cat([v[:, cap:cap + n_blocks_max * chunk], v[:, :cap]], dim=1).double()
    qs = q[0][:, rows].double().view(Hkv, H // Hkv * len(rows), D)
    sc = torch.bmm(qs, keys_k.transpose(1, 2)) / (D ** 0.5)                      # [Hkv, G * rows, 32768]
    qpos = torch.tensor([q_pos0 + r for r in rows], device=device).repeat(H // Hkv)
    sc.masked_fill_(torch.arange(keys_k.shape[1], device=device)[None, None, :] > qpos[None, :, None], float("-inf"))
    dense = torch.bmm(sc.softmax(dim=-1), keys_v).view(1, H, len(rows), D)
    parity = {"max_abs_vs_dense_fp64": float((out[:, :, rows].double() - dense).abs().max()),
              "rows_checked": f"first and last row of every unit of the last chunk ({len(rows)} rows x {H} heads)",
              "tol": PARITY_TOL}
    del keys_k, keys_v, sc, dense
    arena.close()
    tflops = flops / (ms / 1e3) / 1e12
    peak, kind = bf16_peak()
    return {
        "workload": "prefill32k_chunk2048_bf16",
        "desc": PREFILL_DESC,
        "value": 32768 / (ms / 1e3),
        "unit": "prompt tokens/s (one layer's attention)",
        "ms_per_layer": ms,
        "useful_tflop_per_layer": flops / 1e12,
        "roofline": {
            "bound": "tensor",
            "achieved": tflops,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": tflops / peak,
            "peak_kind": kind,
            "tensor_work_factor": 1.5,
            "kernel": "rfsn::prefill::prefill_attn_kernel (tcgen05, TMEM accumulators)",
        },
        "q": "bf16 values (a bf16 model's projection + RoPE output), passed as float32",
        "float32_q": {"ms_per_layer": ms_fp32_q, "tflops_useful": flops / (ms_fp32_q / 1e3) / 1e12,
                      "frac": flops / (ms_fp32_q / 1e3) / 1e12 / peak, "tensor_work_factor": 2},
        "l2": "K/V 67 MB + q/out per call; every chunk streams its whole causal context",
        "parity": parity,
    }


WARM_WORKLOAD = "warm_reload_bf16"
WARM_DESC = ("one layer, 32 q / 8 kv heads, head_dim 128, bf16; a 32,768-token context appended in chunks of 2,048 "
             "(hot ring 4,096, blocks of 2,048) with warm capacity 14,336 tokens, so half the archived blocks are "
             "cold; each decode step then reloads every cold block (the reference's policy) and demotes others")


def run_warm(args):
    """``--workload warm_reload_bf16``: decode steps whose attention needs cold
    blocks back in HBM. Disk path (npz read, checksum, decompress; demotions
    write npz) vs. the pinned host tier (reloads stream from pinned host memory
    on the side stream); residency decisions and metrics must be identical."""
    import torch

    from rfsn_b200.cache import LayerKVCache, paged_attention
    from rfsn_b200.config import RFSNConfig, RuntimeMode

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "GPU-only workload; the reference CPU arm times the "
                          "decode-attention workloads"}), flush=True)
        return 0
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    H, Hkv, D = 32, 8, 128
    results, metrics = {}, {}
    for mode, steps in (("disk", 1), ("host_tier", 32)):
        with tempfile.TemporaryDirectory() as tmp:
            cfg = RFSNConfig(hidden_dim=H * D, num_heads=H, num_kv_heads=Hkv, head_dim=D, num_layers=1,
                             hot_capacity=4096, block_size_seq=2048, warm_capacity=14336, cold_capacity=65536,
                             model_dtype="bfloat16", runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=tmp,
                             session_id="warm")
            cache = LayerKVCache(cfg, 1, H, Hkv, layer_id=0, session_id="warm", device=device,
                                 host_tier=(mode == "host_tier"))
            gen = torch.Generator(device=device).manual_seed(5)
            for a in range(0, 32768, 2048):
                k = torch.randn((1, Hkv, 2048, D), generator=gen, device=device).to(torch.bfloat16)
                v = torch.randn((1, Hkv, 2048, D), generator=gen, device=device).to(torch.bfloat16)
                cache.evict_for_append(2048)
                cache.append_exact(k, v)
            torch.cuda.synchronize()
            pos = 32768
            times = []
            for i in range(steps + 1):
                q = torch.randn((1, H, 1, D), generator=gen, device=device)
                k = torch.randn((1, Hkv, 1, D), generator=gen, device=device)
                v = torch.randn((1, Hkv, 1, D), generator=gen, device=device)
                t0 = time.perf_counter()
                # attention_step with the decode prefetch awaited right after it is
                # scheduled: residency decisions then do not depend on load speed
                cache.evict_for_append(1)
                q_rot = cache.append_rope(q, k, v, pos)
                cache.maybe_prefetch_for_decode(pos)
                cache.residency_manager.wait_for_prefetches(cache, timeout=120.0)
                paged_attention(cache, q_rot, pos, cache.get_attention_segments())
                torch.cuda.synchronize()
                if i > 0:  # the first step also seals the full ring into a new block
                    times.append(time.perf_counter() - t0)
                pos += 1
                if i == 1:  # after 2 steps: the counters the disk run ends with
                    metrics[mode + "_after_2_steps"] = dict(cache.residency_manager.get_metrics())
            m = cache.residency_manager.get_metrics()
            metrics[mode] = {"steps": steps + 1, **m}
            entry = {"steps_timed": steps, "ms_per_step": 1e3 * statistics.median(times),
                     "blocks": sum(1 for _ in cache.block_manager.iter_blocks(layer_id=0)),
                     "sync_loads_per_step": m["sync_loads"] / (steps + 1)}
            if mode == "host_tier":
                # H2D bandwidth of one reload: a held block copied pinned -> HBM on the side stream
                bid, (kp, vp) = next(iter(cache._host_tier.items()))
                n = kp.shape[1]
                row = cache._allocate_rows(n)
                cache._ops.upload(row, n, kp, vp)
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                reps = 20
                for _ in range(reps):
                    cache._ops.upload(row, n, kp, vp)
                torch.cuda.synchronize()
                dt = (time.perf_counter() - t0) / reps
                entry["h2d_gbs"] = 2 * kp.numel() * kp.element_size() / dt / 1e9
                entry["block_bytes"] = 2 * kp.numel() * kp.element_size()
            results[mode] = entry
    # identical residency decisions: the counters after the same 2 steps
    same = metrics["disk_after_2_steps"] == metrics["host_tier_after_2_steps"]
    line = {"metric": "decode step latency with cold-block reloads (ms, one layer)", "workload": WARM_WORKLOAD,
            "desc": WARM_DESC, "n_gpus": 1, "dtype": "bf16", "higher_is_better": False,
            "data": "synthetic N(0,1) K/V (seeded)", "value": results["host_tier"]["ms_per_step"], "unit": "ms/step",
            "host_tier": results["host_tier"], "disk": results["disk"], "per_step_policy_equal": same,
            "metrics": metrics}
    print(json.dumps(line), flush=True)
    return 0


MODEL_WORKLOAD = "model8b_e2e_bf16"
MODEL_DESC = ("Llama-3-8B-shaped model, random init normal(0, 0.02) seed 4: 32 layers, hidden 4096, 32 q / 8 kv "
              "heads, head_dim 128, SwiGLU FFN 14336, vocab 128256, RoPE theta 500000, bf16; 4,096-token prompt of "
              "uniform random ids prefilled in slices of 512, then 256 greedy decode steps; hot ring 2,048, blocks "
              "of 256, warm capacity 8,192 (every archived block stays in HBM)")


def run_model(args):
    """``--workload model8b_e2e_bf16``: whole-model prefill and greedy decode through
    ``rfsn_b200.model`` (dense layers in torch/cuBLAS, attention on this
    library's kernels). Timed with CUDA events; decode includes the argmax and
    the host-side cache logic of every step."""
    import torch

    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode
    from rfsn_b200.model import RFSNModel

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the 8B-shaped model needs a GPU; the reference CPU "
                          "arm times the decode-attention workloads"}), flush=True)
        return 0
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    with tempfile.TemporaryDirectory() as tmp:
        cfg = RFSNConfig(hidden_dim=4096, num_heads=32, num_kv_heads=8, head_dim=128, num_layers=32,
                         vocab_size=128256, ffn_dim=14336, rope_base=500000.0, norm_eps=1e-5, model_dtype="bfloat16",
                         hot_capacity=2048, block_size_seq=256, warm_capacity=8192, cold_capacity=16384,
                         runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=tmp, session_id="bench")
        model = RFSNModel(cfg, device=device, seed=4)
        gen = torch.Generator().manual_seed(4)
        prompt = torch.randint(0, cfg.vocab_size, (1, 4096), generator=gen, dtype=torch.int32)
        n_decode = 256

        def one_run():
            cache = RFSNCache(cfg, batch_size=1, device=device)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record()
            logits = None
            for a in range(0, 4096, 512):
                logits = model.prefill(prompt[:, a:a + 512], cache)
            ev[1].record()
            tok = torch.argmax(logits[:, -1, :], dim=-1).to(torch.int32)
            toks = [tok]
            for pos in range(4096, 4096 + n_decode - 1):
                out = model.decode_step(tok, cache, pos)
                tok = torch.argmax(out, dim=-1).to(torch.int32)
                toks.append(tok)
            ev[2].record()
            ev[2].synchronize()
            blocks = sum(1 for _ in cache.layer(0).block_manager.iter_blocks(layer_id=0))
            return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), blocks, torch.stack(toks).cpu()

        one_run()  # warm-up (cuBLAS heuristics, allocator, kernels)
        pre_ms, dec_ms, blocks, toks = one_run()
    line = {
        "metric": "model end-to-end prefill and decode tokens/s (Llama-3-8B shape, bf16)",
        "workload": MODEL_WORKLOAD, "desc": MODEL_DESC, "n_gpus": 1, "dtype": "bf16",
        "data": "synthetic: random weights and prompt ids (seeded)", "higher_is_better": True,
        "value": (n_decode - 1) / (dec_ms / 1e3), "unit": "decode tokens/s",
        "decode_ms_per_token": dec_ms / (n_decode - 1),
        "prefill_tokens_per_s": 4096 / (pre_ms / 1e3), "prefill_ms": pre_ms,
        "archived_blocks_after": blocks,
        "notes": "q|k|v and gate|up fused; decode projections on this library's GEMV, prefill projections and the "
                 "LM head on cuBLAS; RMSNorm (+ residual add), SwiGLU and attention (RoPE+append, seal, paged "
                 "attention, tcgen05 prefill) on this library's kernels",
    }
    print(json.dumps(line), flush=True)
    return 0


MODEL7B_WORKLOAD = "model7b_prefill32k_warm_bf16"
MODEL7B_DESC = ("Mistral-7B-shaped model, random init normal(0, 0.02) seed 5: 32 layers, hidden 4096, 32 q / 8 kv "
                "heads, head_dim 128, SwiGLU FFN 14336, vocab 32000, RoPE theta 1e6, bf16; 32,768-token prompt of "
                "uniform random ids prefilled in chunks of 2,048 (tensor-core chunk attention over every archived "
                "block), then greedy decode steps; hot ring 4,096, block size 512, warm capacity 14,336 tokens per "
                "layer, so half the archived blocks are cold, held in pinned host memory and reloaded by every "
                "decode step (the reference's residency policy); npz persistence of demotions write-behind")


def run_model7b(args):
    """``--workload model7b_prefill32k_warm_bf16``: whole-model chunked prefill of a
    32K prompt and greedy decode with half of every layer's archived blocks in the
    pinned host tier (demotions persisted write-behind). A throwaway 2,048-token
    prefill and two decode steps on a separate cache warm up cuBLAS and the
    kernels; the timed run starts from an empty cache. Decode runs op by op (the
    cold blocks change the page table every step)."""
    import torch

    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig, RuntimeMode
    from rfsn_b200.model import RFSNModel

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the 7B-shaped model needs a GPU; the reference CPU "
                          "arm times the decode-attention workloads"}), flush=True)
        return 0
    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    prompt_len, chunk = 32768, 2048
    n_decode = args.decode_steps if args.decode_steps is not None else 128
    with tempfile.TemporaryDirectory() as tmp:
        cfg = RFSNConfig(hidden_dim=4096, num_heads=32, num_kv_heads=8, head_dim=128, num_layers=32,
                         vocab_size=32000, ffn_dim=14336, rope_base=1e6, norm_eps=1e-5, model_dtype="bfloat16",
                         hot_capacity=4096, block_size_seq=512, warm_capacity=14336, cold_capacity=65536,
                         runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=tmp, session_id="bench7b")
        model = RFSNModel(cfg, device=device, seed=5)
        gen = torch.Generator().manual_seed(5)
        prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=gen, dtype=torch.int32)

        warm = RFSNCache(cfg, batch_size=1, device=device, host_tier=True, persist_async=True,
                         session_id="bench7b_warmup")
        logits = model.prefill(prompt[:, :chunk], warm)
        tok = torch.argmax(logits[:, -1, :], dim=-1).to(torch.int32)
        for pos in range(chunk, chunk + 2):
            tok = torch.argmax(model.decode_step(tok, warm, pos), dim=-1).to(torch.int32)
        torch.cuda.synchronize()
        warm.reset()
        del warm, logits

        cache = RFSNCache(cfg, batch_size=1, device=device, host_tier=True, persist_async=True)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        for a in range(0, prompt_len, chunk):
            logits = model.prefill(prompt[:, a:a + chunk], cache)
        ev[1].record()
        tok = torch.argmax(logits[:, -1, :], dim=-1).to(torch.int32)
        for pos in range(prompt_len, prompt_len + n_decode):
            tok = torch.argmax(model.decode_step(tok, cache, pos), dim=-1).to(torch.int32)
        ev[2].record()
        ev[2].synchronize()
        pre_ms, dec_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        layer0 = cache.layer(0)
        blocks = list(layer0.block_manager.iter_blocks(layer_id=0))
        cold = sum(1 for m in blocks if not layer0.is_manifest_resident(m))
        metrics: dict = {}
        for lc in cache.layers:
            for k, v in lc.residency_manager.get_metrics().items():
                metrics[k] = metrics.get(k, 0) + v
        pending = sum(1 for lc in cache.layers for j in lc._write_jobs if not j.done())
        # the write-behind npz persistence still queued is finished and timed, not dropped
        t_flush = time.perf_counter()
        cache.flush_persistence()
        flush_s = time.perf_counter() - t_flush
        files = sum(1 for _ in Path(tmp).rglob("*.npz"))
        cache.reset()
    pairs = prompt_len * (prompt_len + 1) // 2
    line = {
        "metric": "model end-to-end chunked prefill tokens/s and decode tokens/s with warm-tier reloads "
                  "(Mistral-7B shape, bf16)",
        "workload": MODEL7B_WORKLOAD, "desc": MODEL7B_DESC, "n_gpus": 1, "dtype": "bf16",
        "data": "synthetic: random weights and prompt ids (seeded)", "higher_is_better": True,
        "value": prompt_len / (pre_ms / 1e3), "unit": "prefill tokens/s", "prefill_ms": pre_ms,
        "prefill_attention_tflop": 4 * cfg.num_heads * cfg.head_dim * pairs * cfg.num_layers / 1e12,
        "decode_steps": n_decode, "decode_ms_per_token": dec_ms / max(n_decode, 1),
        "decode_tokens_per_s": n_decode / (dec_ms / 1e3) if n_decode else None,
        "layer0_blocks_after": len(blocks), "layer0_cold_blocks_after": cold,
        "residency_metrics_all_layers": metrics, "npz_writes_pending_at_end": pending,
        "npz_flush_s": flush_s, "npz_files_written": files,
        "notes": "prefill projections and the LM head on cuBLAS; RMSNorm, SwiGLU, RoPE+append, seals, the tcgen05 "
                 "chunk attention and the paged decode attention on this library's kernels; cold blocks reload from "
                 "pinned host memory on the side stream; npz persistence on a writer thread per layer",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_prefill(args):
    """``--workload prefill32k_chunk2048_bf16``: the chunked-prefill measurement as
    its own line (1 GPU; the reference arm has no GPU counterpart)."""
    import torch

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable": "the prefill workload is measured on the GPU arm only; "
                          "the reference CPU arm times the decode workloads"}), flush=True)
        return 0
    torch.cuda.set_device(0)
    r = prefill_32k(args, torch.device("cuda", 0))
    line = {"metric": "chunked-prefill attention prompt tokens/s and TFLOP/s (tensor roofline)", "n_gpus": 1,
            "steps": max(3, min(args.steps, 10)), "warmup": 2, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic N(0,1) q/K/V (seeded); K/V resident in HBM", **r}
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + [PREFILL_WORKLOAD, MODEL_WORKLOAD, WARM_WORKLOAD, MODEL7B_WORKLOAD], default="decode128k_bf16")
    ap.add_argument("--calls-per-step", type=int, default=200)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the chunked-prefill measurement (N = 1)")
    ap.add_argument("--decode-steps", type=int, default=None,
                    help="greedy decode steps of the model7b workload (default 128)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="time rank 0's shard of an N-way partition alone on one GPU (kernel only)")
    ap.add_argument("--merge", choices=["p2p", "nccl"], default="p2p",
                    help="cross-GPU merge for N > 1: fused NVLink mailboxes (default) or NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.workload == PREFILL_WORKLOAD:
        return run_prefill(args)
    if args.workload == MODEL_WORKLOAD:
        return run_model(args)
    if args.workload == WARM_WORKLOAD:
        return run_warm(args)
    if args.workload == MODEL7B_WORKLOAD:
        return run_model7b(args)
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, w)
    if args.shard_of > 1:
        return run_shard(args, w)
    return run_ours(args, w)


if __name__ == "__main__":
    sys.exit(main())
