"""Bench helpers and CLI (drop-in for rfsn_v10_5.bench / launcher bench)."""

import pytest

from rfsn_b200.__main__ import build_parser, config_from_args
from rfsn_b200.bench import BenchResult


def test_cli_defaults_match_reference_launcher():
    a = build_parser().parse_args(["bench"])
    # launcher.py:316-345 (model flags) and :370-377 (bench flags)
    assert (a.hidden_dim, a.num_heads, a.num_kv_heads, a.head_dim, a.num_layers, a.vocab_size) == (512, 8, 0, 64, 4, 50000)
    assert (a.hot_capacity, a.warm_capacity, a.cold_capacity, a.block_size_seq) == (512, 2048, 8192, 64)
    assert (a.runtime_mode, a.model_dtype, a.rope_base, a.ffn_dim) == ("archived", "bfloat16", 10000.0, 0)
    assert (a.prompt_len, a.decode_steps, a.warmup, a.repeats, a.seed_prompt_len, a.archive_seed_steps) == (256, 100, 2, 5, 8, 0)
    cfg = config_from_args(a)
    assert cfg.num_kv_heads == 8 and cfg.ffn_dim == 2048 and cfg.runtime_mode.value == "archived"


def test_bench_result_string():
    r = BenchResult("decode(steps=4)", 2.0, 1.5, 2.5, 2000.0, [1.5, 2.5])
    assert str(r) == "decode(steps=4): mean=2.0ms  min=1.5ms  max=2.5ms  throughput=2000.0 tok/s"


@pytest.mark.gpu
def test_bench_prefill_and_decode_run_with_archiving_and_warmup(tmp_path):
    from rfsn_b200.bench import bench_decode, bench_prefill
    from rfsn_b200.cache import RFSNCache
    from rfsn_b200.config import RFSNConfig
    from rfsn_b200.model import RFSNModel

    cfg = RFSNConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64, num_layers=2, vocab_size=512,
                     hot_capacity=16, block_size_seq=8, warm_capacity=64, cold_capacity=128, model_dtype="float32",
                     disk_cache_dir=str(tmp_path))
    model = RFSNModel(cfg, device="cuda", seed=1)
    cache = RFSNCache(cfg, batch_size=1, device="cuda")
    p = bench_prefill(model, cache, prompt_len=12, warmup=2, repeats=2)
    assert p.name == "prefill(len=12)" and len(p.raw_ms) == 2 and p.throughput > 0
    # warmup >= 2 raised in the reference (same position reused); here it runs
    d = bench_decode(model, cache, steps=6, warmup=3, repeats=2, seed_prompt_len=8, archive_seed_steps=20)
    assert d.name == "decode(steps=6)" and len(d.raw_ms) == 2 and d.throughput > 0
    assert cache.layer(0).hot_seq_len == 0  # reset at the end, like the reference


@pytest.mark.gpu
def test_cli_bench_runs(tmp_path, capsys):
    from rfsn_b200.__main__ import main

    main(["bench", "--hidden-dim", "128", "--num-heads", "2", "--head-dim", "64", "--num-layers", "1",
          "--vocab-size", "128", "--hot-capacity", "8", "--warm-capacity", "16", "--cold-capacity", "64",
          "--block-size-seq", "4", "--model-dtype", "float32", "--disk-cache-dir", str(tmp_path),
          "--prompt-len", "8", "--decode-steps", "5", "--warmup", "2", "--repeats", "2", "--archive-seed-steps", "9"])
    out = capsys.readouterr().out.splitlines()
    assert out[0].startswith("[bench] Model: 1L x 128d, 2H/2KVH, dtype=float32, runtime_mode=archived")
    assert out[1].startswith("prefill(len=8): mean=") and out[2].startswith("decode(steps=5): mean=")


def _run_bench(args, env_extra=None):
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    env = dict(os.environ, **(env_extra or {}))
    proc = subprocess.run([sys.executable, str(root / "bench.py"), *args], cwd=root, env=env, capture_output=True,
                          text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    return [json.loads(ln) for ln in lines]


def test_reference_arm_prints_one_contract_line_on_host_cores():
    """bench.py --impl reference: the reference algorithm on the host cores,
    one JSON line with the arm's metric, a cpu_baseline describing the run and
    an e2e object without device copies."""
    (line,) = _run_bench(["--impl", "reference", "--workload", "decode8k_fp16", "--steps", "1", "--warmup", "0"])
    assert line["impl"] == "reference" and line["n_gpus"] == 1 and line["steps"] == 1
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["config"]["workload"] == "decode8k_fp16"
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    assert _run_bench(["--impl", "reference", "--workload", "decode8k_fp16", "--steps", "1", "--warmup", "0"],
                      {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}) == []


def test_shard_rotation_keeps_every_call_out_of_l2():
    """At N > 1 every rank rotates enough copies of its shard that the copies
    together exceed twice the 126 MB L2 (the same count on every rank); one
    GPU reads the whole context and needs none."""
    import importlib.util
    from pathlib import Path

    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parent.parent / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    w = bench.WORKLOADS["decode128k_bf16"]
    total = sum(w["blocks"]) + w["hot"]
    assert bench.shard_copies(w, 1, total) == 1
    for world in (2, 4, 8):
        copies = bench.shard_copies(w, world, total)
        per_rank = bench.algorithmic_bytes(w, total) / world
        assert copies * per_rank >= bench.L2_ROTATION_BYTES >= 2 * 126e6
        assert (copies - 1) * per_rank < bench.L2_ROTATION_BYTES
    assert [bench.shard_copies(w, n, total) for n in (2, 4, 8)] == [1, 2, 4]


def test_cpu_baseline_work_items_cover_every_head_and_segment_once():
    """The CPU baseline's work items: each KV head's segments in consecutive
    runs, every (head, segment) exactly once, at least two items per worker
    where the segments allow it; the combined result equals one evaluation."""
    import numpy as np

    from oracle.cpu_baseline import attention_all_cores, synthetic_decode_inputs, work_items
    from oracle.segmented_attention import run_segmented_attention

    for heads, segs, threads in ((8, 129, 16), (8, 25, 32), (2, 3, 8), (8, 1, 4)):
        items = work_items(heads, segs, threads)
        seen = sorted((h, s) for h, a, b in items for s in range(a, b))
        assert seen == [(h, s) for h in range(heads) for s in range(segs)]
        assert len(items) >= min(2 * threads, heads * segs)
    q, seg_list, qpos = synthetic_decode_inputs([40] * 6 + [9], 30, 2, 8, 16, "float16", 5)
    out, workers = attention_all_cores(q, seg_list, qpos, 4)
    ref = run_segmented_attention(q, seg_list, qpos)
    assert workers == 4 and float(np.abs(out - ref).max()) <= 2e-6
