"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout where the reference implementation (rfsn-MLX, package
``rfsn_v10_5``) is available, e.g.::

    python tests/golden/make_golden.py --reference /root/reference

MLX cannot be installed here, so the reference's unmodified modules are imported
over ``oracle/mlx_shim`` (a torch-CPU stand-in for ``mlx``). Everything below
calls reference code: ``LayerKVCache`` for ring/seal/page-table/residency
traces, ``run_segmented_attention`` / ``exact_attention`` for attention
outputs, and ``RFSNMLX`` for the tiny end-to-end model. The fixtures written
are:

* ``segattn_golden.npz``  attention cases (inputs in their storage dtype,
  outputs float32), incl. GQA, causal Lq > 1, one-segment exact path.
* ``ring_traces.json``    ring state, seal boundaries, page tables and segment
  lists after every evict+append, for several capacity / block-size mixes,
  plus EXACT-mode errors.
* ``residency_trace.json`` warm/cold residency, prefetch and metrics for a
  small warm capacity (the reference's prefetch test scenario, extended).
* ``rope_golden.npz``     the reference's ``build_rope_tables`` and
  ``_apply_rope`` with tables in the model dtype or another dtype (the RoPE of
  a layer called without tables, or with tables passed in).
* ``model_slices_golden.npz`` two-layer float32 slices at the head geometry
  of the Llama-3-8B- and Mistral-7B-shaped configurations (head_dim 128, GQA
  4, RoPE theta 5e5 / 1e6) with small rings, blocks and warm capacity, so the
  prompt seals blocks, blocks go cold and decode steps reload them: logits,
  greedy tokens, layer-0 ring/page-table states and residency counters.
  Weights are regenerated from the seeds (``slice_weights``).
* ``tiny_model_golden.npz`` the CPU-runnable tiny model (1 layer, hidden 128,
  2/2 heads, head_dim 64, SwiGLU 4x, vocab 128, tied head, theta 1e4, fp32,
  hot 8 / block 4): prompt of 8 ids (seed 1) + 8 greedy decode steps, with
  weights drawn normal(0, 0.02) from seed 0, the logits, ring state per step
  and every attention call's q / segments / output.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _setup(reference: Path):
    sys.path.insert(0, str(REPO / "oracle" / "mlx_shim"))
    sys.path.insert(0, str(reference))
    import mlx.core as mx  # noqa: F401  (the shim)
    import rfsn_v10_5  # noqa: F401
    return mx


def _storage(arr_f32: np.ndarray, dtype: str) -> np.ndarray:
    sys.path.insert(0, str(REPO))
    from oracle.numerics import to_storage

    return to_storage(arr_f32, dtype)


# --------------------------------------------------------------------------------------
# attention cases
# --------------------------------------------------------------------------------------
ATTN_CASES = [
    # name, dtype, B, Hq, Hkv, D, segment lengths, Lq, q_start offset from end (0 = last key)
    ("gqa2_f16_d64", "float16", 1, 4, 2, 64, [7, 16, 5], 1, 0),
    ("gqa4_bf16_d128", "bfloat16", 1, 8, 2, 128, [33, 64, 1, 100, 3], 1, 0),
    ("causal_lq3_f32_d64", "float32", 1, 4, 4, 64, [8, 8, 5], 3, 2),
    ("single_segment_bf16", "bfloat16", 1, 4, 1, 128, [50], 1, 0),
    ("single_segment_causal_lq4_f32", "float32", 1, 2, 2, 64, [12], 4, 3),
    ("batch2_gqa2_f16", "float16", 2, 4, 2, 64, [9, 17, 4], 2, 1),
    ("decode8k_shape_f16", "float16", 1, 32, 8, 128, [64, 64, 64, 40, 24], 1, 0),
    ("decode128k_shape_bf16", "bfloat16", 1, 32, 8, 128, [40, 40, 24, 64], 1, 0),
]


def make_attention(mx, out_path: Path) -> None:
    from rfsn_v10_5.attention_exact import exact_attention, run_segmented_attention

    rng = np.random.default_rng(20240601)
    blobs: dict[str, np.ndarray] = {}
    names = []
    for name, dtype, B, Hq, Hkv, D, lens, Lq, back in ATTN_CASES:
        names.append(name)
        mdt = {"float16": mx.float16, "bfloat16": mx.bfloat16, "float32": mx.float32}[dtype]
        total = sum(lens)
        q = rng.standard_normal((B, Hq, Lq, D)).astype(np.float32)
        q_start = total - Lq - back
        starts = np.cumsum([0] + lens[:-1]).tolist()
        segs = []
        for i, (s, n) in enumerate(zip(starts, lens)):
            k = rng.standard_normal((B, Hkv, n, D)).astype(np.float32)
            v = rng.standard_normal((B, Hkv, n, D)).astype(np.float32)
            k_m = mx.array(k).astype(mdt)
            v_m = mx.array(v).astype(mdt)
            blobs[f"{name}/k{i}"] = _storage(np.array(k_m.astype(mx.float32)), dtype)
            blobs[f"{name}/v{i}"] = _storage(np.array(v_m.astype(mx.float32)), dtype)
            groups = Hq // Hkv
            # layer.py:140-150 expands GQA with mx.repeat before the attention call.
            segs.append((mx.repeat(k_m, groups, axis=1), mx.repeat(v_m, groups, axis=1), int(s)))
        q_m = mx.array(q)
        if len(segs) == 1:
            out = exact_attention(q_m, segs[0][0], segs[0][1], q_start_pos=q_start, k_start_pos=segs[0][2])
        else:
            out = run_segmented_attention(q_m, segs, q_start)
        blobs[f"{name}/q"] = q
        blobs[f"{name}/out"] = np.array(out.astype(mx.float32))
        blobs[f"{name}/meta"] = np.array([B, Hq, Hkv, D, Lq, q_start, len(lens)], np.int64)
        blobs[f"{name}/lens"] = np.array(lens, np.int64)
        blobs[f"{name}/starts"] = np.array(starts, np.int64)
        blobs[f"{name}/dtype"] = np.array(dtype)
    blobs["__cases__"] = np.array(names)
    np.savez_compressed(out_path, **blobs)


# --------------------------------------------------------------------------------------
# ring / seal / page-table traces
# --------------------------------------------------------------------------------------
RING_SCENARIOS = [
    # name, hot_capacity, block_size, mode, list of incoming chunk lengths
    ("tiny_model_hot8_bs4", 8, 4, "archived", [8] + [1] * 8),
    ("prefetch_hot4_bs4", 4, 4, "archived", [4, 4, 4, 1, 1, 1]),
    ("mixed_hot16_bs4", 16, 4, "archived", [5, 7, 9, 16, 1, 3, 16, 2, 1, 1, 15]),
    ("odd_hot10_bs3", 10, 3, "archived", [10, 1, 1, 1, 4, 10, 2, 9, 1, 1, 7]),
    ("block_gt_cap_hot7_bs100", 7, 100, "archived", [7, 1, 3, 7, 2]),
    ("decode_hot32_bs8", 32, 8, "archived", [32] + [1] * 40),
    ("chunks_hot2048_bs256", 2048, 256, "archived", [512, 512, 512, 512] + [1] * 300),
    ("exact_mode_overflow", 8, 4, "exact", [5, 3, 1]),
]


def _cache_state(cache) -> dict:
    spans = [
        {
            "block_id": m.block_id.block_id,
            "start": m.logical_start,
            "end": m.logical_end,
            "residency": m.residency.value,
            "materializable": m.materializable,
            "shape": list(m.shape_metadata["keys"]),
        }
        for m in cache.block_manager.iter_blocks(layer_id=cache.layer_id)
    ]
    segs = [[int(seg[2]), int(seg[0].shape[2])] for seg in cache.get_attention_segments()]
    return {
        "hot_head_index": cache.hot_head_index,
        "hot_seq_len": cache.hot_seq_len,
        "hot_start": cache.hot_start,
        "hot_write_index": cache.hot_write_index,
        "hot_end": cache.hot_end,
        "blocks": spans,
        "segments": segs,
        "total_length": cache.get_total_length(),
    }


def make_ring_traces(mx, out_path: Path) -> None:
    from rfsn_v10_5.cache import LayerKVCache
    from rfsn_v10_5.config import RFSNConfig, RuntimeMode

    out = {}
    for name, cap, bs, mode, chunks in RING_SCENARIOS:
        with tempfile.TemporaryDirectory() as tmp:
            cfg = RFSNConfig(
                hidden_dim=8, num_heads=2, num_kv_heads=1, head_dim=4, num_layers=1, vocab_size=16,
                hot_capacity=cap, warm_capacity=max(cap, 1 << 20), cold_capacity=1 << 21,
                block_size_seq=bs, runtime_mode=RuntimeMode(mode), model_dtype="float32",
                disk_cache_dir=tmp,
            )
            cache = LayerKVCache(cfg, batch_size=1, num_heads=2, num_kv_heads=1, layer_id=0, session_id="golden")
            steps = []
            pos = 0
            for n in chunks:
                rec = {"incoming": n}
                try:
                    cache.evict_for_append(n)
                    k = mx.array(np.arange(pos, pos + n, dtype=np.float32)[None, None, :, None] * np.ones((1, 1, 1, 4), np.float32))
                    cache.append_exact(k, k + 0.5)
                    pos += n
                    rec.update(_cache_state(cache))
                except RuntimeError as exc:
                    rec["error"] = str(exc)
                steps.append(rec)
            out[name] = {"hot_capacity": cap, "block_size": bs, "mode": mode, "steps": steps}
    out_path.write_text(json.dumps(out, indent=1, sort_keys=True))


def make_residency_trace(mx, out_path: Path) -> None:
    from rfsn_v10_5.cache import LayerKVCache
    from rfsn_v10_5.config import RFSNConfig, RuntimeMode

    scenarios = {}
    for name, cap, warm, bs, chunks in [
        ("hot4_warm4_bs4", 4, 4, 4, [4, 4, 4] + [1] * 10),
        ("hot8_warm8_bs4", 8, 8, 4, [8, 8, 8] + [1] * 12),
        ("hot4_warm12_bs2", 4, 12, 2, [4, 4, 4, 4, 4] + [1] * 9),
    ]:
        with tempfile.TemporaryDirectory() as tmp:
            cfg = RFSNConfig(
                hidden_dim=8, num_heads=2, num_kv_heads=1, head_dim=4, num_layers=1, vocab_size=16,
                hot_capacity=cap, warm_capacity=warm, cold_capacity=1 << 20, block_size_seq=bs,
                runtime_mode=RuntimeMode.ARCHIVED, model_dtype="float32", disk_cache_dir=tmp,
            )
            cache = LayerKVCache(cfg, batch_size=1, num_heads=2, num_kv_heads=1, layer_id=0, session_id="golden")
            steps = []
            pos = 0
            for n in chunks:
                cache.evict_for_append(n)
                k = mx.array(np.arange(pos, pos + n, dtype=np.float32)[None, None, :, None] * np.ones((1, 1, 1, 4), np.float32))
                cache.append_exact(k, -k)
                if n == 1:
                    # layer.py:136-137 (decode only), then wait so the trace is deterministic.
                    cache.maybe_prefetch_for_decode(pos)
                    cache.residency_manager.wait_for_prefetches(cache)
                pos += n
                before = [m.residency.value for m in cache.block_manager.iter_blocks(layer_id=0)]
                segs = cache.get_attention_segments()
                rec = {
                    "incoming": n,
                    "residency_before_fetch": before,
                    "residency_after_fetch": [m.residency.value for m in cache.block_manager.iter_blocks(layer_id=0)],
                    "spans": [[m.logical_start, m.logical_end] for m in cache.block_manager.iter_blocks(layer_id=0)],
                    "segments": [[int(s[2]), int(s[0].shape[2])] for s in segs],
                    "segment_first_values": [float(np.array(s[0])[0, 0, 0, 0]) for s in segs],
                    "metrics": cache.residency_manager.get_metrics(),
                    "hot": [cache.hot_head_index, cache.hot_seq_len, cache.hot_start],
                }
                steps.append(rec)
            scenarios[name] = {"hot_capacity": cap, "warm_capacity": warm, "block_size": bs, "steps": steps}
    out_path.write_text(json.dumps(scenarios, indent=1, sort_keys=True))


# --------------------------------------------------------------------------------------
# tiny end-to-end model
# --------------------------------------------------------------------------------------
def tiny_model_weights(param_shapes: dict[str, tuple[int, ...]]) -> dict[str, np.ndarray]:
    """normal(0, 0.02) from seed 0 for every projection/embedding weight in
    sorted-name order; norm weights keep their reference initialisation."""
    rng = np.random.default_rng(0)
    out = {}
    for key in sorted(param_shapes):
        if "norm" in key:
            continue
        out[key] = rng.normal(0.0, 0.02, size=param_shapes[key]).astype(np.float32)
    return out


def make_tiny_model(mx, out_path: Path) -> None:
    import rfsn_v10_5.layer as ref_layer
    from mlx.utils import tree_flatten, tree_unflatten
    from rfsn_v10_5.cache import RFSNCache
    from rfsn_v10_5.config import RFSNConfig, RuntimeMode
    from rfsn_v10_5.model import RFSNMLX

    with tempfile.TemporaryDirectory() as tmp:
        cfg = RFSNConfig(
            hidden_dim=128, num_heads=2, num_kv_heads=2, head_dim=64, num_layers=1, vocab_size=128,
            hot_capacity=8, block_size_seq=4, rope_base=10000.0, ffn_multiplier=4, model_dtype="float32",
            runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=tmp, session_id="tiny",
        )
        model = RFSNMLX(cfg)
        shapes = {k: tuple(v.shape) for k, v in tree_flatten(model.parameters())}
        weights = tiny_model_weights(shapes)
        model.update(tree_unflatten([(k, mx.array(v)) for k, v in weights.items()]))
        cache = RFSNCache(cfg, batch_size=1)

        calls: list[dict] = []
        orig_exact, orig_seg = ref_layer.exact_attention, ref_layer.run_segmented_attention

        def rec_exact(q, k, v, q_start_pos, k_start_pos):
            out = orig_exact(q, k, v, q_start_pos=q_start_pos, k_start_pos=k_start_pos)
            calls.append({"q": np.array(q), "segs": [(np.array(k), np.array(v), int(k_start_pos))], "q_start": q_start_pos, "out": np.array(out)})
            return out

        def rec_seg(q, segments, q_start_pos):
            out = orig_seg(q, segments, q_start_pos)
            calls.append({"q": np.array(q), "segs": [(np.array(k), np.array(v), int(s)) for k, v, s in segments], "q_start": q_start_pos, "out": np.array(out)})
            return out

        ref_layer.exact_attention, ref_layer.run_segmented_attention = rec_exact, rec_seg
        try:
            prompt = np.random.default_rng(1).integers(0, 128, size=(1, 8)).astype(np.int32)
            logits = model.prefill(mx.array(prompt), cache)
            states = []
            lc = cache.layer(0)

            def snap():
                states.append([lc.hot_head_index, lc.hot_seq_len, lc.hot_start] + [
                    x for m in lc.block_manager.iter_blocks(layer_id=0) for x in (m.logical_start, m.logical_end)
                ])

            snap()
            token = mx.argmax(logits[:, -1, :], axis=-1).astype(mx.int32)
            tokens = [int(np.array(token)[0])]
            dec_logits = []
            pos = 8
            for _ in range(8):
                out = model.decode_step(token, cache, pos)
                dec_logits.append(np.array(out))
                snap()
                token = mx.argmax(out, axis=-1).astype(mx.int32)
                tokens.append(int(np.array(token)[0]))
                pos += 1
        finally:
            ref_layer.exact_attention, ref_layer.run_segmented_attention = orig_exact, orig_seg

        blobs = {f"w/{k}": v for k, v in weights.items()}
        blobs["prompt"] = prompt
        blobs["prefill_logits"] = np.array(logits)
        blobs["decode_logits"] = np.stack(dec_logits)
        blobs["tokens"] = np.array(tokens, np.int32)
        width = max(len(s) for s in states)
        blobs["ring_states"] = np.array([s + [-1] * (width - len(s)) for s in states], np.int64)
        blobs["n_calls"] = np.array(len(calls))
        for i, c in enumerate(calls):
            blobs[f"call{i}/q"] = c["q"]
            blobs[f"call{i}/q_start"] = np.array(c["q_start"])
            blobs[f"call{i}/out"] = c["out"]
            blobs[f"call{i}/nseg"] = np.array(len(c["segs"]))
            for j, (k, v, s) in enumerate(c["segs"]):
                blobs[f"call{i}/k{j}"] = k
                blobs[f"call{i}/v{j}"] = v
                blobs[f"call{i}/s{j}"] = np.array(s)
        np.savez_compressed(out_path, **blobs)


MODEL_SLICES = [
    # name, seed, config overrides, prompt length, decode steps
    ("cfg4_slice", 4, dict(rope_base=500000.0, vocab_size=256, hot_capacity=32, block_size_seq=16,
                           warm_capacity=48, cold_capacity=4096), 96, 12),
    ("cfg5_slice", 5, dict(rope_base=1e6, vocab_size=320, hot_capacity=64, block_size_seq=32, warm_capacity=64,
                           cold_capacity=4096), 192, 12),
]
SLICE_DIMS = dict(hidden_dim=1024, num_heads=8, num_kv_heads=2, head_dim=128, num_layers=2, ffn_dim=3584,
                  norm_eps=1e-5, model_dtype="float32")


class _InlineExecutor:
    """Runs a submitted load at once on the caller's thread: a prefetch is
    complete as soon as it is scheduled, so the residency decisions of a run do
    not depend on when a worker thread finishes (a deterministic schedule of
    the reference's policy)."""

    def submit(self, fn, *args):
        from concurrent.futures import Future

        f = Future()
        try:
            f.set_result(fn(*args))
        except Exception as exc:  # noqa: BLE001 - delivered through the future, as a pool would
            f.set_exception(exc)
        return f


def slice_weights(param_shapes: dict[str, tuple[int, ...]], seed: int) -> dict[str, np.ndarray]:
    """normal(0, 0.02) float32 from ``seed`` for every projection/embedding
    weight in sorted-name order; norm weights keep their initialisation."""
    rng = np.random.default_rng(seed)
    return {k: rng.normal(0.0, 0.02, size=param_shapes[k]).astype(np.float32)
            for k in sorted(param_shapes) if "norm" not in k}


def make_model_slices(mx, out_path: Path) -> None:
    from mlx.utils import tree_flatten, tree_unflatten
    from rfsn_v10_5.cache import RFSNCache
    from rfsn_v10_5.config import RFSNConfig, RuntimeMode
    from rfsn_v10_5.model import RFSNMLX

    blobs: dict[str, np.ndarray] = {}
    for name, seed, over, n_prompt, n_decode in MODEL_SLICES:
        with tempfile.TemporaryDirectory() as tmp:
            cfg = RFSNConfig(**SLICE_DIMS, **over, runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=tmp,
                             session_id=name.replace("_", "-"))
            model = RFSNMLX(cfg)
            shapes = {k: tuple(v.shape) for k, v in tree_flatten(model.parameters())}
            model.update(tree_unflatten([(k, mx.array(v)) for k, v in slice_weights(shapes, seed).items()]))
            cache = RFSNCache(cfg, batch_size=1)
            for i in range(cfg.num_layers):  # prefetches complete when scheduled: no timing races
                cache.layer(i).residency_manager._executor = _InlineExecutor()
            prompt = np.random.default_rng(seed + 100).integers(0, cfg.vocab_size, size=(1, n_prompt)).astype(np.int32)
            logits = model.prefill(mx.array(prompt), cache)
            lc = cache.layer(0)
            states = []

            def snap():
                states.append([lc.hot_head_index, lc.hot_seq_len, lc.hot_start] + [
                    x for m in lc.block_manager.iter_blocks(layer_id=0)
                    for x in (m.logical_start, m.logical_end, 1 if m.residency.value == "warm_ram" else 0)])

            snap()
            token = mx.argmax(logits[:, -1, :], axis=-1).astype(mx.int32)
            tokens = [int(np.array(token)[0])]
            dec = []
            pos = n_prompt
            for _ in range(n_decode):
                out = model.decode_step(token, cache, pos)
                dec.append(np.array(out))
                snap()
                token = mx.argmax(out, axis=-1).astype(mx.int32)
                tokens.append(int(np.array(token)[0]))
                pos += 1
            metrics = [[cache.layer(i).residency_manager.get_metrics()[k] for k in sorted(
                cache.layer(i).residency_manager.get_metrics())] for i in range(cfg.num_layers)]
        width = max(len(x) for x in states)
        blobs[f"{name}/prompt"] = prompt
        blobs[f"{name}/prefill_logits"] = np.array(logits)
        blobs[f"{name}/decode_logits"] = np.stack(dec)
        blobs[f"{name}/tokens"] = np.array(tokens, np.int32)
        blobs[f"{name}/ring_states"] = np.array([x + [-1] * (width - len(x)) for x in states], np.int64)
        blobs[f"{name}/residency_metrics"] = np.array(metrics, np.int64)
    blobs["__cases__"] = np.array([c[0] for c in MODEL_SLICES])
    np.savez_compressed(out_path, **blobs)


ROPE_CASES = [
    # name, x dtype, table dtype, heads, L, D, start position, base
    ("bf16_tables_bf16", "bfloat16", "bfloat16", 4, 5, 128, 131000, 500000.0),
    ("bf16_tables_f32", "bfloat16", "float32", 4, 3, 128, 4093, 1e6),
    ("f16_tables_f16", "float16", "float16", 2, 4, 64, 70, 10000.0),
    ("f16_tables_bf16", "float16", "bfloat16", 2, 2, 128, 30000, 500000.0),
    ("f32_tables_bf16", "float32", "bfloat16", 2, 3, 64, 9, 10000.0),
]


def make_rope(mx, out_path: Path) -> None:
    from rfsn_v10_5.layer import _apply_rope, build_rope_tables

    rng = np.random.default_rng(20240607)
    blobs: dict[str, np.ndarray] = {}
    for name, xd, td, H, L, D, start, base in ROPE_CASES:
        x32 = rng.standard_normal((1, H, L, D)).astype(np.float32)
        x = mx.array(x32).astype(getattr(mx, xd))  # layer.py:116-118: q/k in the model dtype
        cos_t, sin_t = build_rope_tables(D, base, L, start_pos=start, dtype=getattr(mx, td))
        out = _apply_rope(x, cos_t, sin_t)
        f32 = lambda a: np.array(a.astype(mx.float32))  # noqa: E731
        blobs[f"{name}/x"] = _storage(f32(x), xd)
        blobs[f"{name}/cos"] = _storage(f32(cos_t), td)
        blobs[f"{name}/sin"] = _storage(f32(sin_t), td)
        blobs[f"{name}/out"] = f32(out)
        blobs[f"{name}/meta"] = np.array([H, L, D, start], np.int64)
        blobs[f"{name}/base"] = np.array(base, np.float64)
        blobs[f"{name}/dtypes"] = np.array([xd, td, str(out.dtype).split(".")[-1]])
    blobs["__cases__"] = np.array([c[0] for c in ROPE_CASES])
    np.savez_compressed(out_path, **blobs)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RFSN_REFERENCE", "/root/reference"))
    ap.add_argument("--out", default=str(HERE), help="directory the fixtures are written to")
    args = ap.parse_args()
    out = Path(args.out).resolve()
    out.mkdir(parents=True, exist_ok=True)
    mx = _setup(Path(args.reference))
    os.chdir(tempfile.mkdtemp())
    make_attention(mx, out / "segattn_golden.npz")
    make_ring_traces(mx, out / "ring_traces.json")
    make_residency_trace(mx, out / "residency_trace.json")
    make_tiny_model(mx, out / "tiny_model_golden.npz")
    make_rope(mx, out / "rope_golden.npz")
    make_model_slices(mx, out / "model_slices_golden.npz")
    for p in sorted(out.iterdir()):
        if p.suffix in (".npz", ".json"):
            print(f"{p.name}: {p.stat().st_size} bytes")


if __name__ == "__main__":
    main()
