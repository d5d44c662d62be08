"""CPU baseline: the reference's segmented attention, timed on host cores.

TEST / MEASUREMENT INFRASTRUCTURE: used only by ``bench.py`` (the
``cpu_baseline`` field and the ``--impl reference`` arm). It runs the oracle's
restatement of the reference algorithm (attention_exact.py:122-164 with the
GQA ``mx.repeat`` of layer.py:140-150: float32 upcast copies of every segment,
per-segment logits kept for a second pass, global max, exp-weighted sum).
MLX itself cannot be installed here, so this port stands in for the
reference's MLX CPU backend. The work of one decode-attention call is split
over KV heads across a thread pool (numpy releases the GIL), so every host
core can be used; each head group follows the reference formula unchanged.
"""

from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .numerics import from_storage
from .segmented_attention import run_segmented_attention


def synthetic_decode_inputs(block_lens, hot_len, kv_heads, q_heads, head_dim, dtype, seed):
    """Seeded N(0,1) K/V per segment (archived blocks then the hot window) and q."""
    rng = np.random.default_rng(seed)
    segs = []
    pos = 0
    for n in list(block_lens) + ([hot_len] if hot_len else []):
        k = rng.standard_normal((1, kv_heads, n, head_dim), dtype=np.float32)
        v = rng.standard_normal((1, kv_heads, n, head_dim), dtype=np.float32)
        if dtype != "float32":
            from .numerics import to_storage

            k = from_storage(to_storage(k, dtype), dtype)
            v = from_storage(to_storage(v, dtype), dtype)
        segs.append((k, v, pos))
        pos += n
    q = rng.standard_normal((1, q_heads, 1, head_dim), dtype=np.float32)
    return q, segs, pos - 1


def attention_all_cores(q, segs, q_pos, threads: int):
    """One decode-attention call, KV heads spread over `threads` workers."""
    kv_heads = segs[0][0].shape[1]
    G = q.shape[1] // kv_heads

    def one(h):
        qh = q[:, h * G:(h + 1) * G]
        sh = [(k[:, h:h + 1], v[:, h:h + 1], s) for k, v, s in segs]
        return run_segmented_attention(qh, sh, q_pos)

    with ThreadPoolExecutor(max_workers=threads) as pool:
        parts = list(pool.map(one, range(kv_heads)))
    return np.concatenate(parts, axis=1)


def time_calls(q, segs, q_pos, *, calls: int, warmup: int = 1, budget_s: float = 30.0, threads: int | None = None):
    """Seconds per call (median), number of timed calls, threads used."""
    threads = threads or os.cpu_count() or 1
    for _ in range(warmup):
        attention_all_cores(q, segs, q_pos, threads)
    times = []
    start = time.perf_counter()
    for _ in range(calls):
        t0 = time.perf_counter()
        attention_all_cores(q, segs, q_pos, threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget_s:
            break
    return float(np.median(times)), len(times), threads
