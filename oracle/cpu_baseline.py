"""CPU baseline: the reference's segmented attention, timed on host cores.

TEST / MEASUREMENT INFRASTRUCTURE: used only by ``bench.py`` (the
``cpu_baseline`` field and the ``--impl reference`` arm). It runs the oracle's
restatement of the reference algorithm (attention_exact.py:122-164 with the
GQA ``mx.repeat`` of layer.py:140-150: float32 upcast copies of every segment,
per-segment logits kept for a second pass, global max, exp-weighted sum).
MLX itself cannot be installed here, so this port stands in for the
reference's MLX CPU backend. The work of one decode-attention call is split
into (KV head, run of consecutive segments) items on a thread pool with one
BLAS thread per worker (numpy releases the GIL), at least two items per worker,
so every host core does useful work without oversubscription. Each item follows
the reference formula unchanged over its segments and returns its log-sum-exp;
the items of a head are combined by the associative log-sum-exp form of the
same global-max merge (attention_exact.py:141-164).
"""

from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .numerics import from_storage
from .segmented_attention import merge_partials, run_segmented_attention


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


def work_items(kv_heads: int, n_segments: int, threads: int):
    """(head, first segment, end segment) items: at least 2 per worker thread
    where the segments allow it, each head's segments in consecutive runs."""
    runs = max(1, min(n_segments, -(-2 * threads // kv_heads)))
    bounds = [round(i * n_segments / runs) for i in range(runs + 1)]
    return [(h, bounds[i], bounds[i + 1]) for h in range(kv_heads) for i in range(runs) if bounds[i + 1] > bounds[i]]


def attention_all_cores(q, segs, q_pos, threads: int):
    """One decode-attention call on `threads` workers (one BLAS thread each);
    returns the output and the number of workers that had work."""
    from threadpoolctl import threadpool_limits

    kv_heads = segs[0][0].shape[1]
    G = q.shape[1] // kv_heads
    items = work_items(kv_heads, len(segs), threads)

    def one(item):
        h, a, b = item
        qh = q[:, h * G:(h + 1) * G]
        sh = [(k[:, h:h + 1], v[:, h:h + 1], s) for k, v, s in segs[a:b]]
        return run_segmented_attention(qh, sh, q_pos, return_lse=True)

    workers = min(threads, len(items))
    with threadpool_limits(limits=1), ThreadPoolExecutor(max_workers=workers) as pool:
        parts = list(pool.map(one, items))
    heads = []
    for h in range(kv_heads):
        mine = [p for it, p in zip(items, parts) if it[0] == h]
        heads.append(merge_partials([p[0] for p in mine], [p[1] for p in mine]))
    return np.concatenate(heads, axis=1), workers


def time_calls(q, segs, q_pos, *, calls: int, warmup: int = 1, budget_s: float = 30.0, threads: int | None = None):
    """Seconds per call (median), number of timed calls, threads used."""
    threads = threads or len(os.sched_getaffinity(0)) or os.cpu_count() or 1
    workers = threads
    for _ in range(warmup):
        _, workers = attention_all_cores(q, segs, q_pos, threads)
    times = []
    start = time.perf_counter()
    for _ in range(calls):
        t0 = time.perf_counter()
        _, workers = attention_all_cores(q, segs, q_pos, threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - start > budget_s:
            break
    return float(np.median(times)), len(times), workers
