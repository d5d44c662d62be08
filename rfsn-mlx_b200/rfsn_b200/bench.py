"""Prefill / decode timing helpers (drop-in for ``rfsn_v10_5.bench``, bench.py:58-243).

``bench_prefill`` times time-to-first-token for a zero prompt of
``prompt_len`` tokens (the cache is reset before every iteration);
``bench_decode`` seeds the cache with a zero prompt (plus optional
``archive_seed_steps`` decode steps that push the context into archived
blocks) and times ``steps`` greedy decode steps. Both return a
``BenchResult`` with wall-clock statistics in milliseconds.

Differences from the reference, on purpose:
* the device is synchronised (``torch.cuda.synchronize``) at the end of each
  timed iteration instead of ``mx.eval`` after every forward pass; the argmax
  of one step feeds the next on the device, so nothing waits in between;
* warm-up decode steps run at consecutive positions. The reference re-used
  one position for every warm-up step (bench.py:219-222), so any
  ``warmup >= 2`` raised in ``_validate_decode_bounds``.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import List

import torch

from .cache import RFSNCache
from .model import RFSNModel


@dataclass
class BenchResult:
    """bench.py:58-91: timings of one benchmark run."""

    name: str
    mean_ms: float
    min_ms: float
    max_ms: float
    throughput: float
    raw_ms: List[float] = field(default_factory=list)

    def __str__(self) -> str:
        return (
            f"{self.name}: mean={self.mean_ms:.1f}ms  "
            f"min={self.min_ms:.1f}ms  max={self.max_ms:.1f}ms  "
            f"throughput={self.throughput:.1f} tok/s"
        )


def _sync(model: RFSNModel) -> None:
    if model.device.type == "cuda":
        torch.cuda.synchronize(model.device)


def _result(name: str, raw_ms: List[float], tokens: int) -> BenchResult:
    mean_ms = sum(raw_ms) / len(raw_ms)
    return BenchResult(name=name, mean_ms=mean_ms, min_ms=min(raw_ms), max_ms=max(raw_ms),
                       throughput=tokens / (mean_ms / 1000.0), raw_ms=raw_ms)


def bench_prefill(model: RFSNModel, cache: RFSNCache, prompt_len: int = 256, batch_size: int = 1, warmup: int = 2,
                  repeats: int = 5) -> BenchResult:
    """bench.py:94-154: time-to-first-token of a zero prompt."""
    if repeats < 1:
        raise ValueError("repeats must be >= 1")
    prompt_ids = torch.zeros((batch_size, prompt_len), dtype=torch.int32)

    def _run() -> None:
        cache.reset(clear_persisted=False)
        model.prefill(prompt_ids, cache)
        _sync(model)

    cache.reset(clear_persisted=True)
    try:
        for _ in range(warmup):
            _run()
        raw_ms: List[float] = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            _run()
            raw_ms.append((time.perf_counter() - t0) * 1000.0)
    finally:
        cache.reset(clear_persisted=True)
    return _result(f"prefill(len={prompt_len})", raw_ms, prompt_len)


def bench_decode(model: RFSNModel, cache: RFSNCache, steps: int = 100, batch_size: int = 1, warmup: int = 5,
                 repeats: int = 3, seed_prompt_len: int = 8, archive_seed_steps: int = 0) -> BenchResult:
    """bench.py:157-243: greedy decode throughput after a zero seed prompt."""
    if repeats < 1:
        raise ValueError("repeats must be >= 1")
    seed_ids = torch.zeros((batch_size, seed_prompt_len), dtype=torch.int32)

    def _decode(pos: int, n: int) -> int:
        token_id = torch.zeros((batch_size,), dtype=torch.int32, device=model.device)
        for step in range(n):
            out = model.decode_step(token_id, cache, pos + step)
            token_id = torch.argmax(out, dim=-1).to(torch.int32)
        return pos + n

    def _seed_cache() -> int:
        cache.reset(clear_persisted=False)
        model.prefill(seed_ids, cache)
        return _decode(seed_prompt_len, archive_seed_steps)

    cache.reset(clear_persisted=True)
    try:
        _decode(_seed_cache(), warmup)
        _sync(model)
        raw_ms: List[float] = []
        for _ in range(repeats):
            pos = _seed_cache()
            _sync(model)
            t0 = time.perf_counter()
            _decode(pos, steps)
            _sync(model)
            raw_ms.append((time.perf_counter() - t0) * 1000.0)
    finally:
        cache.reset(clear_persisted=True)
    return _result(f"decode(steps={steps})", raw_ms, steps)
