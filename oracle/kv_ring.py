"""Hot ring buffer + seal rule, restated as integer bookkeeping (test infrastructure).

Follows ``rfsn_v10_5/cache.py`` of the reference:

* ring state ``head`` / ``length`` / ``start`` -> cache.py:108-110, write index
  ``(head + length) % capacity`` -> cache.py:130-131, ``hot_end`` -> :134-135.
* ``hot_spans``        -> ``_hot_span_segments`` cache.py:184-218 (one piece, or
  two when the live window wraps past the end of the buffer).
* ``evict_for_append`` -> cache.py:363-383 (oversized chunk error, EXACT-mode
  overflow error, then seal ``min(max(need, block_size), length)`` tokens from
  the head while the append would overflow).
* ``seal``             -> ``_seal_hot_prefix`` cache.py:324-339 (new block spans
  [start, start + n); head advances modulo capacity).
* ``append``           -> ``append_exact`` cache.py:341-361 (overflow error; the
  write splits at the end of the buffer).

Values are not modelled: the oracle for tensor contents keeps a float32 copy of
the ring next to this state (see ``RingContents``).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class RingOracle:
    capacity: int
    block_size: int
    exact_mode: bool = False
    head: int = 0
    length: int = 0
    start: int = 0
    sealed: list = field(default_factory=list)

    @property
    def write_index(self) -> int:
        return (self.head + self.length) % self.capacity

    @property
    def end(self) -> int:
        return self.start + self.length

    def hot_spans(self) -> list[tuple[int, int, int]]:
        """[(physical_start, length, absolute_start)] for the live window."""
        if self.length == 0:
            return []
        first = min(self.length, self.capacity - self.head)
        spans = [(self.head, first, self.start)]
        if self.length - first > 0:
            spans.append((0, self.length - first, self.start + first))
        return spans

    def seal(self, n: int) -> tuple[int, int, list[tuple[int, int]]]:
        """Seal ``n`` tokens from the head; returns (start, end, physical pieces)."""
        pieces = []
        first = min(n, self.capacity - self.head)
        pieces.append((self.head, first))
        if n - first > 0:
            pieces.append((0, n - first))
        span = (self.start, self.start + n, pieces)
        self.sealed.append((self.start, self.start + n))
        self.head = (self.head + n) % self.capacity
        self.start += n
        self.length -= n
        return span

    def evict_for_append(self, incoming: int) -> list:
        if incoming > self.capacity:
            raise RuntimeError(
                f"Chunk length {incoming} exceeds hot_capacity={self.capacity}. "
                "Call model.prefill() with chunking rather than appending oversized segments."
            )
        projected = self.length + incoming
        if self.exact_mode and projected > self.capacity:
            raise RuntimeError(
                "runtime_mode='exact' keeps all live context in the hot window; "
                f"the requested append would exceed hot_capacity={self.capacity}"
            )
        events = []
        while projected > self.capacity and self.length > 0:
            need = projected - self.capacity
            chunk = min(max(need, self.block_size), self.length)
            if chunk <= 0:
                break
            events.append(self.seal(chunk))
            projected = self.length + incoming
        return events

    def append(self, n: int) -> list[tuple[int, int]]:
        """Returns [(physical_start, count)] of the write (split at the wrap)."""
        if self.length + n > self.capacity:
            raise RuntimeError(
                f"append_exact: hot buffer overflow ({self.length + n} > {self.capacity}). "
                "Chunk prefill should evict before append."
            )
        w = self.write_index
        first = min(n, self.capacity - w)
        writes = [(w, first)] if first > 0 else []
        if n - first > 0:
            writes.append((0, n - first))
        self.length += n
        return writes


class RingContents:
    """Float32 model of one layer's K/V storage: ring + archived blocks."""

    def __init__(self, batch: int, kv_heads: int, capacity: int, head_dim: int, block_size: int, *, exact_mode=False):
        self.state = RingOracle(capacity, block_size, exact_mode)
        self.k = np.zeros((batch, kv_heads, capacity, head_dim), np.float32)
        self.v = np.zeros_like(self.k)
        self.blocks: list[tuple[np.ndarray, np.ndarray, int]] = []

    def evict_for_append(self, incoming: int) -> None:
        for start, _end, pieces in self.state.evict_for_append(incoming):
            ks = [self.k[:, :, p:p + n] for p, n in pieces]
            vs = [self.v[:, :, p:p + n] for p, n in pieces]
            self.blocks.append((np.concatenate(ks, axis=2).copy(), np.concatenate(vs, axis=2).copy(), start))

    def append(self, k: np.ndarray, v: np.ndarray) -> None:
        offset = 0
        for p, n in self.state.append(k.shape[2]):
            self.k[:, :, p:p + n] = k[:, :, offset:offset + n]
            self.v[:, :, p:p + n] = v[:, :, offset:offset + n]
            offset += n

    def segments(self) -> list[tuple[np.ndarray, np.ndarray, int]]:
        """cache.py:425-428: archived blocks in logical order, then hot pieces."""
        segs = [(k, v, s) for k, v, s in self.blocks]
        for p, n, s in self.state.hot_spans():
            segs.append((self.k[:, :, p:p + n], self.v[:, :, p:p + n], s))
        return segs
