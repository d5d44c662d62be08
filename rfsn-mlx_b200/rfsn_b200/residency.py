"""Warm-set bound and one-block sequential prefetch for one layer's blocks.

Drop-in for ``rfsn_v10_5.residency`` (residency.py:26-156): the decisions
and the counters are the reference's, so residency traces replay bit for bit.

* Demotion: while the warm set holds more than ``warm_capacity`` tokens, the
  warm, materializable, unpinned block (other than a protected one) with the
  smallest ``(last_accessed_at, logical_start)`` goes to the cold tier.
* Prefetch: along the layer's materializable blocks in page-table order, the
  first warm -> cold boundary whose warm block the query has (nearly) reached
  (``query_pos >= logical_end - margin``) names the cold block after it; failing
  that, the first cold -> warm boundary whose warm block is reached names the
  cold block before it. One load per block in flight, on one worker thread.
* Completions are applied on the caller's thread when it next drains them.

The pieces are separate here: two pure decision functions over manifests
(``demotion_victim`` and ``prefetch_target``, one pass each), a small queue of
loads in flight (``_LoadQueue``), and the manager that applies their outcomes
to the cache. The data path is this package's: the worker reads, verifies
and decompresses a cold payload; applying it stages the payload in pinned
memory and copies it into the device arena on a side stream, which the
compute stream waits on before its next kernel. A layer with no cold block
skips the prefetch scan (both rules need one).
"""

from __future__ import annotations

from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import asdict, dataclass
from typing import TYPE_CHECKING, Callable, Iterator, Optional, Sequence

from .block_manager import BlockId, BlockLocation, BlockManifest

if TYPE_CHECKING:
    from .cache import LayerKVCache

_WARM, _COLD = BlockLocation.WARM_RAM, BlockLocation.COLD_DISK


@dataclass
class ResidencyMetrics:
    """Counters of residency.py:26-33 (same names, reported by get_metrics)."""

    warm_evictions: int = 0
    prefetch_requests: int = 0
    prefetch_completions: int = 0
    sync_loads: int = 0
    missing_blocks: int = 0
    unmaterializable_blocks: int = 0


def demotion_victim(manifests: Sequence[BlockManifest], protected: Optional[BlockId] = None) -> Optional[BlockManifest]:
    """The block a full warm set gives up: least recently used among the
    demotable ones, ties broken by the earlier position (residency.py:51-66)."""
    best: Optional[tuple] = None
    for m in manifests:
        if m.residency != _WARM or not m.materializable or m.pin_count or m.block_id == protected:
            continue
        rank = (m.last_accessed_at, m.logical_start)
        if best is None or rank < best[0]:
            best = (rank, m)
    return None if best is None else best[1]


def prefetch_target(blocks: Sequence[BlockManifest], query_pos: int, margin: int) -> Optional[BlockManifest]:
    """The cold block to load next for a query at ``query_pos`` (residency.py:85-130),
    found in one walk over adjacent pairs: a warm -> cold boundary whose warm
    side is reached wins at once; otherwise the first cold -> warm boundary
    whose warm side is reached."""
    behind: Optional[BlockManifest] = None
    for left, right in zip(blocks, blocks[1:]):
        if left.residency == _WARM and right.residency == _COLD:
            if query_pos >= left.logical_end - margin:
                return right
        elif behind is None and left.residency == _COLD and right.residency == _WARM:
            if query_pos >= right.logical_end - margin:
                behind = left
    return behind


class _LoadQueue:
    """Cold-payload loads on one worker thread, keyed by block. With
    ``inline`` set a load runs on the caller's thread when it is submitted
    (its result waits for the next drain like any finished load): residency
    decisions then follow one fixed schedule, whatever the thread timing."""

    def __init__(self) -> None:
        self._pool = ThreadPoolExecutor(max_workers=1, thread_name_prefix="rfsn-prefetch")
        self._inflight: dict[BlockId, Future] = {}
        self.inline = False

    def __len__(self) -> int:
        return len(self._inflight)

    def __contains__(self, block_id: BlockId) -> bool:
        return block_id in self._inflight

    def submit(self, block_id: BlockId, load: Callable, manifest: BlockManifest) -> None:
        if not self.inline:
            self._inflight[block_id] = self._pool.submit(load, manifest)
            return
        done: Future = Future()
        try:
            done.set_result(load(manifest))
        except Exception as exc:  # noqa: BLE001 - delivered by the drain, as from the worker
            done.set_exception(exc)
        self._inflight[block_id] = done

    def finished(self) -> Iterator[tuple[BlockId, Future]]:
        """Loads that are done when the walk reaches them, oldest first, each
        handed out once (loads submitted meanwhile wait for the next walk)."""
        for block_id, future in list(self._inflight.items()):
            if future.done():
                del self._inflight[block_id]
                yield block_id, future

    def wait_all(self, timeout: float) -> None:
        for future in list(self._inflight.values()):
            future.result(timeout=timeout)

    def clear(self) -> None:
        for future in self._inflight.values():
            future.cancel()
        self._inflight.clear()


class ResidencyManager:
    """Manage warm-set sizing and sequential prefetch of one layer's blocks."""

    def __init__(self, *, prefetch_margin_tokens: int = 1) -> None:
        self.prefetch_margin_tokens = max(1, prefetch_margin_tokens)
        self._loads = _LoadQueue()
        self.metrics = ResidencyMetrics()

    @property
    def has_pending(self) -> bool:
        return len(self._loads) > 0

    @property
    def inline_loads(self) -> bool:
        """Run prefetch loads on the caller's thread when they are scheduled
        (a deterministic schedule for replays and parity runs); off by default."""
        return self._loads.inline

    @inline_loads.setter
    def inline_loads(self, value: bool) -> None:
        self._loads.inline = bool(value)

    def reset(self) -> None:
        self._loads.clear()
        self.metrics = ResidencyMetrics()

    def choose_warm_eviction_victim(
        self, manifests: list[BlockManifest], *, protected_block_id: Optional[BlockId] = None
    ) -> Optional[BlockManifest]:
        return demotion_victim(manifests, protected_block_id)

    def evict_warm_excess(self, cache: "LayerKVCache", *, protected_block_id: Optional[BlockId] = None) -> None:
        cap = cache.config.warm_capacity
        while cache._warm_token_count() > cap:
            victim = demotion_victim(cache._warm_manifests(), protected_block_id)
            if victim is None:
                break
            cache.demote_manifest_to_cold(victim)
            self.metrics.warm_evictions += 1

    def maybe_schedule_prefetch(self, cache: "LayerKVCache", query_abs_pos: int) -> None:
        self.drain_completed_prefetches(cache)
        if cache.all_blocks_resident():
            return
        live = cache.block_manager.page_table.layer_entries(cache.layer_id)
        if all(m.residency != _COLD for m in live):
            return
        target = prefetch_target([m for m in live if m.materializable], query_abs_pos, self.prefetch_margin_tokens)
        if target is None or target.block_id in self._loads or cache.is_manifest_resident(target):
            return
        self._loads.submit(target.block_id, cache.load_manifest_payload_only, target)
        self.metrics.prefetch_requests += 1

    def drain_completed_prefetches(self, cache: "LayerKVCache") -> None:
        if not self.has_pending:
            return
        for block_id, future in self._loads.finished():
            manifest = cache.block_manager.get_block(block_id)
            error = future.exception()
            if error is not None:
                # a load that raised leaves the block MISSING (residency.py:131-134)
                cache.block_manager.mark_missing(block_id, reason=f"prefetch failed: {error}")
                self.metrics.missing_blocks += 1
            else:
                payload = future.result()
                if payload is not None:
                    cache.promote_manifest_from_payload(manifest, payload)
                    self.evict_warm_excess(cache, protected_block_id=block_id)
                    self.metrics.prefetch_completions += 1
                    continue
                # no payload: the storage marked it missing or unreadable
                self.metrics.missing_blocks += manifest.residency == BlockLocation.MISSING
                self.metrics.unmaterializable_blocks += not manifest.materializable
            cache._note_table_change()

    def wait_for_prefetches(self, cache: "LayerKVCache", *, timeout: float = 1.0) -> None:
        self._loads.wait_all(timeout)
        self.drain_completed_prefetches(cache)

    def note_sync_load(self) -> None:
        self.metrics.sync_loads += 1

    def get_metrics(self) -> dict[str, int]:
        return asdict(self.metrics)
