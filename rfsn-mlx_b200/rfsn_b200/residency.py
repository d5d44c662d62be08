"""Warm-set sizing and sequential prefetch (drop-in for ``rfsn_v10_5.residency``).

Policy identical to the reference (residency.py:26-156) so residency
decisions and metrics match bit for bit:

* warm set bounded by ``warm_capacity`` tokens; the victim is the eligible
  (warm, materializable, unpinned, not protected) block with the smallest
  ``(last_accessed_at, logical_start)`` and is demoted to the cold tier;
* one-block sequential prefetch: the cold block right after the warm
  frontier once ``query_pos >= warm.logical_end - margin``, else the cold
  block right before a warm block under the same condition;
* completions are consumed on the caller's thread.

What changes is the data path. The worker thread reads, verifies and
decompresses the cold payload (numpy, off the caller's thread). When the
caller drains it, the payload is staged in pinned host memory and copied into
the device arena with an asynchronous host-to-device copy on a side stream;
the compute stream waits on that copy's event before its next kernel.
One exact shortcut: a decode-step prefetch check on a layer without any cold
block returns at once (both candidate rules need a cold block); when every
live block is resident in HBM that is known without a scan.
"""

from __future__ import annotations

from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import asdict, dataclass
from typing import TYPE_CHECKING, Optional

from .block_manager import BlockId, BlockLocation, BlockManifest

if TYPE_CHECKING:
    from .cache import LayerKVCache


@dataclass
class ResidencyMetrics:
    warm_evictions: int = 0
    prefetch_requests: int = 0
    prefetch_completions: int = 0
    sync_loads: int = 0
    missing_blocks: int = 0
    unmaterializable_blocks: int = 0


class ResidencyManager:
    """Manage warm-set sizing and simple sequential prefetch."""

    def __init__(self, *, prefetch_margin_tokens: int = 1) -> None:
        self.prefetch_margin_tokens = max(1, prefetch_margin_tokens)
        self._executor = ThreadPoolExecutor(max_workers=1, thread_name_prefix="rfsn-prefetch")
        self._prefetch_futures: dict[BlockId, Future] = {}
        self.metrics = ResidencyMetrics()

    @property
    def has_pending(self) -> bool:
        return bool(self._prefetch_futures)

    def reset(self) -> None:
        for future in self._prefetch_futures.values():
            future.cancel()
        self._prefetch_futures.clear()
        self.metrics = ResidencyMetrics()

    def choose_warm_eviction_victim(
        self, manifests: list[BlockManifest], *, protected_block_id: Optional[BlockId] = None
    ) -> Optional[BlockManifest]:
        best: Optional[BlockManifest] = None
        best_key = None
        for m in manifests:
            if (
                m.residency != BlockLocation.WARM_RAM
                or not m.materializable
                or m.pin_count != 0
                or m.block_id == protected_block_id
            ):
                continue
            key = (m.last_accessed_at, m.logical_start)
            if best_key is None or key < best_key:
                best, best_key = m, key
        return best

    def evict_warm_excess(self, cache: "LayerKVCache", *, protected_block_id: Optional[BlockId] = None) -> None:
        while cache._warm_token_count() > cache.config.warm_capacity:
            victim = self.choose_warm_eviction_victim(cache._warm_manifests(), protected_block_id=protected_block_id)
            if victim is None:
                return
            cache.demote_manifest_to_cold(victim)
            self.metrics.warm_evictions += 1

    def maybe_schedule_prefetch(self, cache: "LayerKVCache", query_abs_pos: int) -> None:
        self.drain_completed_prefetches(cache)
        live = cache.block_manager.page_table.layer_entries(cache.layer_id)
        # Both candidate rules need a cold block; with none, nothing can be scheduled.
        # O(1) when every live block is resident in HBM, else a scan.
        all_resident = getattr(cache, "all_blocks_resident", None)
        if all_resident is not None and all_resident():
            return
        if not any(m.residency == BlockLocation.COLD_DISK for m in live):
            return
        manifests = [m for m in live if m.materializable]
        if len(manifests) < 2:
            return
        trigger = lambda m: query_abs_pos >= m.logical_end - self.prefetch_margin_tokens  # noqa: E731
        candidate: Optional[BlockManifest] = None
        for cur, nxt in zip(manifests, manifests[1:]):
            if cur.residency == BlockLocation.WARM_RAM and nxt.residency == BlockLocation.COLD_DISK and trigger(cur):
                candidate = nxt
                break
        if candidate is None:
            for prev, cur in zip(manifests, manifests[1:]):
                if prev.residency == BlockLocation.COLD_DISK and cur.residency == BlockLocation.WARM_RAM and trigger(cur):
                    candidate = prev
                    break
        if candidate is None or candidate.block_id in self._prefetch_futures or cache.is_manifest_resident(candidate):
            return
        self._prefetch_futures[candidate.block_id] = self._executor.submit(cache.load_manifest_payload_only, candidate)
        self.metrics.prefetch_requests += 1

    def drain_completed_prefetches(self, cache: "LayerKVCache") -> None:
        if not self._prefetch_futures:
            return
        for block_id, future in list(self._prefetch_futures.items()):
            if not future.done():
                continue
            self._prefetch_futures.pop(block_id, None)
            manifest = cache.block_manager.get_block(block_id)
            try:
                payload = future.result()
            except Exception as exc:  # the worker's failure becomes a MISSING block
                cache.block_manager.mark_missing(block_id, reason=f"prefetch failed: {exc}")
                cache._note_table_change()
                self.metrics.missing_blocks += 1
                continue
            if payload is None:
                if manifest.residency == BlockLocation.MISSING:
                    self.metrics.missing_blocks += 1
                if not manifest.materializable:
                    self.metrics.unmaterializable_blocks += 1
                cache._note_table_change()
                continue
            cache.promote_manifest_from_payload(manifest, payload)
            self.evict_warm_excess(cache, protected_block_id=manifest.block_id)
            self.metrics.prefetch_completions += 1

    def wait_for_prefetches(self, cache: "LayerKVCache", *, timeout: float = 1.0) -> None:
        for future in list(self._prefetch_futures.values()):
            future.result(timeout=timeout)
        self.drain_completed_prefetches(cache)

    def note_sync_load(self) -> None:
        self.metrics.sync_loads += 1

    def get_metrics(self) -> dict[str, int]:
        return asdict(self.metrics)
