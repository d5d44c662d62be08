"""Exact per-layer KV cache on the device (drop-in for ``rfsn_v10_5.cache``).

The Python surface (class names, constructor arguments, methods, attributes,
ring / seal / residency semantics and error messages) follows the reference
(cache.py:41-559). The storage underneath is B200-native:

* **Arena.** Each layer owns one K and one V tensor in HBM laid out
  ``[batch * kv_heads][rows][head_dim]`` in the model dtype. Rows
  ``[0, hot_capacity)`` are the hot ring buffer; the remaining rows form the
  warm block pool. An archived block is a contiguous run of rows per head, so
  every block (and every ring piece) is a contiguous ``tokens x head_dim``
  slab per head, which the decode kernel streams with TMA.
* **Device page table.** The attended archived blocks (page-table order,
  resident, materializable) are mirrored into a device int32 array of records
  ``{row, logical_start, token_count, tile_begin}`` that the attention kernels
  walk; it is re-uploaded only when the set of blocks or their rows changes.
* **Seal** (cache.py:324-339) copies the ring's oldest rows into freshly
  allocated pool rows with one device kernel; append (cache.py:341-361) is the
  fused RoPE + ring-write kernel.
* **Warm <-> cold.** Demotion downloads the block's rows and persists them
  in the reference's npz format; loads (synchronous or prefetched) upload the
  payload into newly allocated pool rows.

Segments returned by ``get_*_attention_segments`` are a ``PagedSegments``
sequence: indexing or iterating it yields ``(k, v, start)`` tensor views
exactly like the reference's list, while ``attention_exact`` recognises it and
runs the paged kernel straight off the device page table. Views alias the
arena: they stay valid until the next ``evict_for_append`` / ``append`` on the
layer (rows freed by a demotion are only reused after that point).
"""

from __future__ import annotations

import hashlib
import json
import shutil
import threading
import time
import uuid
from collections.abc import Sequence
from concurrent.futures import Future, ThreadPoolExecutor
from pathlib import Path
from typing import Any, Optional

import numpy as np
import torch

from . import _native as native
from .block_manager import BlockId, BlockLocation, BlockManager, BlockManifest, BlockSpan
from .config import RFSNConfig, RuntimeMode, resolve_dtype, validate_session_id
from .residency import ResidencyManager
from .storage import BlockStorage

_EXACT_CODEC_VERSION = "v11-exact-kv"


def derive_model_id(config: RFSNConfig) -> str:
    """sha256 of the stable config fields, first 16 hex chars (cache.py:41-56)."""
    fields = (
        "hidden_dim", "num_heads", "num_kv_heads", "head_dim", "num_layers", "vocab_size", "rope_base", "ffn_dim",
        "norm_eps", "model_dtype",
    )
    payload = {name: getattr(config, name) for name in fields}
    blob = json.dumps(payload, sort_keys=True, separators=(",", ":")).encode("utf-8")
    return hashlib.sha256(blob).hexdigest()[:16]


def _resolve_session_id(config: RFSNConfig, session_id: Optional[str], *, restore: bool) -> str:
    """cache.py:59-72."""
    candidate = validate_session_id(session_id if session_id is not None else config.session_id)
    if candidate:
        return candidate
    if restore:
        raise ValueError(
            "restore_cache requires an explicit session_id so the persisted archive can be resolved safely"
        )
    return uuid.uuid4().hex


def _tiles(n: int) -> int:
    return (n + native.TILE_KEYS - 1) // native.TILE_KEYS


class _RowAllocator:
    """First-fit allocator of row ranges inside the block pool."""

    def __init__(self, start: int, end: int) -> None:
        self.start, self.end = start, end
        self.free: list[list[int]] = [[start, end]]

    def allocate(self, n: int) -> Optional[int]:
        for i, (a, b) in enumerate(self.free):
            if b - a >= n:
                if b - a == n:
                    self.free.pop(i)
                else:
                    self.free[i][0] = a + n
                return a
        return None

    def release(self, row: int, n: int) -> None:
        lo, hi = row, row + n
        i = 0
        while i < len(self.free) and self.free[i][0] < lo:
            i += 1
        self.free.insert(i, [lo, hi])
        merged: list[list[int]] = []
        for a, b in self.free:
            if merged and merged[-1][1] == a:
                merged[-1][1] = b
            else:
                merged.append([a, b])
        self.free = merged

    def grow(self, new_end: int) -> None:
        if self.free and self.free[-1][1] == self.end:
            self.free[-1][1] = new_end
        else:
            self.free.append([self.end, new_end])
        self.end = new_end

    def reset(self) -> None:
        self.free = [[self.start, self.end]]


def _as(x: torch.Tensor, device: torch.device, dtype: torch.dtype) -> torch.Tensor:
    """x on ``device`` in ``dtype``, contiguous; returned as is when it already is
    (the per-call conversions of the decode path are mostly no-ops)."""
    if x.dtype == dtype and x.device == device and x.is_contiguous():
        return x
    return x.to(device=device, dtype=dtype).contiguous()


class DeviceOps:
    """Device mechanics of one layer cache: arena allocation, ring writes,
    seal copies, block transfers and the page-table upload. Every method is a
    native CUDA call; there is no host fallback. (Tests may substitute an
    object with the same methods to exercise the bookkeeping without a GPU.)"""

    def __init__(self, device: Optional[torch.device | str] = None) -> None:
        native.lib()  # raises NativeUnavailable without the library or a CUDA device
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.arena: Optional[native.Arena] = None
        self._upload_stream: Optional[torch.cuda.Stream] = None
        self._inflight: list[tuple[torch.cuda.Event, Any]] = []

    def new_arena(self, groups: int, rows: int, head_dim: int, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        k = torch.zeros((groups, rows, head_dim), dtype=dtype, device=self.device)
        v = torch.zeros_like(k)
        self.arena = native.Arena(k, v)
        return k, v

    def copy_rows(self, src_row0: int, src_offset: int, src_wrap: int, dst_row0: int, count: int) -> None:
        native.check(
            native.lib().rfsn_arena_copy_rows(self.arena.handle, src_row0, src_offset, src_wrap, dst_row0, count,
                                              native.stream_ptr()),
            "rfsn_arena_copy_rows",
        )

    def append(self, q: Optional[torch.Tensor], k: torch.Tensor, v: torch.Tensor, inv_freq: Optional[torch.Tensor],
               start_pos: int, capacity: int, write_index: int) -> Optional[torch.Tensor]:
        B, Hkv, L, D = (int(x) for x in k.shape)
        q_out = None
        if q is not None:
            q_out = torch.empty(q.shape, dtype=torch.float32, device=self.device)
        native.check(
            native.lib().rfsn_rope_append(
                q.data_ptr() if q is not None else None, k.data_ptr(), v.data_ptr(), native.dtype_code(k.dtype),
                inv_freq.data_ptr() if inv_freq is not None else None, int(start_pos), B,
                int(q.shape[1]) if q is not None else 0, Hkv, L, D,
                q_out.data_ptr() if q_out is not None else None, self.arena.handle, 0, capacity, write_index,
                native.stream_ptr(),
            ),
            "rfsn_rope_append",
        )
        return q_out

    def append_tables(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos_t: Optional[torch.Tensor],
                      sin_t: Optional[torch.Tensor], table_dtype: torch.dtype, inv_freq: torch.Tensor, start_pos: int,
                      capacity: int, write_index: int) -> torch.Tensor:
        B, Hkv, L, D = (int(x) for x in k.shape)
        q_out = torch.empty(q.shape, dtype=torch.float32, device=self.device)
        native.check(
            native.lib().rfsn_rope_append_tables(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), native.dtype_code(k.dtype),
                cos_t.data_ptr() if cos_t is not None else None, sin_t.data_ptr() if sin_t is not None else None,
                native.dtype_code(table_dtype), inv_freq.data_ptr(), int(start_pos), B, int(q.shape[1]), Hkv, L, D,
                q_out.data_ptr(), self.arena.handle, 0, capacity, write_index, native.stream_ptr(),
            ),
            "rfsn_rope_append_tables",
        )
        return q_out

    def rotate_q(self, q: torch.Tensor, inv_freq: torch.Tensor, start_pos: int) -> torch.Tensor:
        B, H, L, D = (int(x) for x in q.shape)
        q_out = torch.empty(q.shape, dtype=torch.float32, device=self.device)
        native.check(
            native.lib().rfsn_rope_append(
                q.data_ptr(), None, None, native.dtype_code(q.dtype), inv_freq.data_ptr(), int(start_pos), B, H, 0, L,
                D, q_out.data_ptr(), self.arena.handle, 0, 1, 0, native.stream_ptr(),
            ),
            "rfsn_rope_append",
        )
        return q_out

    def download(self, row: int, n: int, out_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
        a = self.arena
        k_host = torch.empty((a.groups, n, a.head_dim), dtype=a.dtype, pin_memory=True)
        v_host = torch.empty_like(k_host, pin_memory=True)
        native.check(
            native.lib().rfsn_block_download(a.handle, row, n, k_host.data_ptr(), v_host.data_ptr(),
                                             native.stream_ptr(), None),
            "rfsn_block_download",
        )
        torch.cuda.current_stream().synchronize()
        return k_host.to(out_dtype), v_host.to(out_dtype)

    def download_pinned(self, row: int, n: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Arena rows -> pinned host tensors in the arena dtype (no conversion)."""
        a = self.arena
        k_host = torch.empty((a.groups, n, a.head_dim), dtype=a.dtype, pin_memory=True)
        v_host = torch.empty_like(k_host, pin_memory=True)
        native.check(
            native.lib().rfsn_block_download(a.handle, row, n, k_host.data_ptr(), v_host.data_ptr(),
                                             native.stream_ptr(), None),
            "rfsn_block_download",
        )
        torch.cuda.current_stream().synchronize()
        return k_host, v_host

    def upload(self, row: int, n: int, k_host: torch.Tensor, v_host: torch.Tensor) -> None:
        """Host -> arena copy on a side stream from pinned memory; the current
        (compute) stream waits on the copy's event before later kernels. Tensors
        already pinned, contiguous and in the arena dtype are copied as they are."""
        k = k_host.to(self.arena.dtype).contiguous().pin_memory()
        v = v_host.to(self.arena.dtype).contiguous().pin_memory()
        if self._upload_stream is None:
            self._upload_stream = torch.cuda.Stream(device=self.device)
        side = self._upload_stream
        side.wait_stream(torch.cuda.current_stream())  # the rows may still be read by earlier kernels
        native.check(
            native.lib().rfsn_block_upload(self.arena.handle, row, n, k.data_ptr(), v.data_ptr(),
                                           native.stream_ptr(side), None),
            "rfsn_block_upload",
        )
        # Recorded through torch: a torch.cuda.Event has no CUDA event until torch
        # records it (its handle reads 0 before), and waiting on an unrecorded one
        # does nothing.
        done = torch.cuda.Event()
        done.record(side)
        torch.cuda.current_stream().wait_event(done)
        self._inflight.append((done, (k, v)))
        self._inflight = [(e, keep) for e, keep in self._inflight if not e.query()]

    def new_table(self, rows: int) -> torch.Tensor:
        return torch.zeros((rows, 4), dtype=torch.int32, device=self.device)


class PagedSegments(Sequence):
    """Segments of one layer: archived blocks (page-table order) then hot pieces.

    A sequence of ``(k, v, start)`` with ``k``/``v`` views shaped
    ``[batch, kv_heads, n, head_dim]`` (cache.py:184-218, :413-428), created
    on access. ``attention_exact`` uses the attached device page table instead.
    """

    def __init__(self, cache: "LayerKVCache", archived: list[tuple[int, int, int]], hot: list[tuple[int, int, int]],
                 table: Optional[tuple[torch.Tensor, int, int, int]], hot_state: Optional[tuple[int, int, int]]):
        self.cache = cache
        self.spans = archived + hot           # (row, start, length)
        self.n_archived = len(archived)
        self.table = table                    # (device records, n_blocks, archived_tokens, archived_tiles) or None
        self.hot_state = hot_state            # (head_index, length, start) or None when hot pieces excluded

    def __len__(self) -> int:
        return len(self.spans)

    def _view(self, i: int) -> tuple[torch.Tensor, torch.Tensor, int]:
        row, start, n = self.spans[i]
        c = self.cache
        k = c._arena_k[:, row:row + n, :].unflatten(0, (c.batch_size, c.num_kv_heads))
        v = c._arena_v[:, row:row + n, :].unflatten(0, (c.batch_size, c.num_kv_heads))
        return k, v, start

    def __getitem__(self, i):  # type: ignore[override]
        if isinstance(i, slice):
            return [self._view(j) for j in range(*i.indices(len(self)))]
        if i < 0:
            i += len(self)
        if not 0 <= i < len(self):
            raise IndexError(i)
        return self._view(i)

    @property
    def total_tokens(self) -> int:
        return sum(n for _, _, n in self.spans)


class LayerKVCache:
    """Exact KV cache for one transformer layer, resident in HBM."""

    def __init__(
        self,
        config: RFSNConfig,
        batch_size: int,
        num_heads: int,
        num_kv_heads: Optional[int] = None,
        *,
        layer_id: int = 0,
        model_id: Optional[str] = None,
        session_id: str,
        device: Optional[torch.device | str] = None,
        pool_tokens: Optional[int] = None,
        ops: Optional[Any] = None,
        host_tier: bool = False,
        persist_async: bool = False,
    ) -> None:
        if persist_async and not host_tier:
            raise ValueError("persist_async requires host_tier=True (the pinned copy serves reloads meanwhile)")
        self.config = config
        self.batch_size = batch_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        self.layer_id = layer_id
        self.model_id = model_id or derive_model_id(config)
        self.session_id = session_id
        self.dtype = resolve_dtype(config.model_dtype)
        self.storage_array_dtype = np.float16 if self.dtype == torch.float16 else np.float32
        self._ops = ops if ops is not None else DeviceOps(device)
        self.device = self._ops.device

        cap = config.hot_capacity
        biggest_block = max(cap, config.block_size_seq)
        pool = pool_tokens if pool_tokens is not None else config.warm_capacity + 2 * biggest_block
        self._ring_rows = cap
        self._alloc = _RowAllocator(cap, cap + max(pool, 1))
        self._make_arena(cap + max(pool, 1))

        self.hot_seq_len = 0
        self.hot_start = 0
        self.hot_head_index = 0

        self.block_manager = BlockManager(self.model_id)
        self.storage = BlockStorage(Path(config.disk_cache_dir) / self.model_id / self.session_id / f"layer_{layer_id}")
        self.residency_manager = ResidencyManager(prefetch_margin_tokens=max(1, config.block_size_seq // 2))
        self._resident_rows: dict[BlockId, int] = {}
        # Pinned host copies of demoted blocks (arena dtype), when enabled: the
        # warm/cold policy and the npz persistence are unchanged, but a reload
        # streams the block from pinned host memory on the side stream instead of
        # reading, verifying and decompressing the npz file.
        self._host_tier: Optional[dict[BlockId, tuple[torch.Tensor, torch.Tensor]]] = {} if host_tier else None
        # Write-behind persistence (optional, host tier only): a demotion stages
        # the manifest change on the caller's thread and one writer thread per
        # layer compresses, hashes and writes the npz and sidecars in the order
        # they were staged. flush_persistence() waits for them; restore and
        # reset flush (or drop) them first.
        self._writer: Optional[ThreadPoolExecutor] = (
            ThreadPoolExecutor(max_workers=1, thread_name_prefix="rfsn-persist") if persist_async else None
        )
        self._write_jobs: list[Future] = []
        self._persisted: set[BlockId] = set()
        # Sidecar rewrites not yet started, one per block: a newer state of the
        # same block replaces the queued one instead of queueing another write.
        self._queued_sidecars: dict[BlockId, dict[str, Any]] = {}
        self._sidecar_lock = threading.Lock()
        self._deferred_free: list[tuple[int, int]] = []
        self._block_serial = 0

        self._table_dev = self._ops.new_table(1)
        self._attended: list[BlockManifest] = []
        self._attended_spans: list[tuple[int, int, int]] = []
        self._table_meta = (0, 0, 0)
        self._dirty = True
        self._seen_version = -1
        self._inv_freq: Optional[torch.Tensor] = None

    # ------------------------------------------------------------------ storage
    def _make_arena(self, rows: int) -> None:
        groups = self.batch_size * self.num_kv_heads
        self._arena_k, self._arena_v = self._ops.new_arena(groups, rows, self.config.head_dim, self.dtype)

    def _grow_arena(self, min_extra: int) -> None:
        old_rows = self._arena_k.shape[1]
        new_rows = max(old_rows * 2, old_rows + min_extra)
        old_k, old_v = self._arena_k, self._arena_v
        self._make_arena(new_rows)
        self._arena_k[:, :old_rows].copy_(old_k)
        self._arena_v[:, :old_rows].copy_(old_v)
        self._alloc.grow(new_rows)
        self._dirty = True

    def _allocate_rows(self, n: int) -> int:
        row = self._alloc.allocate(n)
        if row is None:
            self._grow_arena(n)
            row = self._alloc.allocate(n)
            assert row is not None
        return row

    def _free_rows(self, row: int, n: int) -> None:
        self._deferred_free.append((row, n))

    def _flush_deferred_free(self) -> None:
        for row, n in self._deferred_free:
            self._alloc.release(row, n)
        self._deferred_free.clear()

    def _note_table_change(self) -> None:
        self._dirty = True

    @property
    def arena(self) -> native.Arena:
        return self._ops.arena

    # ------------------------------------------------------------------ reference surface
    @property
    def model_root(self) -> Path:
        return Path(self.config.disk_cache_dir) / self.model_id

    @property
    def session_root(self) -> Path:
        return self.model_root / self.session_id

    @property
    def hot_write_index(self) -> int:
        return (self.hot_head_index + self.hot_seq_len) % self.config.hot_capacity

    @property
    def hot_end(self) -> int:
        return self.hot_start + self.hot_seq_len

    @property
    def hot_k(self) -> torch.Tensor:
        return self._arena_k[:, : self._ring_rows].unflatten(0, (self.batch_size, self.num_kv_heads))

    @property
    def hot_v(self) -> torch.Tensor:
        return self._arena_v[:, : self._ring_rows].unflatten(0, (self.batch_size, self.num_kv_heads))

    def _clear_device_state(self) -> None:
        self._arena_k.zero_()
        self._arena_v.zero_()
        self._alloc.reset()
        self._resident_rows.clear()
        if self._host_tier is not None:
            self._host_tier.clear()
        self._deferred_free.clear()
        self._attended, self._attended_spans = [], []
        self._dirty = True

    def flush_persistence(self) -> None:
        """Wait for every npz and sidecar write staged by write-behind demotions
        of this layer; raises RuntimeError with the first failure."""
        jobs, self._write_jobs = self._write_jobs, []
        first: Optional[BaseException] = None
        for job in jobs:
            try:
                job.result()
            except Exception as exc:  # noqa: BLE001 - reported below, after every job has ended
                first = first or exc
        if first is not None:
            raise RuntimeError(f"write-behind persistence failed at layer {self.layer_id}: {first}") from first

    def _drop_pending_writes(self) -> None:
        """Cancel staged writes that have not started and wait for the running one."""
        jobs, self._write_jobs = self._write_jobs, []
        for job in jobs:
            job.cancel()
        for job in jobs:
            if not job.cancelled():
                try:
                    job.result()
                except Exception:  # noqa: BLE001 - the files are being removed anyway
                    pass
        self._persisted.clear()
        with self._sidecar_lock:
            self._queued_sidecars.clear()

    def _stage_write(self, fn, *args) -> None:
        self._write_jobs = [j for j in self._write_jobs if not j.done() or j.exception() is not None]
        self._write_jobs.append(self._writer.submit(fn, *args))

    def _stage_sidecar(self, manifest: BlockManifest) -> None:
        snapshot = manifest.to_dict()
        with self._sidecar_lock:
            queued = manifest.block_id in self._queued_sidecars
            self._queued_sidecars[manifest.block_id] = snapshot
        if not queued:
            self._stage_write(self._write_queued_sidecar, manifest)

    def _write_queued_sidecar(self, manifest: BlockManifest) -> None:
        with self._sidecar_lock:
            snapshot = self._queued_sidecars.pop(manifest.block_id, None)
        if snapshot is not None:
            self.storage.write_snapshot(manifest, snapshot)

    def reset(self, *, clear_persisted: bool = True) -> None:
        """cache.py:137-150."""
        if self._writer is not None:
            if clear_persisted:
                self._drop_pending_writes()
            else:
                self.flush_persistence()
                self._persisted.clear()
        self._clear_device_state()
        self.hot_seq_len = 0
        self.hot_start = 0
        self.hot_head_index = 0
        self.block_manager.clear()
        self._block_serial = 0
        self.residency_manager.reset()
        if clear_persisted:
            shutil.rmtree(self.storage.root_dir, ignore_errors=True)
            self.storage.root_dir.mkdir(parents=True, exist_ok=True)
            self.storage.quarantine_dir.mkdir(parents=True, exist_ok=True)

    def restore_from_disk(self) -> list[BlockManifest]:
        """cache.py:152-175: rebuild the page table from persisted manifests."""
        if self._writer is not None:
            self.flush_persistence()
            self._persisted.clear()
        self._clear_device_state()
        self.hot_seq_len = 0
        self.hot_head_index = 0
        self.hot_start = 0
        self.block_manager.clear()
        manifests = self.storage.rebuild_manager(self.block_manager)
        contiguous_end = 0
        for manifest in manifests:
            if manifest.residency == BlockLocation.MISSING or not manifest.materializable:
                raise RuntimeError(
                    f"Persisted archive for session '{self.session_id}' contains an unreadable block "
                    f"at layer {self.layer_id}; restore cannot safely continue"
                )
            if manifest.logical_start != contiguous_end:
                raise RuntimeError(
                    f"Persisted archive for session '{self.session_id}' contains a gap at layer "
                    f"{self.layer_id}: expected {contiguous_end}, found {manifest.logical_start}"
                )
            contiguous_end = manifest.logical_end
        self.hot_start = contiguous_end
        return manifests

    def _empty_context(self) -> tuple[torch.Tensor, torch.Tensor, int, int]:
        empty = self._arena_k[:, :0].unflatten(0, (self.batch_size, self.num_kv_heads))
        return empty, empty, self.hot_start, self.hot_start

    def _hot_pieces(self, logical_start: int = 0, length: Optional[int] = None) -> list[tuple[int, int, int]]:
        """(row, absolute start, length) of the live window (cache.py:184-218)."""
        if self.hot_seq_len == 0:
            return []
        if length is None:
            length = self.hot_seq_len - logical_start
        if length <= 0:
            return []
        cap = self.config.hot_capacity
        phys = (self.hot_head_index + logical_start) % cap
        first = min(length, cap - phys)
        pieces = [(phys, self.hot_start + logical_start, first)] if first > 0 else []
        if length - first > 0:
            pieces.append((0, self.hot_start + logical_start + first, length - first))
        return pieces

    def _hot_span_segments(self, logical_start: int = 0, length: Optional[int] = None) -> PagedSegments:
        return PagedSegments(self, [], self._hot_pieces(logical_start, length), None, None)

    def _materialize_hot_span(self, logical_start: int = 0, length: Optional[int] = None):
        segs = self._hot_span_segments(logical_start, length)
        if len(segs) == 0:
            return self._empty_context()
        views = list(segs)
        k = views[0][0] if len(views) == 1 else torch.cat([s[0] for s in views], dim=2)
        v = views[0][1] if len(views) == 1 else torch.cat([s[1] for s in views], dim=2)
        start = int(views[0][2])
        return k, v, start, start + k.shape[2]

    def _storage_dtype_name(self) -> str:
        return np.dtype(self.storage_array_dtype).name

    def _next_block_manifest(self, start: int, end: int, dtype_name: str) -> BlockManifest:
        """cache.py:236-248."""
        block_id = BlockId(self.model_id, self.layer_id, f"block-{self._block_serial:08d}")
        self._block_serial += 1
        shape = (self.batch_size, self.num_kv_heads, end - start, self.config.head_dim)
        return BlockManifest(
            block_id=block_id,
            span=BlockSpan(start, end),
            codec_version=_EXACT_CODEC_VERSION,
            dtype=dtype_name,
            shape_metadata={"keys": shape, "values": shape},
            residency=BlockLocation.WARM_RAM,
        )

    def _warm_manifests(self) -> list[BlockManifest]:
        return [
            m for m in self.block_manager.page_table.layer_entries(self.layer_id) if m.residency == BlockLocation.WARM_RAM
        ]

    def _warm_token_count(self) -> int:
        return sum(
            m.token_count
            for m in self.block_manager.page_table.layer_entries(self.layer_id)
            if m.residency == BlockLocation.WARM_RAM
        )

    # ------------------------------------------------------------------ warm <-> cold
    def _download_block(self, row: int, n: int) -> dict[str, np.ndarray]:
        out_dtype = torch.float16 if self.storage_array_dtype == np.float16 else torch.float32
        k_host, v_host = self._ops.download(row, n, out_dtype)
        shape = (self.batch_size, self.num_kv_heads, n, self.config.head_dim)
        return {"keys": k_host.numpy().reshape(shape), "values": v_host.numpy().reshape(shape)}

    def _spill_manifest_to_disk(self, manifest: BlockManifest) -> None:
        """cache.py:280-295."""
        row = self._resident_rows.pop(manifest.block_id, None)
        self._dirty = True
        if row is None:
            self.block_manager.mark_unmaterializable(manifest.block_id, reason="warm payload missing from resident set")
            return
        if self._host_tier is not None:
            n = manifest.token_count
            if self._writer is not None:
                persisted = manifest.block_id in self._persisted
            else:
                persisted = bool(manifest.checksum and manifest.payload_path and Path(manifest.payload_path).exists())
            if manifest.block_id in self._host_tier and persisted:
                # already persisted and held in pinned memory: the state change of
                # persist_block without rewriting identical bytes
                self._free_rows(row, n)
                manifest.residency = BlockLocation.COLD_DISK
                manifest.materializable = True
                manifest.failure_reason = None
                manifest.touch()
                if self._writer is not None:
                    self._stage_sidecar(manifest)
                else:
                    self.storage.write_manifest(manifest)
                return
            k_pin, v_pin = self._ops.download_pinned(row, n)
            self._free_rows(row, n)
            self._host_tier[manifest.block_id] = (k_pin, v_pin)
            out = np.float16 if self.storage_array_dtype == np.float16 else np.float32
            shape = (self.batch_size, self.num_kv_heads, n, self.config.head_dim)

            def payload() -> dict[str, np.ndarray]:
                return {"keys": k_pin.to(torch.float32).numpy().astype(out).reshape(shape),
                        "values": v_pin.to(torch.float32).numpy().astype(out).reshape(shape)}

            if self._writer is not None:
                self.storage.stage_persist(manifest, np.dtype(out).name)
                self._persisted.add(manifest.block_id)
                snapshot = manifest.to_dict()
                self._stage_write(lambda: self.storage.write_staged(manifest, snapshot, payload()))
                return
            arrays = payload()
            manifest.dtype = arrays["keys"].dtype.name
            self.storage.persist_block(manifest, arrays)
            return
        payload = self._download_block(row, manifest.token_count)
        self._free_rows(row, manifest.token_count)
        manifest.dtype = payload["keys"].dtype.name
        self.storage.persist_block(manifest, payload)

    def demote_manifest_to_cold(self, manifest: BlockManifest) -> None:
        self._spill_manifest_to_disk(manifest)

    def _spill_warm_if_needed(self) -> None:
        self.residency_manager.evict_warm_excess(self)

    def is_manifest_resident(self, manifest: BlockManifest) -> bool:
        return manifest.block_id in self._resident_rows

    def all_blocks_resident(self) -> bool:
        """Every live block of this layer has rows in the arena (the resident set
        only ever holds live blocks, so equal sizes mean no cold block)."""
        return len(self._resident_rows) == len(self.block_manager.page_table.layer_entries(self.layer_id))

    def load_manifest_payload_only(self, manifest: BlockManifest) -> Optional[dict[str, np.ndarray]]:
        if self._host_tier is not None:
            held = self._host_tier.get(manifest.block_id)
            if held is not None:
                return {"keys": held[0], "values": held[1]}  # pinned tensors, arena dtype
        return self.storage.load_block(manifest)

    def promote_manifest_from_payload(self, manifest: BlockManifest, payload: dict[str, np.ndarray]) -> None:
        """cache.py:309-319: the payload is uploaded into fresh pool rows."""
        n = manifest.token_count
        groups, D = self.batch_size * self.num_kv_heads, self.config.head_dim
        keys, values = payload["keys"], payload["values"]
        if isinstance(keys, torch.Tensor):
            k, v = keys.reshape(groups, n, D), values.reshape(groups, n, D)
        else:
            k = torch.as_tensor(np.asarray(keys)).reshape(groups, n, D)
            v = torch.as_tensor(np.asarray(values)).reshape(groups, n, D)
        row = self._allocate_rows(n)
        self._ops.upload(row, n, k, v)
        self._resident_rows[manifest.block_id] = row
        manifest.residency = BlockLocation.WARM_RAM
        manifest.touch()
        self._dirty = True

    def maybe_prefetch_for_decode(self, query_abs_pos: int) -> None:
        self.residency_manager.maybe_schedule_prefetch(self, query_abs_pos)

    # ------------------------------------------------------------------ ring
    def _seal_hot_prefix(self, prefix_len: int) -> None:
        """cache.py:324-339: the oldest prefix_len ring tokens become a block."""
        start, end = self.hot_start, self.hot_start + prefix_len
        row = self._allocate_rows(prefix_len)
        self._ops.copy_rows(0, self.hot_head_index, self.config.hot_capacity, row, prefix_len)
        manifest = self._next_block_manifest(start, end, self._storage_dtype_name())
        self.block_manager.register_block(manifest)
        self._resident_rows[manifest.block_id] = row
        self._dirty = True
        self.hot_head_index = (self.hot_head_index + prefix_len) % self.config.hot_capacity
        self.hot_start = end
        self.hot_seq_len -= prefix_len
        self._spill_warm_if_needed()

    def _check_append(self, seq_len: int) -> None:
        end = self.hot_seq_len + seq_len
        if end > self.config.hot_capacity:
            raise RuntimeError(
                f"append_exact: hot buffer overflow ({end} > {self.config.hot_capacity}). "
                "Chunk prefill should evict before append."
            )

    def _kv_arg(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 4 or x.shape[0] != self.batch_size or x.shape[1] != self.num_kv_heads:
            raise ValueError(f"expected K/V shaped [{self.batch_size}, {self.num_kv_heads}, L, {self.config.head_dim}]")
        return _as(x, self.device, self.dtype)

    def append_exact(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """cache.py:341-361: write already-rotated K and V into the ring."""
        seq_len = int(k.shape[2])
        self._check_append(seq_len)
        kc, vc = self._kv_arg(k), self._kv_arg(v)
        self._ops.append(None, kc, vc, None, 0, self.config.hot_capacity, self.hot_write_index)
        self.hot_seq_len += seq_len

    def inv_freq(self) -> torch.Tensor:
        """1 / base ** (arange(0, half) / half) in float32 (layer.py:29), on the device."""
        if self._inv_freq is None:
            half = self.config.head_dim // 2
            exponent = np.arange(0, half, dtype=np.float32) / np.float32(half)
            table = (np.float32(1.0) / np.power(np.float32(self.config.rope_base), exponent, dtype=np.float32)).astype(
                np.float32
            )
            self._inv_freq = torch.from_numpy(table).to(self.device)
        return self._inv_freq

    def append_rope(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, start_pos: int) -> torch.Tensor:
        """Fused layer.py:131-135: RoPE on q and k, then append k, v to the ring.

        q: [B, H, L, D], k/v: [B, Hkv, L, D] in any float dtype (cast to the
        model dtype first, layer.py:116-118). Returns the rotated q in float32.
        """
        seq_len = int(k.shape[2])
        self._check_append(seq_len)
        qc = _as(q, self.device, self.dtype)
        kc, vc = self._kv_arg(k), self._kv_arg(v)
        q_out = self._ops.append(qc, kc, vc, self.inv_freq(), int(start_pos), self.config.hot_capacity,
                                 self.hot_write_index)
        self.hot_seq_len += seq_len
        return q_out

    def append_rope_tables(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, start_pos: int,
                           rope_tables: Optional[tuple] = None) -> torch.Tensor:
        """layer.py:118-135 for a layer called with ``rope_tables``, or without
        them: RoPE from the given (cos, sin) tables ([L, D] each, used as given)
        or from tables built in the model dtype (build_rope_tables with
        dtype = the model dtype), every product and sum rounded to the promoted
        dtype of q/k and the tables; then the append. Returns the rotated q as
        float32 (holding values of that promoted dtype)."""
        seq_len = int(k.shape[2])
        D = self.config.head_dim
        cos_t = sin_t = None
        table_dtype = self.dtype
        if rope_tables is not None:
            if not isinstance(rope_tables, (tuple, list)) or len(rope_tables) != 2:
                raise ValueError("rope_tables must be a (cos, sin) pair of tensors")
            cos_t, sin_t = rope_tables
            if not (isinstance(cos_t, torch.Tensor) and isinstance(sin_t, torch.Tensor)):
                raise ValueError("rope_tables must be a (cos, sin) pair of tensors")
            if cos_t.dtype != sin_t.dtype or cos_t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                raise ValueError("rope_tables: cos and sin must share one float dtype (float32, float16, bfloat16)")
            if tuple(cos_t.shape[-2:]) != (seq_len, D) or tuple(sin_t.shape[-2:]) != (seq_len, D) or \
                    cos_t.numel() != seq_len * D or sin_t.numel() != seq_len * D:
                raise ValueError(f"rope_tables must be [{seq_len}, {D}] (one row per new position)")
            table_dtype = cos_t.dtype
            cos_t = cos_t.to(self.device).reshape(seq_len, D).contiguous()
            sin_t = sin_t.to(self.device).reshape(seq_len, D).contiguous()
        self._check_append(seq_len)
        qc = _as(q, self.device, self.dtype)
        kc, vc = self._kv_arg(k), self._kv_arg(v)
        q_out = self._ops.append_tables(qc, kc, vc, cos_t, sin_t, table_dtype, self.inv_freq(), int(start_pos),
                                        self.config.hot_capacity, self.hot_write_index)
        self.hot_seq_len += seq_len
        return q_out

    def rope_query(self, q: torch.Tensor, start_pos: int) -> torch.Tensor:
        """RoPE on q alone (layer.py:131) for a shard that does not own the hot window."""
        qc = q.to(device=self.device, dtype=self.dtype).contiguous()
        return self._ops.rotate_q(qc, self.inv_freq(), int(start_pos))

    def import_block(self, k: torch.Tensor, v: torch.Tensor, logical_start: int) -> BlockManifest:
        """Register an exact archived block from device K/V [B, Hkv, n, D]
        (already rotated) at absolute positions logical_start .. + n, as a
        warm block of this layer. Used to assemble context shards and to load
        blocks produced elsewhere; the page-table rules (no overlap) apply."""
        kc, vc = self._kv_arg(k), self._kv_arg(v)
        n = int(kc.shape[2])
        manifest = self._next_block_manifest(int(logical_start), int(logical_start) + n, self._storage_dtype_name())
        self.block_manager.register_block(manifest)
        row = self._allocate_rows(n)
        groups, D = self.batch_size * self.num_kv_heads, self.config.head_dim
        self._arena_k[:, row:row + n].copy_(kc.reshape(groups, n, D))
        self._arena_v[:, row:row + n].copy_(vc.reshape(groups, n, D))
        self._resident_rows[manifest.block_id] = row
        self._dirty = True
        return manifest

    def evict_for_append(self, incoming_len: int) -> None:
        """cache.py:363-383: seal from the head until the append fits."""
        self._flush_deferred_free()
        cap = self.config.hot_capacity
        if incoming_len > cap:
            raise RuntimeError(
                f"Chunk length {incoming_len} exceeds hot_capacity={cap}. "
                "Call model.prefill() with chunking rather than appending oversized segments."
            )
        projected = self.hot_seq_len + incoming_len
        if self.config.runtime_mode == RuntimeMode.EXACT and projected > cap:
            raise RuntimeError(
                "runtime_mode='exact' keeps all live context in the hot window; "
                f"the requested append would exceed hot_capacity={cap}"
            )
        while projected > cap and self.hot_seq_len > 0:
            chunk = min(max(projected - cap, self.config.block_size_seq), self.hot_seq_len)
            if chunk <= 0:
                break
            self._seal_hot_prefix(chunk)
            projected = self.hot_seq_len + incoming_len

    # ------------------------------------------------------------------ segments
    def _load_archived_payload(self, manifest: BlockManifest) -> Optional[int]:
        """cache.py:385-408; returns the block's arena row."""
        self.residency_manager.drain_completed_prefetches(self)
        row = self._resident_rows.get(manifest.block_id)
        if row is not None:
            manifest.touch()
            return row
        if manifest.residency == BlockLocation.WARM_RAM:
            self.block_manager.mark_unmaterializable(manifest.block_id, reason="warm payload missing from resident set")
            self._dirty = True
            return None
        if manifest.residency == BlockLocation.COLD_DISK:
            self.residency_manager.note_sync_load()
            payload = self.load_manifest_payload_only(manifest)
            if payload is None:
                self._dirty = True
                return None
            self.promote_manifest_from_payload(manifest, payload)
            self.residency_manager.evict_warm_excess(self, protected_block_id=manifest.block_id)
            return self._resident_rows[manifest.block_id]
        return None

    def _refresh_archived(self) -> None:
        """Walk the page table like cache.py:413-423 and rebuild the device table."""
        attended: list[BlockManifest] = []
        spans: list[tuple[int, int, int]] = []
        for manifest in self.block_manager.iter_blocks(layer_id=self.layer_id):
            if manifest.residency == BlockLocation.MISSING or not manifest.materializable:
                continue
            row = self._load_archived_payload(manifest)
            if row is None:
                continue
            attended.append(manifest)
            spans.append((row, manifest.logical_start, manifest.token_count))
        records = np.zeros((len(spans) + 1, 4), dtype=np.int32)
        tile = 0
        for i, (row, start, n) in enumerate(spans):
            records[i] = (row, start, n, tile)
            tile += _tiles(n)
        records[len(spans), 3] = tile
        if self._table_dev.shape[0] < records.shape[0]:
            self._table_dev = self._ops.new_table(max(records.shape[0], 2 * self._table_dev.shape[0]))
        self._table_dev[: records.shape[0]].copy_(torch.from_numpy(records))
        self._attended, self._attended_spans = attended, spans
        self._table_meta = (len(spans), sum(n for _, _, n in spans), tile)
        # every block still attended must be resident for the fast path to stay valid
        self._dirty = any(m.block_id not in self._resident_rows for m in attended)
        self._seen_version = self.block_manager.version

    def _archived_current(self) -> None:
        self.residency_manager.drain_completed_prefetches(self)
        if self._dirty or self._seen_version != self.block_manager.version:
            self._refresh_archived()
            return
        # Every attended block is resident: the reference's walk reduces to
        # touching each block in page-table order (cache.py:387-390).
        now = time.time()
        for manifest in self._attended:
            manifest.last_accessed_at = now

    def _table_snapshot(self) -> tuple[torch.Tensor, int, int, int]:
        n, toks, tiles = self._table_meta
        return (self._table_dev, n, toks, tiles)

    def get_hot_attention_segments(self) -> PagedSegments:
        return PagedSegments(self, [], self._hot_pieces(), None, None)

    def get_archived_attention_segments(self) -> PagedSegments:
        self._archived_current()
        return PagedSegments(self, list(self._attended_spans), [], self._table_snapshot(), None)

    def get_attention_segments(self) -> PagedSegments:
        self._archived_current()
        return PagedSegments(
            self,
            list(self._attended_spans),
            self._hot_pieces(),
            self._table_snapshot(),
            (self.hot_head_index, self.hot_seq_len, self.hot_start),
        )

    def get_mixed_attention_segments(self, _unused: Any = None) -> PagedSegments:
        return self.get_attention_segments()

    def _concatenate_segments(self, segments: Sequence, *, require_contiguous: bool):
        if not len(segments):
            raise RuntimeError("No context available")
        ordered = sorted(list(segments), key=lambda s: s[2])
        if require_contiguous:
            for prev, cur in zip(ordered, ordered[1:]):
                prev_end = prev[2] + prev[0].shape[2]
                if cur[2] != prev_end:
                    raise RuntimeError(
                        f"Non-contiguous context: previous block end {prev_end}, next block start {cur[2]}"
                    )
        start = int(ordered[0][2])
        k = ordered[0][0] if len(ordered) == 1 else torch.cat([s[0] for s in ordered], dim=2)
        v = ordered[0][1] if len(ordered) == 1 else torch.cat([s[1] for s in ordered], dim=2)
        return k, v, start, start + k.shape[2]

    def materialize_exact_context(self):
        if self.hot_seq_len == 0:
            return self._empty_context()
        return self._materialize_hot_span(0, self.hot_seq_len)

    def materialize_archived_context(self, _unused: Any = None):
        return self._concatenate_segments(self.get_archived_attention_segments(), require_contiguous=True)

    def materialize_mixed_context(self, _unused: Any = None):
        return self._concatenate_segments(self.get_attention_segments(), require_contiguous=True)

    def get_total_length(self) -> int:
        archived = sum(
            m.token_count
            for m in self.block_manager.page_table.layer_entries(self.layer_id)
            if m.residency != BlockLocation.MISSING and m.materializable
        )
        return self.hot_seq_len + archived

    def get_block_stats(self) -> dict[str, Any]:
        stats = self.block_manager.get_residency_stats()
        stats["hot_tokens"] = self.hot_seq_len
        stats["hot_start"] = self.hot_start
        stats["hot_end"] = self.hot_end
        stats["residency_metrics"] = self.residency_manager.get_metrics()
        return stats

    # ------------------------------------------------------------------ attention
    def attend(self, q: torch.Tensor, q_start_pos: int, segments: Optional[PagedSegments] = None,
               *, want_lse: bool = False, max_splits: int = 0):
        """Exact attention of float32 q [B, H, Lq, D] against this layer's
        archived blocks and hot window (the work of layer.py:139-162)."""
        if segments is None:
            segments = self.get_attention_segments()
        return paged_attention(self, q, q_start_pos, segments, want_lse=want_lse, max_splits=max_splits)


def paged_attention(cache: LayerKVCache, q: torch.Tensor, q_start_pos: int, segments: PagedSegments,
                    *, want_lse: bool = False, max_splits: int = 0, workspace: Optional[native.Workspace] = None,
                    peers: Optional[Any] = None, step_state: Optional[torch.Tensor] = None,
                    out: Optional[torch.Tensor] = None):
    """Exact attention of q over a layer's page table + hot window.

    With ``peers`` (a ``sharded.PeerGroup``) the kernel also merges the
    results of every rank of the group over NVLink, so the returned output is
    the attention over the whole sharded context (an empty local shard is
    allowed then).

    With ``step_state`` (device int32[8], ``_native.STEP_*``) the query position
    and the hot window are read from device memory when the kernel runs, so a
    captured CUDA graph of the call stays valid while the ring advances (the
    page table is still captured by value).

    ``out`` (float32 [B, H, Lq, D], contiguous) receives the result instead of
    a new tensor: a tensor on the cache's device, or a pinned CPU tensor that
    the kernel writes across the bus (no separate copy back)."""
    if len(segments) == 0 and peers is None:
        raise RuntimeError("run_segmented_attention requires at least one KV segment")
    if q.dim() != 4 or q.shape[0] != cache.batch_size or q.shape[3] != cache.config.head_dim:
        raise ValueError(f"q must be [batch={cache.batch_size}, heads, q_len, head_dim={cache.config.head_dim}]")
    qf = _as(q, cache.device, torch.float32)
    B, H, Lq, D = (int(x) for x in qf.shape)
    if out is None:
        out = torch.empty((B, H, Lq, D), dtype=torch.float32, device=cache.device)
        out_ptr = out.data_ptr()
    else:
        if out.dtype != torch.float32 or tuple(out.shape) != (B, H, Lq, D) or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous float32 tensor of shape {(B, H, Lq, D)}")
        if out.device.type == "cpu":
            out_ptr = native.host_device_pointer(out)
        elif out.device == cache.device:
            out_ptr = out.data_ptr()
        else:
            raise ValueError(f"out must be on {cache.device} or pinned host memory")
    lse = torch.empty((B, H, Lq), dtype=torch.float32, device=cache.device) if want_lse else None
    if segments.table is not None:
        table_dev, n_blocks, toks, tiles = segments.table
    else:
        table_dev, n_blocks, toks, tiles = cache._table_dev, 0, 0, 0
    table = native.PageTableC(table_dev.data_ptr(), n_blocks, toks, tiles, 0)
    if segments.hot_state is not None:
        head, hlen, hstart = segments.hot_state
    else:
        head, hlen, hstart = 0, 0, 0
        if segments.n_archived != len(segments):
            # hot-only view taken without a snapshot: use the live ring state
            head, hlen, hstart = cache.hot_head_index, cache.hot_seq_len, cache.hot_start
    hot = native.HotWindowC(0, cache.config.hot_capacity, head, hlen, hstart, 0,
                            step_state.data_ptr() if step_state is not None else None)
    ws = workspace if workspace is not None else native.default_workspace(cache.device)
    nbytes = native.workspace_bytes(B, H, cache.num_kv_heads, Lq, D, max_splits)
    buf = ws.get(nbytes)
    if peers is not None:
        native.check(
            native.lib().rfsn_paged_attention_peer(
                cache.arena.handle, qf.data_ptr(), B, H, cache.num_kv_heads, Lq, int(q_start_pos),
                native.ctypes.byref(table), native.ctypes.byref(hot), peers.handle, out_ptr,
                lse.data_ptr() if lse is not None else None, buf.data_ptr(), buf.numel(), max_splits,
                native.stream_ptr(),
            ),
            "rfsn_paged_attention_peer",
        )
        return (out, lse) if want_lse else out
    native.check(
        native.lib().rfsn_paged_attention(
            cache.arena.handle, qf.data_ptr(), B, H, cache.num_kv_heads, Lq, int(q_start_pos),
            native.ctypes.byref(table), native.ctypes.byref(hot), out_ptr,
            lse.data_ptr() if lse is not None else None, buf.data_ptr(), buf.numel(), max_splits,
            native.stream_ptr(),
        ),
        "rfsn_paged_attention",
    )
    return (out, lse) if want_lse else out


class RFSNCache:
    """Per-layer caches of one session (cache.py:488-559)."""

    def __init__(
        self,
        config: RFSNConfig,
        batch_size: int,
        *,
        model_id: Optional[str] = None,
        session_id: Optional[str] = None,
        restore: bool = False,
        device: Optional[torch.device | str] = None,
        pool_tokens: Optional[int] = None,
        ops_factory: Optional[Any] = None,
        host_tier: bool = False,
        persist_async: bool = False,
    ) -> None:
        self.config = config
        self.model_id = model_id or derive_model_id(config)
        self.session_id = _resolve_session_id(config, session_id, restore=restore)
        self.layers = [
            LayerKVCache(
                config,
                batch_size=batch_size,
                num_heads=config.num_heads,
                num_kv_heads=config.num_kv_heads,
                layer_id=i,
                model_id=self.model_id,
                session_id=self.session_id,
                device=device,
                pool_tokens=pool_tokens,
                ops=ops_factory() if ops_factory is not None else None,
                host_tier=host_tier,
                persist_async=persist_async,
            )
            for i in range(config.num_layers)
        ]

    def flush_persistence(self) -> None:
        """Wait for every layer's write-behind npz and sidecar writes."""
        for layer_cache in self.layers:
            layer_cache.flush_persistence()

    @property
    def model_root(self) -> Path:
        return Path(self.config.disk_cache_dir) / self.model_id

    @property
    def session_root(self) -> Path:
        return self.model_root / self.session_id

    def layer(self, idx: int) -> LayerKVCache:
        return self.layers[idx]

    def reset(self, *, clear_persisted: bool = True) -> None:
        for layer_cache in self.layers:
            layer_cache.reset(clear_persisted=clear_persisted)

    def restore_from_disk(self) -> list[list[BlockManifest]]:
        if not self.session_id:
            raise ValueError(
                "restore_cache requires an explicit session_id so the persisted archive can be resolved safely"
            )
        missing = (
            f"Restore requested for session '{self.session_id}' but no persisted archive exists "
            f"for model '{self.model_id}'"
        )
        self.flush_persistence()  # writes staged by this object land before the archive is read
        if not self.model_root.exists():
            raise FileNotFoundError(missing)
        if not self.session_root.exists():
            known = sorted(p.name for p in self.model_root.iterdir() if p.is_dir())
            if known:
                raise FileNotFoundError(
                    f"Restore requested for unknown session '{self.session_id}' for model '{self.model_id}'. "
                    f"Available sessions: {', '.join(known)}"
                )
            raise FileNotFoundError(missing)
        restored = [layer_cache.restore_from_disk() for layer_cache in self.layers]
        if sum(len(x) for x in restored) == 0:
            raise FileNotFoundError(
                f"Restore requested for session '{self.session_id}' but the persisted archive is empty"
            )
        return restored
