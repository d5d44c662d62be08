"""Archived-block metadata and the host page table (drop-in for
``rfsn_v10_5.block_manager``).

The records, their JSON form (``to_dict`` keys), the ordering and overlap
rules of the page table and the error messages are kept identical to the
reference (block_manager.py:18-411) because sessions persisted by one must
restore in the other and page tables are compared bit-exactly. The device
copy that the attention kernels walk is built from this host table by
``cache.LayerKVCache`` (int32 records {row, pos, len, tile_begin}).
"""

from __future__ import annotations

import bisect
import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Iterable, Iterator, Optional


class BlockLocation(str, Enum):
    """block_manager.py:18-24."""

    HOT = "hot"
    WARM_RAM = "warm_ram"
    COLD_DISK = "cold_disk"
    MISSING = "missing"


@dataclass(frozen=True, order=True)
class BlockId:
    """block_manager.py:27-56."""

    model_id: str
    layer_id: int
    block_id: str

    def __post_init__(self) -> None:
        for ok, message in (
            (bool(self.model_id), "BlockId.model_id must be non-empty"),
            (self.layer_id >= 0, "BlockId.layer_id must be >= 0"),
            (bool(self.block_id), "BlockId.block_id must be non-empty"),
        ):
            if not ok:
                raise ValueError(message)

    def to_dict(self) -> dict[str, Any]:
        return {"model_id": self.model_id, "layer_id": self.layer_id, "block_id": self.block_id}

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "BlockId":
        return cls(str(payload["model_id"]), int(payload["layer_id"]), str(payload["block_id"]))


@dataclass(frozen=True, order=True)
class BlockSpan:
    """Half-open logical token range [logical_start, logical_end) (block_manager.py:59-91)."""

    logical_start: int
    logical_end: int

    def __post_init__(self) -> None:
        if self.logical_start < 0:
            raise ValueError("BlockSpan.logical_start must be >= 0")
        if self.logical_end <= self.logical_start:
            raise ValueError("BlockSpan.logical_end must be greater than logical_start")

    @property
    def token_count(self) -> int:
        return self.logical_end - self.logical_start

    def overlaps(self, start: int, end: int) -> bool:
        return start < self.logical_end and self.logical_start < end

    def to_dict(self) -> dict[str, int]:
        return {"logical_start": self.logical_start, "logical_end": self.logical_end, "token_count": self.token_count}

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "BlockSpan":
        return cls(int(payload["logical_start"]), int(payload["logical_end"]))


@dataclass
class BlockManifest:
    """Metadata of one archived block (block_manager.py:94-200)."""

    block_id: BlockId
    span: BlockSpan
    codec_version: str
    dtype: str
    shape_metadata: dict[str, tuple[int, ...]]
    checksum: str = ""
    residency: BlockLocation = BlockLocation.HOT
    created_at: float = field(default_factory=time.time)
    last_accessed_at: float = field(default_factory=time.time)
    pin_count: int = 0
    ref_count: int = 0
    payload_format: str = "npz"
    payload_path: Optional[str] = None
    manifest_path: Optional[str] = None
    materializable: bool = True
    failure_reason: Optional[str] = None

    def __post_init__(self) -> None:
        for ok, message in (
            (bool(self.codec_version), "BlockManifest.codec_version must be non-empty"),
            (bool(self.dtype), "BlockManifest.dtype must be non-empty"),
            (self.pin_count >= 0, "BlockManifest.pin_count must be >= 0"),
            (self.ref_count >= 0, "BlockManifest.ref_count must be >= 0"),
            (self.payload_format in ("npz", "safetensors"), "payload_format must be 'npz' or 'safetensors'"),
        ):
            if not ok:
                raise ValueError(message)
        self.shape_metadata = {str(k): tuple(int(d) for d in v) for k, v in self.shape_metadata.items()}

    model_id = property(lambda self: self.block_id.model_id)
    layer_id = property(lambda self: self.block_id.layer_id)
    logical_start = property(lambda self: self.span.logical_start)
    logical_end = property(lambda self: self.span.logical_end)
    token_count = property(lambda self: self.span.token_count)

    def touch(self, *, timestamp: Optional[float] = None) -> None:
        self.last_accessed_at = time.time() if timestamp is None else float(timestamp)

    def to_dict(self) -> dict[str, Any]:
        out: dict[str, Any] = {}
        out.update(self.block_id.to_dict())
        out.update(self.span.to_dict())
        out["codec_version"] = self.codec_version
        out["dtype"] = self.dtype
        out["shape_metadata"] = {k: list(v) for k, v in sorted(self.shape_metadata.items())}
        out["checksum"] = self.checksum
        out["residency"] = self.residency.value
        for key in (
            "created_at", "last_accessed_at", "pin_count", "ref_count", "payload_format", "payload_path",
            "manifest_path", "materializable", "failure_reason",
        ):
            out[key] = getattr(self, key)
        return out

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "BlockManifest":
        now = time.time()
        return cls(
            block_id=BlockId.from_dict(payload),
            span=BlockSpan.from_dict(payload),
            codec_version=str(payload["codec_version"]),
            dtype=str(payload["dtype"]),
            shape_metadata={str(k): tuple(int(d) for d in v) for k, v in dict(payload.get("shape_metadata", {})).items()},
            checksum=str(payload.get("checksum", "")),
            residency=BlockLocation(str(payload.get("residency", BlockLocation.HOT.value))),
            created_at=float(payload.get("created_at", now)),
            last_accessed_at=float(payload.get("last_accessed_at", now)),
            pin_count=int(payload.get("pin_count", 0)),
            ref_count=int(payload.get("ref_count", 0)),
            payload_format=str(payload.get("payload_format", "npz")),
            payload_path=payload.get("payload_path"),
            manifest_path=payload.get("manifest_path"),
            materializable=bool(payload.get("materializable", True)),
            failure_reason=payload.get("failure_reason"),
        )


@dataclass
class PageTable:
    """Per-layer list of manifests sorted by logical_start, no overlaps
    (block_manager.py:203-275)."""

    _entries_by_layer: dict[int, list[BlockManifest]] = field(default_factory=dict)

    def register(self, manifest: BlockManifest) -> None:
        entries = self._entries_by_layer.setdefault(manifest.layer_id, [])
        at = bisect.bisect_left([e.logical_start for e in entries], manifest.logical_start)
        if at > 0 and entries[at - 1].logical_end > manifest.logical_start:
            raise ValueError(f"Block span overlaps previous page-table entry: {entries[at - 1].span} vs {manifest.span}")
        if at < len(entries) and manifest.logical_end > entries[at].logical_start:
            raise ValueError(f"Block span overlaps next page-table entry: {manifest.span} vs {entries[at].span}")
        entries.insert(at, manifest)

    def remove(self, block_id: BlockId) -> None:
        entries = self._entries_by_layer.get(block_id.layer_id, [])
        for i, manifest in enumerate(entries):
            if manifest.block_id == block_id:
                entries.pop(i)
                if not entries:
                    del self._entries_by_layer[block_id.layer_id]
                return
        raise KeyError(f"Unknown block_id: {block_id}")

    def locate(self, layer_id: int, start: int, end: int) -> list[BlockManifest]:
        if start < 0 or end <= start:
            raise ValueError("locate() requires 0 <= start < end")
        return [m for m in self._entries_by_layer.get(layer_id, []) if m.span.overlaps(start, end)]

    def iter_manifests(self, *, layer_id: Optional[int] = None) -> Iterator[BlockManifest]:
        if layer_id is not None:
            yield from list(self._entries_by_layer.get(layer_id, []))
            return
        for lid in sorted(self._entries_by_layer):
            yield from self._entries_by_layer[lid]

    def layer_entries(self, layer_id: int) -> list[BlockManifest]:
        """The live (not copied) sorted list of one layer; callers must not mutate it."""
        return self._entries_by_layer.get(layer_id, [])

    def clear(self) -> None:
        self._entries_by_layer.clear()

    def to_dict(self) -> dict[str, Any]:
        return {
            "layers": {
                str(lid): [m.to_dict() for m in entries] for lid, entries in sorted(self._entries_by_layer.items())
            }
        }

    @classmethod
    def from_dict(cls, payload: dict[str, Any]) -> "PageTable":
        table = cls()
        for entries in dict(payload.get("layers", {})).values():
            for entry in entries:
                table.register(BlockManifest.from_dict(entry))
        return table


class BlockManager:
    """Single authority for archived-block metadata (block_manager.py:278-411)."""

    def __init__(self, model_id: str) -> None:
        if not model_id:
            raise ValueError("BlockManager.model_id must be non-empty")
        self.model_id = model_id
        self.page_table = PageTable()
        self._blocks: dict[BlockId, BlockManifest] = {}
        self.version = 0  # bumped on every structural or residency change

    def clear(self) -> None:
        self.page_table.clear()
        self._blocks.clear()
        self.version += 1

    def register_block(self, manifest: BlockManifest) -> BlockManifest:
        if manifest.model_id != self.model_id:
            raise ValueError(
                f"Manifest model_id '{manifest.model_id}' does not match manager model_id '{self.model_id}'"
            )
        if manifest.block_id in self._blocks:
            raise ValueError(f"Block {manifest.block_id} is already registered")
        self.page_table.register(manifest)
        self._blocks[manifest.block_id] = manifest
        self.version += 1
        return manifest

    def get_block(self, block_id: BlockId) -> BlockManifest:
        manifest = self._blocks.get(block_id)
        if manifest is None:
            raise KeyError(f"Unknown block_id: {block_id}")
        return manifest

    def iter_blocks(self, *, layer_id: Optional[int] = None) -> list[BlockManifest]:
        return list(self.page_table.iter_manifests(layer_id=layer_id))

    def locate_blocks_for_range(self, layer_id: int, start: int, end: int) -> list[BlockManifest]:
        return self.page_table.locate(layer_id, start, end)

    def _move(self, block_id: BlockId, target: BlockLocation) -> BlockManifest:
        if target == BlockLocation.MISSING:
            raise ValueError("Use mark_missing() for MISSING state transitions")
        manifest = self.get_block(block_id)
        manifest.residency = target
        manifest.touch()
        self.version += 1
        return manifest

    def promote_block(self, block_id: BlockId, target_location: BlockLocation) -> BlockManifest:
        return self._move(block_id, target_location)

    def demote_block(self, block_id: BlockId, target_location: BlockLocation) -> BlockManifest:
        return self._move(block_id, target_location)

    def mark_missing(self, block_id: BlockId, *, reason: Optional[str] = None) -> BlockManifest:
        manifest = self.get_block(block_id)
        manifest.residency = BlockLocation.MISSING
        if reason is not None:
            manifest.failure_reason = reason
        manifest.touch()
        self.version += 1
        return manifest

    def mark_unmaterializable(
        self,
        block_id: Optional[BlockId] = None,
        *,
        layer_id: Optional[int] = None,
        span: Optional[BlockSpan] = None,
        reason: Optional[str] = None,
    ) -> list[BlockManifest]:
        if block_id is not None:
            targets = [self.get_block(block_id)]
        else:
            if layer_id is None or span is None:
                raise ValueError("mark_unmaterializable() requires either block_id or layer_id+span")
            targets = self.locate_blocks_for_range(layer_id, span.logical_start, span.logical_end)
            if not targets:
                raise KeyError(
                    f"No blocks registered for layer {layer_id} in span {span.logical_start}:{span.logical_end}"
                )
        for manifest in targets:
            manifest.materializable = False
            if reason is not None:
                manifest.failure_reason = reason
            manifest.touch()
        self.version += 1
        return targets

    def get_residency_stats(self) -> dict[str, Any]:
        by_location = {loc.value: {"blocks": 0, "tokens": 0} for loc in BlockLocation}
        total_tokens = 0
        unmaterializable = 0
        for manifest in self.page_table.iter_manifests():
            bucket = by_location[manifest.residency.value]
            bucket["blocks"] += 1
            bucket["tokens"] += manifest.token_count
            total_tokens += manifest.token_count
            unmaterializable += 0 if manifest.materializable else 1
        return {
            "total_blocks": len(self._blocks),
            "total_tokens": total_tokens,
            "unmaterializable_blocks": unmaterializable,
            "by_location": by_location,
        }

    def serialize_metadata(self) -> dict[str, Any]:
        return {
            "model_id": self.model_id,
            "page_table": self.page_table.to_dict(),
            "blocks": [m.to_dict() for m in self.iter_blocks()],
        }

    @classmethod
    def deserialize_metadata(cls, payload: dict[str, Any]) -> "BlockManager":
        manager = cls(model_id=str(payload["model_id"]))
        manager.rebuild_from_manifests(BlockManifest.from_dict(d) for d in payload.get("blocks", []))
        return manager

    def rebuild_from_manifests(self, manifests: Iterable[BlockManifest]) -> None:
        self.clear()
        for manifest in sorted(manifests, key=lambda m: (m.layer_id, m.logical_start, m.logical_end)):
            self.register_block(manifest)
