"""Cold (disk) tier for archived blocks (drop-in for ``rfsn_v10_5.storage``).

On-disk format kept identical to the reference (storage.py:29-333) so either
implementation restores the other's sessions: per block a compressed ``.npz``
with arrays ``keys``/``values`` (bfloat16 stored as float32), a
``<payload>.manifest.json`` sidecar holding ``BlockManifest.to_dict()``, a
SHA-256 of the npz bytes in the manifest, atomic writes (temp file, fsync,
rename, directory fsync) and a ``quarantine/`` folder for bad payloads.
Failures while loading never raise: the block is marked MISSING /
unmaterializable and ``None`` is returned.
"""

from __future__ import annotations

import hashlib
import io
import json
import logging
import os
import tempfile
import time
import zipfile
from collections.abc import Mapping
from pathlib import Path
from typing import Any, Optional

import numpy as np

from .block_manager import BlockLocation, BlockManager, BlockManifest

LOGGER = logging.getLogger(__name__)


def _fsync_dir(path: Path) -> None:
    try:
        fd = os.open(path, os.O_RDONLY)
    except OSError:
        return
    try:
        os.fsync(fd)
    except OSError:
        pass
    finally:
        os.close(fd)


def _atomic_write(target: Path, data: bytes) -> None:
    target.parent.mkdir(parents=True, exist_ok=True)
    fd, tmp_name = tempfile.mkstemp(dir=target.parent, prefix=f".{target.name}.", suffix=".tmp")
    tmp = Path(tmp_name)
    try:
        with os.fdopen(fd, "wb") as handle:
            handle.write(data)
            handle.flush()
            os.fsync(handle.fileno())
        os.replace(tmp, target)
        _fsync_dir(target.parent)
    finally:
        if tmp.exists():
            tmp.unlink(missing_ok=True)


# Deflate level of the npz payloads. The layout is numpy's savez_compressed
# (one ``<name>.npy`` member per array, deflate, zip64), so np.load and the
# reference read these files unchanged; level 1 compresses a 2,048-token block
# about 7x faster than numpy's default level for a file about 10 % larger.
NPZ_DEFLATE_LEVEL = 1


def _npz_bytes(arrays: Mapping[str, np.ndarray]) -> bytes:
    buffer = io.BytesIO()
    with zipfile.ZipFile(buffer, mode="w", compression=zipfile.ZIP_DEFLATED,
                         compresslevel=NPZ_DEFLATE_LEVEL) as archive:
        for name, arr in arrays.items():
            with archive.open(f"{name}.npy", mode="w", force_zip64=True) as member:
                np.lib.format.write_array(member, np.asanyarray(arr), allow_pickle=False)
    return buffer.getvalue()


def _safe_fragment(value: str) -> str:
    return "".join(c if (c.isalnum() or c in "-_") else "_" for c in value)


class BlockStorage:
    """Persist, load, quarantine and rescan archived blocks."""

    def __init__(self, root_dir: str | Path) -> None:
        self.root_dir = Path(root_dir)
        self.quarantine_dir = self.root_dir / "quarantine"

    # -- paths --------------------------------------------------------------------------
    def _payload_path(self, manifest: BlockManifest) -> Optional[Path]:
        return None if manifest.payload_path is None else Path(manifest.payload_path)

    def _manifest_path(self, manifest: BlockManifest) -> Optional[Path]:
        return None if manifest.manifest_path is None else Path(manifest.manifest_path)

    def _paths(self, manifest: BlockManifest) -> tuple[Path, Path]:
        payload = self._payload_path(manifest)
        if payload is None:
            name = (
                f"{_safe_fragment(manifest.model_id)}.layer{manifest.layer_id}."
                f"{_safe_fragment(manifest.block_id.block_id)}.{manifest.payload_format}"
            )
            payload = self.root_dir / name
        sidecar = self._manifest_path(manifest) or self.root_dir / f"{payload.name}.manifest.json"
        return payload, sidecar

    # -- writing ------------------------------------------------------------------------
    def persist_block(self, manifest: BlockManifest, payload: Mapping[str, np.ndarray]) -> BlockManifest:
        arrays = self._normalize(payload, manifest)
        if manifest.payload_format != "npz":
            raise ValueError(f"Unsupported payload_format '{manifest.payload_format}'")
        blob = _npz_bytes(arrays)
        payload_path, sidecar = self._paths(manifest)
        manifest.payload_path = str(payload_path)
        manifest.manifest_path = str(sidecar)
        manifest.checksum = hashlib.sha256(blob).hexdigest()
        manifest.residency = BlockLocation.COLD_DISK
        manifest.materializable = True
        manifest.failure_reason = None
        manifest.touch()
        try:
            _atomic_write(payload_path, blob)
            self.write_manifest(manifest)
        except Exception:
            payload_path.unlink(missing_ok=True)
            sidecar.unlink(missing_ok=True)
            raise
        return manifest

    # -- write-behind (a cache that holds demoted blocks in pinned host memory) ----------
    def stage_persist(self, manifest: BlockManifest, dtype_name: str) -> None:
        """The in-memory effect of persist_block, without the bytes: payload and
        sidecar paths, dtype, COLD_DISK, materializable, the access stamp. The
        checksum stays empty until write_staged has hashed the payload."""
        if manifest.payload_format != "npz":
            raise ValueError(f"Unsupported payload_format '{manifest.payload_format}'")
        payload_path, sidecar = self._paths(manifest)
        manifest.payload_path = str(payload_path)
        manifest.manifest_path = str(sidecar)
        manifest.dtype = dtype_name
        manifest.checksum = ""
        manifest.residency = BlockLocation.COLD_DISK
        manifest.materializable = True
        manifest.failure_reason = None
        manifest.touch()

    def write_staged(self, manifest: BlockManifest, snapshot: dict[str, Any], payload: Mapping[str, np.ndarray]) -> str:
        """Writer side of stage_persist: the compressed payload, its SHA-256 (set
        on the manifest) and the sidecar as staged, with that checksum."""
        arrays = {name: np.asarray(arr) for name, arr in payload.items()}
        blob = _npz_bytes(arrays)
        checksum = hashlib.sha256(blob).hexdigest()
        _atomic_write(Path(snapshot["payload_path"]), blob)
        manifest.checksum = checksum
        self.write_snapshot(manifest, snapshot)
        return checksum

    def write_snapshot(self, manifest: BlockManifest, snapshot: dict[str, Any]) -> None:
        """Writer side of a sidecar update staged as ``manifest.to_dict()``; a
        checksum the snapshot lacks comes from the payload write staged before it."""
        if not snapshot.get("checksum") and manifest.checksum:
            snapshot = dict(snapshot, checksum=manifest.checksum)
        _atomic_write(Path(snapshot["manifest_path"]),
                      json.dumps(snapshot, indent=2, sort_keys=True).encode("utf-8"))

    def write_manifest(self, manifest: BlockManifest) -> BlockManifest:
        _, sidecar = self._paths(manifest)
        manifest.manifest_path = str(sidecar)
        _atomic_write(sidecar, json.dumps(manifest.to_dict(), indent=2, sort_keys=True).encode("utf-8"))
        return manifest

    def _normalize(self, payload: Mapping[str, np.ndarray], manifest: BlockManifest) -> dict[str, np.ndarray]:
        if not payload:
            raise ValueError("persist_block() requires a non-empty payload mapping")
        arrays = {name: np.asarray(arr) for name, arr in payload.items()}
        dtypes = {arr.dtype.name for arr in arrays.values()}
        if len(dtypes) != 1:
            raise ValueError("All payload arrays must share the same dtype")
        dtype_name = dtypes.pop()
        if manifest.dtype and manifest.dtype != dtype_name:
            raise ValueError(f"Manifest dtype '{manifest.dtype}' does not match payload dtype '{dtype_name}'")
        manifest.dtype = dtype_name
        shapes = manifest.shape_metadata or {name: tuple(arr.shape) for name, arr in arrays.items()}
        for name, arr in arrays.items():
            if name not in shapes:
                raise ValueError(f"Payload array '{name}' missing from shape_metadata")
            if tuple(shapes[name]) != tuple(int(d) for d in arr.shape):
                raise ValueError(f"Payload shape mismatch for '{name}': expected {shapes[name]} got {tuple(arr.shape)}")
        manifest.shape_metadata = {name: tuple(int(d) for d in shape) for name, shape in shapes.items()}
        return arrays

    # -- reading ------------------------------------------------------------------------
    def load_block(self, manifest: BlockManifest) -> Optional[dict[str, np.ndarray]]:
        path = self._payload_path(manifest)
        if path is None or not path.exists():
            LOGGER.warning("Block %s is missing payload file at %s; marking it missing", manifest.block_id, path)
            self._fail(manifest, "payload file missing")
            return None
        try:
            blob = path.read_bytes()
        except OSError as exc:
            LOGGER.warning("Failed to read block payload %s for %s: %s", path, manifest.block_id, exc)
            self._fail(manifest, f"payload read failed: {exc}")
            return None
        digest = hashlib.sha256(blob).hexdigest()
        if manifest.checksum and digest != manifest.checksum:
            LOGGER.warning(
                "Checksum mismatch for block %s at %s; expected %s got %s", manifest.block_id, path, manifest.checksum,
                digest,
            )
            self.quarantine_block(manifest)
            self._fail(manifest, "checksum mismatch")
            return None
        try:
            if manifest.payload_format != "npz":
                raise ValueError(f"Unsupported payload_format '{manifest.payload_format}'")
            with np.load(io.BytesIO(blob), allow_pickle=False) as npz:
                arrays = {name: np.asarray(npz[name]) for name in npz.files}
            self._validate(manifest, arrays)
        except Exception as exc:
            LOGGER.warning("Failed to deserialize block %s from %s: %s", manifest.block_id, path, exc)
            self.quarantine_block(manifest)
            self._fail(manifest, f"deserialization failed: {exc}")
            return None
        manifest.touch()
        self.write_manifest(manifest)
        return arrays

    def _validate(self, manifest: BlockManifest, arrays: Mapping[str, np.ndarray]) -> None:
        missing = set(manifest.shape_metadata) - set(arrays)
        if missing:
            raise ValueError(f"Missing arrays in payload: {sorted(missing)}")
        for name, shape in manifest.shape_metadata.items():
            arr = np.asarray(arrays[name])
            if tuple(int(d) for d in arr.shape) != tuple(shape):
                raise ValueError(f"Payload shape mismatch for '{name}': expected {shape} got {tuple(arr.shape)}")
            if arr.dtype.name != manifest.dtype:
                raise ValueError(f"Payload dtype mismatch for '{name}': expected {manifest.dtype} got {arr.dtype.name}")

    def _fail(self, manifest: BlockManifest, reason: str) -> None:
        manifest.residency = BlockLocation.MISSING
        manifest.materializable = False
        manifest.failure_reason = reason
        manifest.touch()
        if manifest.manifest_path is not None:
            self.write_manifest(manifest)

    # -- maintenance --------------------------------------------------------------------
    def delete_block(self, manifest: BlockManifest, *, remove_manifest: bool = False) -> None:
        path = self._payload_path(manifest)
        if path is not None:
            path.unlink(missing_ok=True)
        sidecar = self._manifest_path(manifest)
        if remove_manifest and sidecar is not None:
            sidecar.unlink(missing_ok=True)
            return
        self._fail(manifest, "payload deleted")

    def quarantine_block(self, manifest: BlockManifest) -> Optional[Path]:
        path = self._payload_path(manifest)
        if path is None or not path.exists():
            return None
        self.quarantine_dir.mkdir(parents=True, exist_ok=True)
        target = self.quarantine_dir / f"{path.name}.{int(time.time() * 1000)}.bad"
        path.replace(target)
        _fsync_dir(self.quarantine_dir)
        return target

    def scan_manifests(self, *, model_id: Optional[str] = None) -> list[BlockManifest]:
        found: list[BlockManifest] = []
        for sidecar in sorted(self.root_dir.glob("*.manifest.json")):
            try:
                manifest = BlockManifest.from_dict(json.loads(sidecar.read_text()))
            except Exception as exc:
                LOGGER.warning("Ignoring unreadable manifest %s: %s", sidecar, exc)
                continue
            manifest.manifest_path = str(sidecar)
            if model_id is not None and manifest.model_id != model_id:
                continue
            path = self._payload_path(manifest)
            if path is None or not path.exists():
                manifest.residency = BlockLocation.MISSING
                manifest.materializable = False
                manifest.failure_reason = manifest.failure_reason or "payload file missing"
                self.write_manifest(manifest)
            found.append(manifest)
        found.sort(key=lambda m: (m.layer_id, m.logical_start, m.logical_end))
        return found

    def rebuild_manager(self, manager: BlockManager) -> list[BlockManifest]:
        manifests = self.scan_manifests(model_id=manager.model_id)
        manager.rebuild_from_manifests(manifests)
        return manifests

