"""Host-side logic of the drop-in cache on CPU (no GPU): ring / seal / page
table / residency replayed against the reference's traces, plus the block
manager, storage and config contracts."""

import json
from pathlib import Path

import numpy as np
import pytest

from cache_replay import check_persisted_session, replay_residency, replay_ring, residency_names, ring_names
from fake_ops import FakeDeviceOps
from rfsn_b200 import (
    BlockId,
    BlockLocation,
    BlockManager,
    BlockManifest,
    BlockSpan,
    BlockStorage,
    PageTable,
    RFSNConfig,
    ResidencyManager,
)
from rfsn_b200.cache import _RowAllocator


@pytest.mark.parametrize("name", ring_names())
def test_ring_and_page_table_match_reference_trace(name):
    replay_ring(name, FakeDeviceOps)


@pytest.mark.parametrize("host_tier", [False, True])
@pytest.mark.parametrize("name", residency_names())
def test_residency_matches_reference_trace(name, host_tier):
    # the pinned host tier changes where a reloaded block's bytes come from,
    # never the warm/cold decisions, metrics or attended values
    replay_residency(name, FakeDeviceOps, host_tier=host_tier)


def test_device_page_table_records():
    cache = replay_ring("odd_hot10_bs3", FakeDeviceOps)
    segs = cache.get_attention_segments()
    table, n, toks, tiles = segs.table
    recs = table[: n + 1].numpy()
    blocks = cache.block_manager.iter_blocks(layer_id=0)
    assert n == len(blocks)
    tile = 0
    for rec, m in zip(recs[:n], blocks):
        assert (rec[1], rec[2], rec[3]) == (m.logical_start, m.token_count, tile)
        assert rec[0] == cache._resident_rows[m.block_id]
        tile += (m.token_count + 63) // 64
    assert recs[n][3] == tiles == tile
    assert toks == sum(m.token_count for m in blocks)


# --------------------------------------------------------------------------------- block manager
def _manifest(name, start, end, where, layer=0, materializable=True):
    return BlockManifest(
        block_id=BlockId("m", layer, name), span=BlockSpan(start, end), codec_version="v11-exact-kv",
        dtype="float32", shape_metadata={"keys": (1, 1, end - start, 2), "values": (1, 1, end - start, 2)},
        checksum=f"c-{name}", residency=where, materializable=materializable,
    )


def test_page_table_sorts_locates_and_counts():
    bm = BlockManager("m")
    for m in (
        _manifest("c", 8, 12, BlockLocation.COLD_DISK),
        _manifest("a", 0, 4, BlockLocation.HOT),
        _manifest("d", 12, 16, BlockLocation.MISSING, materializable=False),
        _manifest("b", 4, 8, BlockLocation.WARM_RAM),
    ):
        bm.register_block(m)
    assert [m.block_id.block_id for m in bm.locate_blocks_for_range(0, 2, 14)] == ["a", "b", "c", "d"]
    bm.mark_unmaterializable(layer_id=0, span=BlockSpan(8, 12), reason="bad")
    stats = bm.get_residency_stats()
    assert stats["total_blocks"] == 4 and stats["total_tokens"] == 16
    assert stats["by_location"]["warm_ram"]["blocks"] == 1
    assert stats["unmaterializable_blocks"] == 2
    with pytest.raises(ValueError, match="overlaps"):
        bm.register_block(_manifest("e", 3, 6, BlockLocation.COLD_DISK))
    with pytest.raises(ValueError, match="already registered"):
        bm.register_block(_manifest("a", 40, 44, BlockLocation.HOT))
    with pytest.raises(KeyError, match="Unknown block_id"):
        bm.get_block(BlockId("m", 0, "zz"))
    with pytest.raises(ValueError, match="mark_missing"):
        bm.promote_block(BlockId("m", 0, "a"), BlockLocation.MISSING)


def test_metadata_json_round_trip():
    bm = BlockManager("m")
    bm.register_block(_manifest("x", 0, 4, BlockLocation.WARM_RAM))
    bm.register_block(_manifest("y", 0, 8, BlockLocation.COLD_DISK, layer=1))
    blob = json.loads(json.dumps(bm.serialize_metadata()))
    back = BlockManager.deserialize_metadata(blob)
    assert [m.to_dict() for m in back.iter_blocks()] == [m.to_dict() for m in bm.iter_blocks()]
    table = PageTable.from_dict(blob["page_table"])
    assert table.locate(1, 0, 8)[0].checksum == "c-y"
    keys = set(bm.iter_blocks()[0].to_dict())
    assert {"model_id", "layer_id", "block_id", "logical_start", "logical_end", "token_count", "codec_version",
            "dtype", "shape_metadata", "checksum", "residency", "created_at", "last_accessed_at", "pin_count",
            "ref_count", "payload_format", "payload_path", "manifest_path", "materializable",
            "failure_reason"} == keys


def test_lru_victim_uses_access_time_then_position():
    rm = ResidencyManager()
    ms = [_manifest(n, s, s + 4, BlockLocation.WARM_RAM) for n, s in (("a", 0), ("b", 4), ("c", 8))]
    for m, t in zip(ms, (5.0, 1.0, 1.0)):
        m.touch(timestamp=t)
    assert rm.choose_warm_eviction_victim(ms).block_id.block_id == "b"
    assert rm.choose_warm_eviction_victim(ms, protected_block_id=ms[1].block_id).block_id.block_id == "c"
    ms[2].pin_count = 1
    assert rm.choose_warm_eviction_victim(ms, protected_block_id=ms[1].block_id).block_id.block_id == "a"


# --------------------------------------------------------------------------------- storage
def _payload(n):
    keys = np.arange(n * 2, dtype=np.float32).reshape(1, 1, n, 2)
    return {"keys": keys, "values": keys + 100}


def test_storage_round_trip_and_rescan(tmp_path):
    st = BlockStorage(tmp_path)
    m = _manifest("blk", 0, 4, BlockLocation.WARM_RAM)
    st.persist_block(m, _payload(4))
    assert m.residency == BlockLocation.COLD_DISK and len(m.checksum) == 64
    assert Path(m.payload_path).name == "m.layer0.blk.npz"
    bm = BlockManager("m")
    scanned = st.rebuild_manager(bm)
    assert [x.checksum for x in scanned] == [m.checksum]
    loaded = st.load_block(scanned[0])
    np.testing.assert_array_equal(loaded["values"], _payload(4)["values"])


@pytest.mark.parametrize("damage,reason", [
    ("delete", "missing"),
    ("tamper", "checksum mismatch"),
])
def test_storage_failures_mark_missing_without_raising(tmp_path, damage, reason):
    st = BlockStorage(tmp_path)
    m = _manifest("blk", 0, 4, BlockLocation.WARM_RAM)
    st.persist_block(m, _payload(4))
    p = Path(m.payload_path)
    if damage == "delete":
        p.unlink()
    else:
        p.write_bytes(b"not an npz")
    assert st.load_block(m) is None
    assert m.residency == BlockLocation.MISSING and not m.materializable
    assert reason in m.failure_reason
    if damage == "tamper":
        assert any(st.quarantine_dir.iterdir())


def test_storage_rejects_bad_payloads(tmp_path):
    st = BlockStorage(tmp_path)
    m = _manifest("blk", 0, 4, BlockLocation.WARM_RAM)
    with pytest.raises(ValueError, match="same dtype"):
        st.persist_block(m, {"keys": np.zeros((1, 1, 4, 2), np.float32), "values": np.zeros((1, 1, 4, 2), np.float16)})
    with pytest.raises(ValueError, match="shape mismatch"):
        st.persist_block(m, _payload(3))


# --------------------------------------------------------------------------------- config
@pytest.mark.parametrize("kwargs,message", [
    (dict(hidden_dim=30), "must equal num_heads"),
    (dict(num_kv_heads=3), "divisible"),
    (dict(hot_capacity=4096), "hot_capacity <= warm_capacity"),
    (dict(block_size_seq=0), "block_size_seq"),
    (dict(model_dtype="int8"), "model_dtype"),
    (dict(session_id="bad id!"), "session_id"),
])
def test_config_validation_matches_reference(kwargs, message):
    base = dict(hidden_dim=32, num_heads=2, head_dim=16)
    base.update(kwargs)
    with pytest.raises(ValueError, match=message):
        RFSNConfig(**base)


def test_config_defaults():
    cfg = RFSNConfig()
    assert cfg.num_kv_heads == cfg.num_heads and cfg.ffn_dim == 4 * cfg.hidden_dim and cfg.kv_groups == 1


def test_row_allocator_first_fit_and_coalescing():
    a = _RowAllocator(10, 30)
    r1, r2, r3 = a.allocate(5), a.allocate(5), a.allocate(5)
    assert (r1, r2, r3) == (10, 15, 20)
    a.release(15, 5)
    a.release(10, 5)
    assert a.free[0] == [10, 20]
    assert a.allocate(12) is None
    a.release(20, 5)
    assert a.free == [[10, 30]]
    a.grow(40)
    assert a.allocate(30) == 10


@pytest.mark.parametrize("seed", range(12))
def test_random_append_sequences_match_ring_oracle(seed):
    """Random chunk sequences (decode steps, ragged chunks, whole-ring chunks,
    oversized chunks that must fail) through the drop-in cache and the ring
    oracle: ring state, sealed block spans, segment order and every key/value
    row agree after each step, bit for bit."""
    import tempfile

    import torch

    from cache_replay import _config, _kv
    from oracle.kv_ring import RingOracle
    from rfsn_b200 import LayerKVCache

    rng = np.random.default_rng(seed)
    cap = int(rng.integers(2, 48))
    bs = int(rng.integers(1, cap + 8))
    with tempfile.TemporaryDirectory() as tmp:
        cache = LayerKVCache(_config(cap, bs, "archived", 1 << 20, tmp), 1, 2, 1, layer_id=0, session_id="rand",
                             ops=FakeDeviceOps())
        ring = RingOracle(cap, bs)
        pos = 0
        for _ in range(40):
            kind = rng.random()
            n = 1 if kind < 0.4 else (cap if kind < 0.5 else (cap + 1 if kind < 0.55 else int(rng.integers(1, cap + 1))))
            if n > cap:
                with pytest.raises(RuntimeError) as err:
                    cache.evict_for_append(n)
                with pytest.raises(RuntimeError) as want:
                    ring.evict_for_append(n)
                assert str(err.value) == str(want.value)
                continue
            cache.evict_for_append(n)
            ring.evict_for_append(n)
            k, v = _kv(pos, n, cache.device)
            cache.append_exact(k, v)
            ring.append(n)
            pos += n
            assert (cache.hot_head_index, cache.hot_seq_len, cache.hot_start, cache.hot_write_index, cache.hot_end) == (
                ring.head, ring.length, ring.start, ring.write_index, ring.end)
            spans = [(m.logical_start, m.logical_end) for m in cache.block_manager.iter_blocks(layer_id=0)]
            assert spans == ring.sealed
            segs = cache.get_attention_segments()
            want_segs = [(s, e - s) for s, e in ring.sealed] + [(s, n_) for _p, n_, s in ring.hot_spans()]
            assert [(int(s[2]), int(s[0].shape[2])) for s in segs] == want_segs
            assert cache.get_total_length() == pos
            for kk, vv, start in segs:
                expect = torch.arange(start, start + kk.shape[2], dtype=torch.float32)
                assert torch.equal(kk[0, 0, :, 0].float().cpu(), expect)
                assert torch.equal(vv[0, 0, :, 0].float().cpu(), expect + 0.5)


@pytest.mark.parametrize("name", residency_names())
def test_write_behind_persistence_keeps_reference_decisions(name):
    # npz writes on the layer's writer thread: residency decisions, metrics and
    # attended values equal the reference trace, and the files written after a
    # flush restore the session
    replay_residency(name, FakeDeviceOps, host_tier=True, persist_async=True,
                     at_end=check_persisted_session(FakeDeviceOps))


def test_write_behind_needs_the_host_tier(tmp_path):
    from cache_replay import _config
    from rfsn_b200 import LayerKVCache

    with pytest.raises(ValueError, match="host_tier"):
        LayerKVCache(_config(8, 4, "archived", 8, str(tmp_path)), 1, 2, 1, session_id="s", ops=FakeDeviceOps(),
                     persist_async=True)


def test_write_behind_reset_drops_pending_writes_and_reports_failures(tmp_path, monkeypatch):
    import threading

    import torch

    from cache_replay import _config, _kv
    from rfsn_b200 import LayerKVCache

    cfg = _config(4, 4, "archived", 4, str(tmp_path))
    cache = LayerKVCache(cfg, 1, 2, 1, session_id="s", ops=FakeDeviceOps(), host_tier=True, persist_async=True)
    gate = threading.Event()
    real = cache.storage.write_staged

    def slow(*a, **kw):
        gate.wait(timeout=10)
        return real(*a, **kw)

    monkeypatch.setattr(cache.storage, "write_staged", slow)
    pos = 0
    for _ in range(6):  # hot 4, blocks of 4, warm 4 tokens: every append seals, older blocks go cold
        cache.evict_for_append(4)
        k, v = _kv(pos, 4, torch.device("cpu"))
        cache.append_exact(k, v)
        pos += 4
    assert cache._write_jobs and not any(j.done() for j in cache._write_jobs)
    gate.set()
    cache.reset(clear_persisted=True)
    assert cache._write_jobs == [] and not list(cache.storage.root_dir.glob("*.npz"))

    def broken(*a, **kw):
        raise OSError("disk full")

    monkeypatch.setattr(cache.storage, "write_staged", broken)
    for _ in range(4):
        cache.evict_for_append(4)
        k, v = _kv(pos, 4, torch.device("cpu"))
        cache.append_exact(k, v)
        pos += 4
    with pytest.raises(RuntimeError, match="disk full"):
        cache.flush_persistence()


def test_write_behind_coalesces_sidecar_rewrites(tmp_path, monkeypatch):
    """Thrashing blocks between warm and cold queues at most one sidecar write
    per block while the writer is busy; after a flush each cold block's sidecar
    is its current manifest, as a synchronous write would have left it."""
    import threading

    import torch

    from cache_replay import _config, _kv
    from rfsn_b200 import LayerKVCache

    cfg = _config(4, 4, "archived", 8, str(tmp_path))
    cache = LayerKVCache(cfg, 1, 2, 1, session_id="s", ops=FakeDeviceOps(), host_tier=True, persist_async=True)
    pos = 0
    for _ in range(6):  # 5 sealed blocks of 4 tokens, 2 of them warm
        cache.evict_for_append(4)
        k, v = _kv(pos, 4, torch.device("cpu"))
        cache.append_exact(k, v)
        pos += 4
    cache.flush_persistence()
    gate = threading.Event()
    real = cache.storage.write_snapshot

    def held(*a, **kw):
        gate.wait(timeout=10)
        return real(*a, **kw)

    monkeypatch.setattr(cache.storage, "write_snapshot", held)
    blocks = list(cache.block_manager.iter_blocks(layer_id=0))
    for _ in range(20):  # every call reloads the cold blocks and demotes others (the reference's thrash)
        cache.get_attention_segments()
    evictions = cache.residency_manager.get_metrics()["warm_evictions"]
    # at most: the running write, one first-time payload write and one queued sidecar per block
    assert len(cache._write_jobs) <= 2 * len(blocks) + 1 < evictions
    gate.set()
    cache.flush_persistence()
    for m in cache.block_manager.iter_blocks(layer_id=0):
        if m.residency == BlockLocation.COLD_DISK:
            assert json.loads(Path(m.manifest_path).read_text()) == m.to_dict()


def test_npz_payload_layout_matches_numpy_savez():
    """Payloads are numpy's npz layout at a faster deflate level: the same
    member names and arrays as np.savez_compressed, read back by np.load."""
    import io
    import zipfile

    from rfsn_b200.storage import NPZ_DEFLATE_LEVEL, _npz_bytes

    arrays = {"keys": np.arange(2 * 3 * 5 * 4, dtype=np.float32).reshape(2, 3, 5, 4),
              "values": -np.ones((2, 3, 5, 4), np.float16)}
    ours = _npz_bytes(arrays)
    ref = io.BytesIO()
    np.savez_compressed(ref, **arrays)
    names = lambda blob: sorted(i.filename for i in zipfile.ZipFile(io.BytesIO(blob)).infolist())  # noqa: E731
    assert names(ours) == names(ref.getvalue()) == ["keys.npy", "values.npy"]
    assert all(i.compress_type == zipfile.ZIP_DEFLATED for i in zipfile.ZipFile(io.BytesIO(ours)).infolist())
    assert NPZ_DEFLATE_LEVEL == 1
    loaded = np.load(io.BytesIO(ours))
    for k, v in arrays.items():
        assert loaded[k].dtype == v.dtype and np.array_equal(loaded[k], v)


def test_session_restore_errors_and_round_trip_match_reference(tmp_path):
    """cache.py:488-559: restoring needs an explicit session id, a missing
    archive and an unknown session raise FileNotFoundError (the latter listing
    the sessions that exist), and a persisted session restores its page table."""
    import dataclasses

    import torch

    from cache_replay import _config, _kv
    from rfsn_b200 import RFSNCache

    base = _config(4, 4, "archived", 4, str(tmp_path))
    alpha, beta = dataclasses.replace(base, session_id="alpha"), dataclasses.replace(base, session_id="beta")
    with pytest.raises(ValueError, match="explicit session_id"):
        RFSNCache(base, 1, restore=True, ops_factory=FakeDeviceOps)
    with pytest.raises(FileNotFoundError, match="no persisted archive exists"):
        RFSNCache(alpha, 1, restore=True, ops_factory=FakeDeviceOps).restore_from_disk()

    kv = RFSNCache(alpha, 1, ops_factory=FakeDeviceOps)
    layer = kv.layer(0)
    pos = 0
    for _ in range(5):  # blocks of 4 beyond a warm capacity of 4 tokens go to disk
        layer.evict_for_append(4)
        k, v = _kv(pos, 4, torch.device("cpu"))
        layer.append_exact(k, v)
        pos += 4
    # restore rebuilds the persisted (cold) blocks; a block still warm was never written
    spans = [(m.logical_start, m.logical_end) for m in layer.block_manager.iter_blocks(layer_id=0)
             if m.residency == BlockLocation.COLD_DISK]
    assert len(spans) >= 2

    with pytest.raises(FileNotFoundError, match="unknown session 'beta'.*Available sessions: alpha"):
        RFSNCache(beta, 1, restore=True, ops_factory=FakeDeviceOps).restore_from_disk()
    restored = RFSNCache(alpha, 1, restore=True, ops_factory=FakeDeviceOps)
    (manifests,) = restored.restore_from_disk()
    assert [(m.logical_start, m.logical_end) for m in manifests] == spans
    assert restored.layer(0).hot_start == spans[-1][1]


@pytest.mark.parametrize("head_dim,base", [(64, 10000.0), (128, 500000.0), (128, 1e6)])
def test_rope_frequency_table_matches_oracle_on_host(tmp_path, head_dim, base):
    # layer.py:29 in float32; the table the fused RoPE kernel reads
    import dataclasses

    from cache_replay import _config
    from oracle.rope import inv_freq
    from rfsn_b200 import LayerKVCache

    cfg = dataclasses.replace(_config(8, 4, "archived", 8, str(tmp_path)), head_dim=head_dim, rope_base=base,
                              hidden_dim=2 * head_dim)
    c = LayerKVCache(cfg, 1, 2, 1, session_id="r", ops=FakeDeviceOps())
    table = c.inv_freq().numpy()
    assert table.dtype == np.float32 and np.array_equal(table, inv_freq(head_dim, base))


def test_rope_tables_are_checked_before_any_device_work(tmp_path):
    """``append_rope_tables`` (a layer called with ``rope_tables``) rejects
    tables that are not a (cos, sin) pair of float tensors of one row per new
    position, with ValueError as the reference's shape errors, before the ring
    or the device is touched."""
    import torch

    from cache_replay import _config
    from rfsn_b200.cache import LayerKVCache

    cache = LayerKVCache(_config(8, 4, "archived", 64, str(tmp_path)), 1, 2, 1, session_id="s", ops=FakeDeviceOps(),
                         device="cpu")
    q = torch.zeros((1, 2, 3, 4))
    k = v = torch.zeros((1, 1, 3, 4))
    good = torch.zeros((3, 4))
    for tables, msg in (((good,), "pair"), ((good, "x"), "pair"), ((good.int(), good.int()), "float dtype"),
                        ((good, good.half()), "float dtype"), ((torch.zeros((2, 4)), torch.zeros((2, 4))), "[3, 4]"),
                        ((torch.zeros((3, 8)), torch.zeros((3, 8))), "[3, 4]")):
        with pytest.raises(ValueError, match=msg.replace("[", r"\[").replace("]", r"\]")):
            cache.append_rope_tables(q, k, v, 0, tables)
    assert cache.hot_seq_len == 0 and not cache._ops.calls
