"""Replays of the reference's ring and residency traces on LayerKVCache.

Shared by the CPU tests (with the FakeDeviceOps double) and the GPU tests
(with the real device ops). K rows carry their absolute position so segment
contents can be checked too.
"""

from __future__ import annotations

import tempfile

import pytest
import torch

from _util import load_json

RING = load_json("ring_traces.json")
RESIDENCY = load_json("residency_trace.json")


def _config(cap, bs, mode, warm, tmp):
    from rfsn_b200 import RFSNConfig, RuntimeMode

    return RFSNConfig(
        hidden_dim=8, num_heads=2, num_kv_heads=1, head_dim=4, num_layers=1, vocab_size=16, hot_capacity=cap,
        warm_capacity=warm, cold_capacity=max(warm, 1 << 21), block_size_seq=bs, runtime_mode=RuntimeMode(mode),
        model_dtype="float32", disk_cache_dir=tmp,
    )


def _kv(pos, n, device):
    """K rows carry their absolute position, V rows position + 0.5 (as in the traces)."""
    k = torch.arange(pos, pos + n, dtype=torch.float32)[None, None, :, None].expand(1, 1, n, 4).contiguous()
    return k.to(device), (k + 0.5).to(device)


def replay_ring(name, ops_factory):
    from rfsn_b200 import LayerKVCache

    sc = RING[name]
    with tempfile.TemporaryDirectory() as tmp:
        cfg = _config(sc["hot_capacity"], sc["block_size"], sc["mode"], max(sc["hot_capacity"], 1 << 20), tmp)
        cache = LayerKVCache(cfg, 1, 2, 1, layer_id=0, session_id="golden", ops=ops_factory())
        pos = 0
        for step in sc["steps"]:
            n = step["incoming"]
            if "error" in step:
                with pytest.raises(RuntimeError) as err:
                    cache.evict_for_append(n)
                    k, v = _kv(pos, n, cache.device)
                    cache.append_exact(k, v)
                assert str(err.value) == step["error"]
                continue
            cache.evict_for_append(n)
            k, v = _kv(pos, n, cache.device)
            cache.append_exact(k, v)
            pos += n
            got = (cache.hot_head_index, cache.hot_seq_len, cache.hot_start, cache.hot_write_index, cache.hot_end)
            want = tuple(step[key] for key in ("hot_head_index", "hot_seq_len", "hot_start", "hot_write_index", "hot_end"))
            assert got == want
            blocks = [
                {"block_id": m.block_id.block_id, "start": m.logical_start, "end": m.logical_end,
                 "residency": m.residency.value, "materializable": m.materializable,
                 "shape": list(m.shape_metadata["keys"])}
                for m in cache.block_manager.iter_blocks(layer_id=0)
            ]
            assert blocks == step["blocks"]
            segs = cache.get_attention_segments()
            assert [[int(s[2]), int(s[0].shape[2])] for s in segs] == step["segments"]
            assert cache.get_total_length() == step["total_length"]
            # contents: every key row holds its absolute position, every value row position + 0.5
            for kk, vv, start in segs:
                n_ = kk.shape[2]
                expect = torch.arange(start, start + n_, dtype=torch.float32)
                assert torch.equal(kk[0, 0, :, 0].float().cpu(), expect)
                assert torch.equal(vv[0, 0, :, 0].float().cpu(), expect + 0.5)
        return cache


def replay_residency(name, ops_factory, host_tier=False, persist_async=False, at_end=None):
    """``at_end(cache, cfg)`` runs after the last step, while the session files still exist."""
    from rfsn_b200 import LayerKVCache

    sc = RESIDENCY[name]
    with tempfile.TemporaryDirectory() as tmp:
        cfg = _config(sc["hot_capacity"], sc["block_size"], "archived", sc["warm_capacity"], tmp)
        cache = LayerKVCache(cfg, 1, 2, 1, layer_id=0, session_id="golden", ops=ops_factory(), host_tier=host_tier,
                             persist_async=persist_async)
        pos = 0
        for step in sc["steps"]:
            n = step["incoming"]
            cache.evict_for_append(n)
            k = torch.arange(pos, pos + n, dtype=torch.float32)[None, None, :, None].expand(1, 1, n, 4).contiguous()
            cache.append_exact(k.to(cache.device), (-k).to(cache.device))
            if n == 1:
                cache.maybe_prefetch_for_decode(pos)
                cache.residency_manager.wait_for_prefetches(cache)
            pos += n
            before = [m.residency.value for m in cache.block_manager.iter_blocks(layer_id=0)]
            segs = cache.get_attention_segments()
            after = [m.residency.value for m in cache.block_manager.iter_blocks(layer_id=0)]
            assert before == step["residency_before_fetch"]
            assert after == step["residency_after_fetch"]
            assert [[m.logical_start, m.logical_end] for m in cache.block_manager.iter_blocks(layer_id=0)] == step["spans"]
            assert [[int(s[2]), int(s[0].shape[2])] for s in segs] == step["segments"]
            assert [float(s[0][0, 0, 0, 0]) for s in segs] == step["segment_first_values"]
            assert cache.residency_manager.get_metrics() == step["metrics"]
            assert [cache.hot_head_index, cache.hot_seq_len, cache.hot_start] == step["hot"]
        if at_end is not None:
            at_end(cache, cfg)
        return cache


def check_persisted_session(ops_factory):
    """``at_end`` check for a write-behind replay: after a flush every cold
    block's npz and sidecar are on disk, the sidecar's checksum is the SHA-256
    of the npz, the payload holds the block's rows, and a fresh cache restores
    the same page table from the files."""

    def check(cache, cfg):
        import hashlib
        import json
        from pathlib import Path

        from rfsn_b200 import LayerKVCache
        from rfsn_b200.block_manager import BlockLocation

        cache.flush_persistence()
        cold = [m for m in cache.block_manager.iter_blocks(layer_id=0) if m.residency == BlockLocation.COLD_DISK]
        assert cold, "the trace demotes blocks"
        for m in cold:
            blob = Path(m.payload_path).read_bytes()
            assert m.checksum == hashlib.sha256(blob).hexdigest()
            side = json.loads(Path(m.manifest_path).read_text())
            assert side["checksum"] == m.checksum and side["residency"] == "cold_disk"
            loaded = cache.storage.load_block(m)
            pos = torch.arange(m.logical_start, m.logical_end, dtype=torch.float32).numpy()
            assert (loaded["keys"][0, 0, :, 0] == pos).all() and (loaded["values"][0, 0, :, 0] == -pos).all()
        spans = [(m.logical_start, m.logical_end) for m in cache.block_manager.iter_blocks(layer_id=0)]
        fresh = LayerKVCache(cfg, 1, 2, 1, layer_id=0, session_id="golden", ops=ops_factory())
        restored = fresh.restore_from_disk()
        assert [(m.logical_start, m.logical_end) for m in restored] == spans

    return check


def ring_names():
    return sorted(RING)


def residency_names():
    return sorted(RESIDENCY)
