"""The drop-in cache on the GPU: reference traces with real device ops, fused
RoPE + append parity, multi-step decode parity through attention_step, and a
warm -> disk -> restore round trip."""

import tempfile

import numpy as np
import pytest
import torch

from cache_replay import check_persisted_session, replay_residency, replay_ring, residency_names, ring_names
from oracle.rope import apply_rope, inv_freq, rope_tables
from oracle.segmented_attention import run_segmented_attention

pytestmark = pytest.mark.gpu
ATOL = 2e-3


@pytest.mark.parametrize("name", ring_names())
def test_ring_trace_on_device(name):
    replay_ring(name, lambda: None)


@pytest.mark.parametrize("host_tier", [False, True])
@pytest.mark.parametrize("name", residency_names())
def test_residency_trace_on_device(name, host_tier):
    replay_residency(name, lambda: None, host_tier=host_tier)


@pytest.mark.parametrize("name", residency_names())
def test_residency_trace_on_device_with_write_behind(name):
    # demotions download into pinned memory and return; the npz writes land on
    # the layer's writer thread and restore the session after a flush
    replay_residency(name, lambda: None, host_tier=True, persist_async=True,
                     at_end=check_persisted_session(lambda: None))


def _round(x, dtype):
    t = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    return torch.from_numpy(np.ascontiguousarray(x)).to(t).float().numpy()


def _cfg(dtype, H, Hkv, D, cap, bs, tmp, base=10000.0, warm=1 << 20):
    from rfsn_b200 import RFSNConfig

    return RFSNConfig(hidden_dim=H * D, num_heads=H, num_kv_heads=Hkv, head_dim=D, num_layers=1, hot_capacity=cap,
                      warm_capacity=warm, cold_capacity=max(warm, 1 << 21), block_size_seq=bs, model_dtype=dtype,
                      rope_base=base, disk_cache_dir=tmp)


def test_inv_freq_table_matches_oracle():
    from rfsn_b200 import LayerKVCache

    with tempfile.TemporaryDirectory() as tmp:
        c = LayerKVCache(_cfg("bfloat16", 8, 2, 128, 16, 4, tmp, base=500000.0), 1, 8, 2, session_id="t")
        np.testing.assert_array_equal(c.inv_freq().cpu().numpy(), inv_freq(128, 500000.0))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_fused_rope_append_matches_oracle(dtype):
    from rfsn_b200 import LayerKVCache

    H, Hkv, D, L, pos0 = 8, 2, 128, 5, 131000  # large positions: float32 angle products
    rng = np.random.default_rng(31)
    q = rng.standard_normal((1, H, L, D)).astype(np.float32)
    k = rng.standard_normal((1, Hkv, L, D)).astype(np.float32)
    v = rng.standard_normal((1, Hkv, L, D)).astype(np.float32)
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    with tempfile.TemporaryDirectory() as tmp:
        c = LayerKVCache(_cfg(dtype, H, Hkv, D, 8, 4, tmp, base=500000.0), 1, H, Hkv, session_id="t")
        c.hot_start = pos0
        c.evict_for_append(6)
        c.append_exact(torch.zeros((1, Hkv, 6, D), dtype=tdt, device="cuda"), torch.zeros((1, Hkv, 6, D), dtype=tdt,
                                                                                             device="cuda"))
        c.evict_for_append(L)  # 6 + 5 > 8: seals 4 tokens; the 5-token write then wraps (slots 6, 7, 0, 1, 2)
        assert (c.hot_head_index, c.hot_seq_len, c.hot_write_index) == (4, 2, 6)
        start = c.hot_end
        q_rot = c.append_rope(torch.from_numpy(q).to(tdt).cuda(), torch.from_numpy(k).to(tdt).cuda(),
                              torch.from_numpy(v).to(tdt).cuda(), start).cpu().numpy()
        cos_t, sin_t = rope_tables(D, 500000.0, L, start)
        np.testing.assert_allclose(q_rot, apply_rope(_round(q, dtype), cos_t, sin_t), atol=2e-5, rtol=1e-5)
        hot = list(c.get_hot_attention_segments())
        k_dev = torch.cat([s[0] for s in hot], dim=2)[:, :, -L:].float().cpu().numpy()
        v_dev = torch.cat([s[1] for s in hot], dim=2)[:, :, -L:].float().cpu().numpy()
        k_ref = _round(apply_rope(_round(k, dtype), cos_t, sin_t), dtype)
        if dtype == "float32":
            np.testing.assert_allclose(k_dev, k_ref, atol=2e-5, rtol=1e-5)
        else:
            # at most one storage ulp apart (float32 angle/trig rounding can flip a rounding boundary)
            ulp = {"bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}[dtype]
            assert np.all(np.abs(k_dev - k_ref) <= ulp * np.maximum(np.abs(k_ref), 1e-3) + 1e-7)
        np.testing.assert_array_equal(v_dev, _round(v, dtype))


@pytest.mark.parametrize("dtype,H,Hkv,D,cap,bs,chunks,decode", [
    ("bfloat16", 32, 8, 128, 256, 96, [256, 256, 100], 40),   # tensor-core decode kernel
    ("float16", 16, 4, 128, 100, 64, [100, 37, 60], 30),      # wrapped ring, odd seals
    ("float32", 2, 2, 64, 8, 4, [8], 8),                       # tiny-model cache shape
    ("bfloat16", 8, 1, 64, 64, 16, [64, 20], 20),              # head_dim 64, 8 q heads per kv head
])
def test_attention_step_decode_sequence_matches_oracle(dtype, H, Hkv, D, cap, bs, chunks, decode):
    from rfsn_b200 import LayerKVCache
    from rfsn_b200.layer import attention_step

    total = sum(chunks) + decode
    rng = np.random.default_rng(41)
    q = rng.standard_normal((1, H, total, D)).astype(np.float32)
    k = rng.standard_normal((1, Hkv, total, D)).astype(np.float32)
    v = rng.standard_normal((1, Hkv, total, D)).astype(np.float32)
    tdt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(tdt).cuda()  # noqa: E731
    cos_t, sin_t = rope_tables(D, 10000.0, total, 0)
    k_all = _round(apply_rope(_round(k, dtype), cos_t, sin_t), dtype)
    v_all = _round(v, dtype)
    with tempfile.TemporaryDirectory() as tmp:
        cache = LayerKVCache(_cfg(dtype, H, Hkv, D, cap, bs, tmp), 1, H, Hkv, session_id="t")
        pos = 0
        steps = list(chunks) + [1] * decode
        worst = 0.0
        for n in steps:
            out = attention_step(dev(q[:, :, pos:pos + n]), dev(k[:, :, pos:pos + n]), dev(v[:, :, pos:pos + n]),
                                 cache, pos).cpu().numpy()
            q_rot = apply_rope(_round(q[:, :, pos:pos + n], dtype), cos_t[pos:pos + n], sin_t[pos:pos + n])
            ref = run_segmented_attention(q_rot, [(k_all[:, :, :pos + n], v_all[:, :, :pos + n], 0)], pos, grouped=True)
            worst = max(worst, float(np.abs(out - ref).max()))
            pos += n
        assert cache.get_block_stats()["total_blocks"] > 0
        assert worst <= ATOL, worst


def test_demote_to_disk_and_restore_session():
    from rfsn_b200 import RFSNCache
    from rfsn_b200.block_manager import BlockLocation
    from rfsn_b200.layer import attention_step

    H, Hkv, D = 8, 2, 128
    rng = np.random.default_rng(51)
    n_prompt = 300
    q = rng.standard_normal((1, H, n_prompt + 1, D)).astype(np.float32)
    k = rng.standard_normal((1, Hkv, n_prompt + 1, D)).astype(np.float32)
    v = rng.standard_normal((1, Hkv, n_prompt + 1, D)).astype(np.float32)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).cuda()  # noqa: E731
    with tempfile.TemporaryDirectory() as tmp:
        cfg = _cfg("bfloat16", H, Hkv, D, 64, 64, tmp, warm=1 << 12)
        cfg.session_id = "restore-me"
        cache = RFSNCache(cfg, 1)
        lc = cache.layer(0)
        for s in range(0, n_prompt, 64):
            n = min(64, n_prompt - s)
            attention_step(dev(q[:, :, s:s + n]), dev(k[:, :, s:s + n]), dev(v[:, :, s:s + n]), lc, s)
        lc.evict_for_append(cfg.hot_capacity)  # seal the whole hot window
        for m in list(lc.block_manager.iter_blocks(layer_id=0)):
            if m.residency == BlockLocation.WARM_RAM:
                lc.demote_manifest_to_cold(m)
        restored = RFSNCache(cfg, 1, restore=True)
        manifests = restored.restore_from_disk()
        assert sum(len(x) for x in manifests) == len(lc.block_manager.iter_blocks(layer_id=0))
        assert restored.layer(0).hot_start == n_prompt
        a = attention_step(dev(q[:, :, n_prompt:]), dev(k[:, :, n_prompt:]), dev(v[:, :, n_prompt:]), lc, n_prompt)
        b = attention_step(dev(q[:, :, n_prompt:]), dev(k[:, :, n_prompt:]), dev(v[:, :, n_prompt:]),
                           restored.layer(0), n_prompt)
        np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
        with pytest.raises(FileNotFoundError, match="unknown session"):
            other = _cfg("bfloat16", H, Hkv, D, 64, 64, tmp, warm=1 << 12)
            other.session_id = "nobody"
            RFSNCache(other, 1, restore=True).restore_from_disk()


def test_graphed_decode_step_matches_attention_step():
    """rfsn_b200.layer.GraphedDecodeStep (host buffers, one graph replay per call,
    re-captured after each seal) against attention_step on a twin cache."""
    from rfsn_b200 import LayerKVCache
    from rfsn_b200.layer import GraphedDecodeStep, attention_step

    with tempfile.TemporaryDirectory() as tmp:
        cfg = _cfg("bfloat16", 16, 4, 128, 256, 96, tmp)
        caches = [LayerKVCache(cfg, 1, 16, 4, layer_id=0, session_id=f"g{i}") for i in range(2)]
        gen = torch.Generator(device="cuda").manual_seed(21)
        for n in (256, 200):  # prefill-like appends: seal rule + archived blocks
            k = torch.randn((1, 4, n, 128), generator=gen, device="cuda").to(torch.bfloat16)
            v = torch.randn((1, 4, n, 128), generator=gen, device="cuda").to(torch.bfloat16)
            for c in caches:
                c.evict_for_append(n)
                c.append_exact(k, v)
        eager, graphed_cache = caches
        step = GraphedDecodeStep(graphed_cache, 16)
        pos = eager.hot_end
        for i in range(300):  # crosses several 96-token seals
            q = torch.randn((1, 16, 1, 128), generator=gen, device="cuda").to(torch.bfloat16)
            k = torch.randn((1, 4, 1, 128), generator=gen, device="cuda").to(torch.bfloat16)
            v = torch.randn((1, 4, 1, 128), generator=gen, device="cuda").to(torch.bfloat16)
            want = attention_step(q, k, v, eager, pos).cpu()
            step.q_host.copy_(q.cpu())
            step.k_host.copy_(k.cpu())
            step.v_host.copy_(v.cpu())
            got = step.step(pos)
            assert float((got - want).abs().max()) <= 1e-5, i
            assert (eager.hot_head_index, eager.hot_seq_len, eager.hot_start) == \
                   (graphed_cache.hot_head_index, graphed_cache.hot_seq_len, graphed_cache.hot_start)
            pos += 1
        assert step.replays > 250 and step.captures >= 3 and step.fallbacks == 0, (step.replays, step.captures)
        step.workspace.check()


def test_paged_attention_into_given_output():
    """paged_attention(out=...) writes the same result into a device tensor or
    into pinned host memory (across the bus); other outputs are refused."""
    from rfsn_b200 import LayerKVCache
    from rfsn_b200 import _native as native
    from rfsn_b200.cache import paged_attention

    with tempfile.TemporaryDirectory() as tmp:
        cfg = _cfg("bfloat16", 8, 2, 128, 256, 128, tmp)
        c = LayerKVCache(cfg, 1, 8, 2, layer_id=0, session_id="out")
        gen = torch.Generator(device="cuda").manual_seed(3)
        k = torch.randn((1, 2, 256, 128), generator=gen, device="cuda").to(torch.bfloat16)
        v = torch.randn((1, 2, 256, 128), generator=gen, device="cuda").to(torch.bfloat16)
        for _ in range(2):
            c.evict_for_append(256)
            c.append_exact(k, v)
        q = torch.randn((1, 8, 1, 128), generator=gen, device="cuda")
        segs = c.get_attention_segments()
        pos = c.hot_end - 1
        want = paged_attention(c, q, pos, segs).cpu()
        dev_out = torch.full((1, 8, 1, 128), float("nan"), device="cuda")
        assert paged_attention(c, q, pos, segs, out=dev_out) is dev_out
        pinned = torch.full((1, 8, 1, 128), float("nan")).pin_memory()
        paged_attention(c, q, pos, segs, out=pinned)
        torch.cuda.synchronize()
        assert torch.equal(dev_out.cpu(), want) and torch.equal(pinned, want)
        with pytest.raises(ValueError):
            paged_attention(c, q, pos, segs, out=torch.zeros((1, 8, 1, 128)))  # pageable host memory
        with pytest.raises(ValueError):
            paged_attention(c, q, pos, segs, out=torch.zeros((1, 8, 2, 128), device="cuda"))
        with pytest.raises(ValueError):
            native.host_device_pointer(torch.zeros(4))


def test_block_upload_is_ordered_before_the_next_compute_kernel():
    """DeviceOps.upload copies a block into the arena on a side stream; the
    compute stream must wait for that copy before its next kernel. A 128 MB
    block (K and V each) read by the very next kernels on the compute stream
    shows the uploaded values every time (the copy takes milliseconds over the
    bus, so a missing wait would show stale rows)."""
    from rfsn_b200.cache import DeviceOps

    ops = DeviceOps("cuda")
    groups, n, D = 8, 65536, 128
    k_arena, v_arena = ops.new_arena(groups, n, D, torch.bfloat16)
    for trial in range(3):
        val = float(trial + 1)
        k = torch.full((groups, n, D), val, dtype=torch.bfloat16).pin_memory()
        v = torch.full((groups, n, D), -val, dtype=torch.bfloat16).pin_memory()
        ops.upload(0, n, k, v)
        assert bool((k_arena == val).all()) and bool((v_arena == -val).all()), trial
    torch.cuda.synchronize()
