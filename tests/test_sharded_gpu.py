"""Context-sharded decode on GPUs.

With one GPU the ranks are emulated: each shard is its own LayerKVCache on the
same device, attends with the paged kernel (returning LSE), and the parts are
combined with the native LSE merge, exactly what each rank does after the
all-gather. With two or more GPUs a real NCCL run (one process per GPU)
checks sharded_decode_step against the unsharded oracle.
"""

import datetime
import multiprocessing as mp
import os
import socket
import tempfile
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
BLOCKS = [1000] * 12 + [1024]
HOT, H, HKV, D = 512, 32, 8, 128


def _data(seed=71):
    rng = np.random.default_rng(seed)
    total = sum(BLOCKS) + HOT
    k = rng.standard_normal((1, HKV, total, D), dtype=np.float32)
    v = rng.standard_normal((1, HKV, total, D), dtype=np.float32)
    q = rng.standard_normal((1, H, 1, D), dtype=np.float32)
    return q, k, v, total


def _shard_cache(rank, world, k, v, device, tmp):
    import torch

    from rfsn_b200 import LayerKVCache, RFSNConfig
    from rfsn_b200.sharded import shard_range

    cfg = RFSNConfig(hidden_dim=H * D, num_heads=H, num_kv_heads=HKV, head_dim=D, num_layers=1, hot_capacity=HOT,
                     warm_capacity=1 << 17, cold_capacity=1 << 18, block_size_seq=1000, model_dtype="bfloat16",
                     disk_cache_dir=tmp)
    cache = LayerKVCache(cfg, 1, H, HKV, session_id=f"s{rank}", device=device)
    lo, hi = shard_range(len(BLOCKS), rank, world)
    starts = np.cumsum([0] + BLOCKS[:-1])
    bf = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).to(device)  # noqa: E731
    for i in range(lo, hi):
        s = int(starts[i])
        cache.import_block(bf(k[:, :, s:s + BLOCKS[i]]), bf(v[:, :, s:s + BLOCKS[i]]), s)
    cache.hot_start = sum(BLOCKS)
    if rank == world - 1:
        a = sum(BLOCKS)
        cache.evict_for_append(HOT)
        cache.append_exact(bf(k[:, :, a:]), bf(v[:, :, a:]))
    return cache


def _oracle(q, k, v, total):
    import torch

    from oracle.segmented_attention import run_segmented_attention

    r = lambda x: torch.from_numpy(x).to(torch.bfloat16).float().numpy()  # noqa: E731
    return run_segmented_attention(q, [(r(k), r(v), 0)], total - 1, grouped=True)


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_emulated_ranks_merge_to_unsharded_result(world):
    import torch

    from rfsn_b200.sharded import merge_parts

    q, k, v, total = _data()
    qd = torch.from_numpy(q).cuda()
    outs, lses = [], []
    with tempfile.TemporaryDirectory() as tmp:
        for rank in range(world):
            cache = _shard_cache(rank, world, k, v, torch.device("cuda", 0), tmp)
            segs = cache.get_attention_segments()
            if len(segs) == 0:
                outs.append(torch.zeros_like(qd))
                lses.append(torch.full(q.shape[:3], float("-inf"), device="cuda"))
                continue
            o, l = cache.attend(qd, total - 1, segs, want_lse=True)
            outs.append(o)
            lses.append(l)
        rows = H
        merged = merge_parts(torch.stack(outs).reshape(world, rows, D), torch.stack(lses).reshape(world, rows), qd.shape)
        full = _shard_cache(0, 1, k, v, torch.device("cuda", 0), tmp).attend(qd, total - 1)
    ref = _oracle(q, k, v, total)
    assert float(np.abs(merged.cpu().numpy() - ref).max()) <= 2e-3
    np.testing.assert_allclose(merged.cpu().numpy(), full.cpu().numpy(), atol=1e-5)


def test_peer_group_of_one_matches_local_attention():
    """The fused-merge kernel path with a single rank: its mailbox exchange
    (store, release flag, acquire wait, merge) must reproduce the local result
    on consecutive calls (both mailbox halves)."""
    import torch

    from rfsn_b200.cache import paged_attention
    from rfsn_b200.sharded import PeerGroup

    q, k, v, total = _data()
    qd = torch.from_numpy(q).cuda()
    with tempfile.TemporaryDirectory() as tmp:
        cache = _shard_cache(0, 1, k, v, torch.device("cuda", 0), tmp)
        segs = cache.get_attention_segments()
        ref, ref_lse = paged_attention(cache, qd, total - 1, segs, want_lse=True)
        peers = PeerGroup(1 * HKV, D)
        for _ in range(3):
            out, lse = paged_attention(cache, qd, total - 1, segs, want_lse=True, peers=peers)
            np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=1e-6)
            np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=1e-5)
        from rfsn_b200 import _native as native

        native.default_workspace(torch.device("cuda", 0)).check()
        peers.close()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, results, mode="nccl"):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "rfsn-mlx_b200"), os.path.join(root, "tests")]
        import torch
        import torch.distributed as dist

        from rfsn_b200.cache import paged_attention
        from rfsn_b200.sharded import PeerGroup, sharded_decode_step

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        q, k, v, total = _data()
        with tempfile.TemporaryDirectory() as tmp:
            # context minus the last token; the hot owner appends that token in the decode step
            kk, vv = k[:, :, :-1], v[:, :, :-1]
            cache = _shard_cache(rank, world, np.concatenate([kk, np.zeros_like(k[:, :, :1])], 2),
                                 np.concatenate([vv, np.zeros_like(v[:, :, :1])], 2), torch.device("cuda", rank), tmp)
            owner = rank == world - 1
            if owner:  # drop the placeholder token again: the step appends the real one
                cache.hot_seq_len -= 1
            # rotate-free check: feed q/k/v that are already "rotated" is not possible through the
            # step (it applies RoPE), so compare against the oracle with RoPE applied.
            import torch as T

            bf = lambda x: T.from_numpy(np.ascontiguousarray(x)).to(T.bfloat16).cuda()  # noqa: E731
            peers = PeerGroup(HKV, D) if mode == "p2p" else None
            out = sharded_decode_step(cache, bf(q), bf(k[:, :, -1:]) if owner else None,
                                      bf(v[:, :, -1:]) if owner else None, total - 1, owns_hot=owner, peers=peers)
            outs = [out.cpu().numpy()]
            if peers is not None:
                # more calls on the same context: alternate mailbox halves, same result
                q_rot = cache.rope_query(bf(q), total - 1)
                for _ in range(3):
                    outs.append(paged_attention(cache, q_rot, total - 1, cache.get_attention_segments(),
                                                peers=peers).cpu().numpy())
                from rfsn_b200 import _native as native

                native.default_workspace(torch.device("cuda", rank)).check()
                peers.close()
            results.put((rank, outs))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results.put((rank, "crash: " + traceback.format_exc()))


def _gpus():
    import torch

    return torch.cuda.device_count()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["nccl", "p2p"])
def test_sharded_decode_step_on_gpus(mode, world):
    """One process per GPU (2, 4 or 8 of them, skipped when fewer are
    visible): the merged result of every rank equals the unsharded oracle, for
    the NCCL gather and for the merge fused into the kernel over NVLink (from
    three ranks on, every peer's words are polled in one round)."""
    import torch

    from oracle.rope import apply_rope, rope_tables

    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, results, mode)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(results.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for rank in range(world):
        assert not isinstance(got[rank], str), got[rank]
    q, k, v, total = _data()
    r = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()  # noqa: E731
    cos_t, sin_t = rope_tables(D, 10000.0, 1, total - 1)
    k_last = r(apply_rope(r(k[:, :, -1:]), cos_t, sin_t))
    k_ctx = np.concatenate([r(k[:, :, :-1]), k_last], axis=2)
    q_rot = apply_rope(r(q), cos_t, sin_t)
    from oracle.segmented_attention import run_segmented_attention

    ref = run_segmented_attention(q_rot, [(k_ctx, r(v), 0)], total - 1, grouped=True)
    for rank in range(world):
        for out in got[rank]:
            assert float(np.abs(out - ref).max()) <= 2e-3


def _silent_peer_worker(rank, port, results):
    """Two processes on cuda:0 form a world-2 peer group (gloo for the handle
    exchange). Rank 1 never runs the attention kernel; rank 0's fused merge must
    give up after its short timeout, report it through the workspace error word,
    and leave the context usable."""
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "rfsn-mlx_b200"), os.path.join(root, "tests")]
        import torch
        import torch.distributed as dist

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(0)
        dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
        from rfsn_b200 import _native as native
        from rfsn_b200.cache import paged_attention
        from rfsn_b200.sharded import PeerGroup

        q, k, v, total = _data()
        with tempfile.TemporaryDirectory() as tmp:
            cache = _shard_cache(rank, 2, k, v, torch.device("cuda", 0), tmp)
            peers = PeerGroup(HKV, D, timeout_s=0.05)
            msg = "no call"
            if rank == 0:
                qd = torch.from_numpy(q).cuda()
                segs = cache.get_attention_segments()
                paged_attention(cache, qd, total - 1, segs, peers=peers)
                ws = native.default_workspace(torch.device("cuda", 0))
                try:
                    ws.check(timeout_s=30.0)
                    msg = "no error reported"
                except TimeoutError as exc:
                    msg = "timeout: " + str(exc)
                # the context still works: a plain local call and a clean error word
                out = paged_attention(cache, qd, total - 1, segs)
                torch.cuda.synchronize()
                ws.check()
                msg += f" | finite={bool(torch.isfinite(out).all())}"
                # the group is unusable now: a second peer call does not wait, does not
                # merge words left from the expired call, and reports the timeout again
                again = paged_attention(cache, qd, total - 1, segs, peers=peers)
                try:
                    ws.check(timeout_s=30.0)
                    msg += " | second call: no error"
                except TimeoutError:
                    msg += " | second call: timeout"
                msg += f" | second call local={bool(torch.equal(again, out))}"
            dist.barrier()  # rank 1 stays idle until rank 0 is done
            peers.close()
            results.put((rank, msg))
        dist.destroy_process_group()
    except Exception:
        results.put((rank, "crash: " + traceback.format_exc()))


def test_peer_merge_timeout_is_reported_and_context_survives():
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_silent_peer_worker, args=(r, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(results.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert got[0].startswith("timeout:") and "the cross-GPU merge timed out" in got[0], got[0]
    assert "finite=True" in got[0], got[0]
    assert got[0].endswith("second call: timeout | second call local=True"), got[0]
    assert got[1] == "no call", got[1]


def test_graphed_sharded_step_with_a_peer_group_of_one_matches_attention_step():
    """GraphedShardedDecodeStep on the hot-window owner of a one-rank peer group
    (the in-kernel merge runs with a single part) against attention_step on a twin
    cache, over enough tokens to seal blocks and re-capture."""
    import torch

    from rfsn_b200.layer import attention_step
    from rfsn_b200.sharded import GraphedShardedDecodeStep, PeerGroup

    q, k, v, total = _data()
    with tempfile.TemporaryDirectory() as tmp:
        dev = torch.device("cuda", 0)
        a = _shard_cache(0, 1, k, v, dev, tmp + "/a")
        b = _shard_cache(0, 1, k, v, dev, tmp + "/b")
        peers = PeerGroup(HKV, D)
        step = GraphedShardedDecodeStep(b, H, owns_hot=True, peers=peers)
        gen = torch.Generator(device="cuda").manual_seed(5)
        pos = a.hot_end
        for i in range(1200):  # the 512-token ring seals 1000-token blocks
            qq = torch.randn((1, H, 1, D), generator=gen, device="cuda").to(torch.bfloat16)
            kk = torch.randn((1, HKV, 1, D), generator=gen, device="cuda").to(torch.bfloat16)
            vv = torch.randn((1, HKV, 1, D), generator=gen, device="cuda").to(torch.bfloat16)
            want = attention_step(qq, kk, vv, a, pos).cpu()
            step.q_host.copy_(qq.cpu())
            step.k_host.copy_(kk.cpu())
            step.v_host.copy_(vv.cpu())
            got = step.step(pos)
            assert float((got - want).abs().max()) <= 1e-5, i
            pos += 1
        assert (a.hot_head_index, a.hot_seq_len, a.hot_start) == (b.hot_head_index, b.hot_seq_len, b.hot_start)
        assert step.replays > 1000 and step.captures >= 2, (step.replays, step.captures)
        step._inner.workspace.check()
        peers.close()


def _graphed_worker(rank, world, port, results, tokens):
    """Each rank drives two copies of its shard with the same peer group: one
    through sharded_decode_step (op by op), one through GraphedShardedDecodeStep
    (one graph replay per token; the owner re-captures after each seal while the
    other ranks keep replaying)."""
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "rfsn-mlx_b200"), os.path.join(root, "tests")]
        import torch
        import torch.distributed as dist

        from rfsn_b200 import _native as native
        from rfsn_b200.sharded import GraphedShardedDecodeStep, PeerGroup, sharded_decode_step

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        q, k, v, total = _data()
        dev = torch.device("cuda", rank)
        owner = rank == world - 1
        with tempfile.TemporaryDirectory() as tmp:
            eager = _shard_cache(rank, world, k, v, dev, tmp + "/e")
            graphed = _shard_cache(rank, world, k, v, dev, tmp + "/g")
            peers = PeerGroup(HKV, D)
            step = GraphedShardedDecodeStep(graphed, H, owns_hot=owner, peers=peers)
            gen = torch.Generator().manual_seed(9)
            worst = 0.0
            for i in range(tokens):
                qq = torch.randn((1, H, 1, D), generator=gen).to(torch.bfloat16)
                kk = torch.randn((1, HKV, 1, D), generator=gen).to(torch.bfloat16)
                vv = torch.randn((1, HKV, 1, D), generator=gen).to(torch.bfloat16)
                pos = total + i
                want = sharded_decode_step(eager, qq.to(dev), kk.to(dev) if owner else None,
                                           vv.to(dev) if owner else None, pos, owns_hot=owner, peers=peers).cpu()
                step.q_host.copy_(qq)
                if owner:
                    step.k_host.copy_(kk)
                    step.v_host.copy_(vv)
                got = step.step(pos)
                worst = max(worst, float((got - want).abs().max()))
            native.default_workspace(dev).check()
            step._inner.workspace.check()
            peers.close()
            results.put((rank, (worst, step.replays, step.captures)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        results.put((rank, "crash: " + traceback.format_exc()))


@pytest.mark.skipif("not __import__('torch').cuda.device_count() >= 2", reason="needs 2 GPUs")
def test_graphed_sharded_step_two_gpus_matches_op_by_op():
    world, tokens = 2, 1100  # the owner's 512-token ring seals twice
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_graphed_worker, args=(r, world, port, results, tokens)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(results.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for rank in range(world):
        assert not isinstance(got[rank], str), got[rank]
        worst, replays, captures = got[rank]
        assert worst <= 1e-5, (rank, worst)
        assert replays + captures == tokens
    assert got[world - 1][2] >= 3  # owner: first token and one per seal
    assert got[0][2] == 1  # the other rank's page table never changes
