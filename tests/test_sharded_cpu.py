"""Rank logic of context-sharded decode with world_size-2 gloo process groups
on CPU: block partitioning, the (output, LSE) gather of rfsn_b200.sharded,
and failure detection when a rank never joins the collective."""

import datetime
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

BLOCKS = [64, 100, 7, 256, 33]
HOT = 48


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(61)
    segs, pos = [], 0
    for n in BLOCKS + [HOT]:
        segs.append((rng.standard_normal((1, 2, n, 64), dtype=np.float32),
                     rng.standard_normal((1, 2, n, 64), dtype=np.float32), pos))
        pos += n
    q = rng.standard_normal((1, 8, 1, 64), dtype=np.float32)
    return q, segs, pos - 1


def _worker(rank, world, port, mode, results):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "rfsn-mlx_b200"), os.path.join(root, "tests")]
        import torch
        import torch.distributed as dist

        from oracle.segmented_attention import merge_partials, run_segmented_attention
        from rfsn_b200.sharded import gather_parts, shard_range

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        q, segs, qpos = _inputs()
        if mode == "dropout" and rank == 1:
            results.put((rank, "left"))
            results.close()
            results.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves between steps, before joining the collective
        lo, hi = shard_range(len(BLOCKS), rank, world)
        mine = segs[lo:hi] + ([segs[-1]] if rank == world - 1 else [])
        if mine:
            out, lse = run_segmented_attention(q, mine, qpos, return_lse=True)
        else:
            out, lse = np.zeros_like(q), np.full(q.shape[:3], -np.inf, np.float32)
        try:
            po, pl = gather_parts(torch.from_numpy(out), torch.from_numpy(lse))
        except Exception as exc:  # the peer vanished: reported on the host, no device involved
            results.put((rank, f"error: {type(exc).__name__}"))
            return
        merged = merge_partials([x.reshape(q.shape) for x in po.numpy()], [x.reshape(q.shape[:3]) for x in pl.numpy()])
        full = run_segmented_attention(q, segs, qpos)
        results.put((rank, float(np.abs(merged - full).max())))
        dist.destroy_process_group()
    except Exception:
        results.put((rank, "crash: " + traceback.format_exc()))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, val = results.get(timeout=120)
        got[rank] = val
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return got


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_gather_and_merge_equals_unsharded(world):
    got = _run(world, "ok")
    for rank in range(world):
        assert isinstance(got[rank], float), got[rank]
        assert got[rank] <= 2e-6


def test_rank_that_never_joins_is_detected_on_the_host():
    got = _run(2, "dropout")
    assert got[1] == "left"
    assert isinstance(got[0], str) and got[0].startswith("error"), got[0]


def test_balanced_shards_are_contiguous_and_balanced():
    from rfsn_b200.sharded import balanced_shards

    blocks = [1000] * 127 + [1024]
    for world in (1, 2, 4, 8):
        ranges = balanced_shards(blocks, 4096, world)
        assert ranges[0][0] == 0 and ranges[-1][1] == len(blocks)
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        loads = [sum(blocks[lo:hi]) + (4096 if r == world - 1 else 0) for r, (lo, hi) in enumerate(ranges)]
        assert max(loads) - min(loads) <= 1024 + 24


def test_shard_ranges_partition_blocks_contiguously():
    from rfsn_b200.sharded import shard_range

    for n in (1, 7, 128):
        for world in (1, 2, 4, 8):
            ranges = [shard_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


def test_balanced_shards_random_layouts():
    """Random block lists and hot windows: ranges are contiguous and cover every
    block, and each rank's end boundary is the block boundary closest to its
    share of the tokens among the boundaries not before the previous rank's."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies
    from rfsn_b200.sharded import balanced_shards

    @hyp.settings(max_examples=300, deadline=None, derandomize=True)
    @hyp.given(blocks=st.lists(st.integers(1, 4096), min_size=0, max_size=200), hot=st.integers(0, 8192),
               world=st.sampled_from([1, 2, 3, 4, 8]))
    def check(blocks, hot, world):
        ranges = balanced_shards(blocks, hot, world)
        assert len(ranges) == world and ranges[0][0] == 0 and ranges[-1][1] == len(blocks)
        assert all(lo <= hi for lo, hi in ranges) and all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        cum = [0]
        for n in blocks:
            cum.append(cum[-1] + n)
        total = cum[-1] + hot
        for r in range(1, world):
            target = total * r / world
            b = ranges[r][0]
            allowed = range(ranges[r - 1][0], len(blocks) + 1)
            assert all(abs(cum[b] - target) <= abs(cum[x] - target) for x in allowed)

    check()
