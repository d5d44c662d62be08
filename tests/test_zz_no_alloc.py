"""rfsn_paged_attention_noalloc: the allocation-free paged attention call.

Callers that cannot allocate device memory while they run attention (an
engine that owns all GPU memory through its own pool, a frozen memory
budget, a plugin host that only passes inputs and outputs) use this entry
point; its split scratch is a fixed array built into the library instead of
a caller workspace. These tests call it through the C ABI and compare it with
rfsn_paged_attention (which takes a workspace) and with the float32 oracle on
two calls in a row, so the second call also shows that the shared scratch is
cleared between calls; the device's free memory is read around the second
call to show that nothing is allocated. Kernel-side failures land in the
array's error word, read and cleared by rfsn_noalloc_check.
This file is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest

from _util import make_layout, to_device_storage
from oracle.segmented_attention import run_segmented_attention

pytestmark = pytest.mark.gpu
ATOL = 2e-3  # the max-abs tolerance used by the attention parity tests


def _device_case(layout, q_np):
    import torch

    from rfsn_b200 import _native as native

    k = to_device_storage(layout.k_store, layout.dtype)
    v = to_device_storage(layout.v_store, layout.dtype)
    arena = native.Arena(k, v)
    rec = torch.from_numpy(layout.records).cuda()
    nblk = len(layout.block_lens)
    table = native.PageTableC(rec.data_ptr(), nblk, int(sum(layout.block_lens)), int(layout.records[nblk, 3]), 0)
    hot = native.HotWindowC(0, layout.ring_cap, layout.hot_head, layout.hot_len, layout.hot_start)
    q = torch.from_numpy(np.ascontiguousarray(q_np)).cuda()
    return dict(k=k, v=v, arena=arena, rec=rec, table=table, hot=hot, q=q)


def _with_workspace(c, layout):
    import torch

    from rfsn_b200 import _native as native

    B, H, Lq, D = c["q"].shape
    out = torch.empty_like(c["q"])
    lse = torch.empty((B, H, Lq), device="cuda")
    nbytes = native.workspace_bytes(B, H, layout.kv_heads, Lq, D)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    native.check(
        native.lib().rfsn_paged_attention(
            c["arena"].handle, c["q"].data_ptr(), B, H, layout.kv_heads, Lq, layout.total_tokens - Lq,
            ctypes.byref(c["table"]), ctypes.byref(c["hot"]), out.data_ptr(), lse.data_ptr(), ws.data_ptr(), nbytes,
            0, native.stream_ptr(),
        ),
        "rfsn_paged_attention",
    )
    torch.cuda.synchronize()
    return out.cpu().numpy(), lse.cpu().numpy()


def _no_alloc(c, layout, *, free_bytes=None):
    """One call of the entry point; with ``free_bytes`` (a list) the device's
    free memory before the call and after it completed is appended to it."""
    import torch

    from rfsn_b200 import _native as native

    B, H, Lq, D = c["q"].shape
    out = torch.empty_like(c["q"])
    lse = torch.empty((B, H, Lq), device="cuda")
    torch.cuda.synchronize()
    if free_bytes is not None:
        free_bytes.append(torch.cuda.mem_get_info()[0])
    status = native.lib().rfsn_paged_attention_noalloc(
        c["arena"].handle, c["q"].data_ptr(), B, H, layout.kv_heads, Lq, layout.total_tokens - Lq,
        ctypes.byref(c["table"]), ctypes.byref(c["hot"]), out.data_ptr(), lse.data_ptr(), 0, native.stream_ptr(),
    )
    torch.cuda.synchronize()
    if free_bytes is not None:
        free_bytes.append(torch.cuda.mem_get_info()[0])
    return status, out.cpu().numpy(), lse.cpu().numpy()


def _noalloc_check():
    from rfsn_b200 import _native as native

    return native.lib().rfsn_noalloc_check(native.stream_ptr(), 30_000_000)


@pytest.mark.parametrize(
    "dtype,B,H,Hkv,Lq,D,blocks",
    [
        ("bfloat16", 1, 32, 8, 1, 128, [1000] * 12 + [24]),  # tensor-core kernel
        ("float16", 1, 32, 8, 1, 128, [256] * 6),
        ("float32", 1, 4, 2, 3, 64, [37, 64, 5]),              # CUDA-core kernel
        ("float16", 1, 32, 8, 1024, 128, [512, 512]),          # tensor-core prefill: no partials when unsplit
    ],
)
def test_noalloc_matches_workspace_entry_point_twice(dtype, B, H, Hkv, Lq, D, blocks):
    from rfsn_b200 import _native as native

    layout = make_layout(dtype, B, Hkv, D, blocks, 256, 200, 100, seed=21)
    q = np.random.default_rng(21).standard_normal((B, H, Lq, D), dtype=np.float32)
    c = _device_case(layout, q)
    ref_out, ref_lse = _with_workspace(c, layout)
    oracle_out, oracle_lse = run_segmented_attention(q, layout.oracle_segments(), layout.total_tokens - Lq,
                                                     return_lse=True, grouped=True)
    free = []
    for call in range(2):
        status, out, lse = _no_alloc(c, layout, free_bytes=free if call == 1 else None)
        assert status == native.RFSN_OK, native.last_error()
        assert _noalloc_check() == native.RFSN_OK, native.last_error()
        assert float(np.abs(out - ref_out).max()) <= ATOL
        np.testing.assert_allclose(lse, ref_lse, atol=1e-4)
        assert float(np.abs(out - oracle_out).max()) <= ATOL
        np.testing.assert_allclose(lse, oracle_lse, atol=1e-4, rtol=1e-5)
    assert free[0] == free[1], f"device free memory changed across the call: {free[0]} -> {free[1]}"
    c["arena"].close()


def test_noalloc_reports_a_record_outside_the_arena_through_its_check():
    """A page-table record that points past the arena is flagged by the kernel
    (its keys are skipped, nothing is read out of bounds); the flag stays in the
    built-in error word until rfsn_noalloc_check reports and clears it."""
    import torch

    from rfsn_b200 import _native as native

    layout = make_layout("bfloat16", 1, 8, 128, [300, 200], 256, 100, 10, seed=23)
    q = np.random.default_rng(123).standard_normal((1, 32, 1, 128), dtype=np.float32)
    c = _device_case(layout, q)
    assert _noalloc_check() == native.RFSN_OK, native.last_error()  # start from a clean word
    bad = layout.records.copy()
    bad[1, 0] = layout.rows - 50  # the 200-row block would run 150 rows past the arena
    c["rec"].copy_(torch.from_numpy(bad))
    status, _, _ = _no_alloc(c, layout)
    assert status == native.RFSN_OK, native.last_error()
    assert _noalloc_check() == native.RFSN_ERR_DEVICE
    assert "outside the arena" in native.last_error()
    assert _noalloc_check() == native.RFSN_OK, native.last_error()  # the check cleared it
    # with the table repaired the next call is clean and correct
    c["rec"].copy_(torch.from_numpy(layout.records))
    status, out, _ = _no_alloc(c, layout)
    assert status == native.RFSN_OK, native.last_error()
    assert _noalloc_check() == native.RFSN_OK, native.last_error()
    ref = run_segmented_attention(q, layout.oracle_segments(), layout.total_tokens - 1, grouped=True)
    assert float(np.abs(out - ref).max()) <= ATOL
    c["arena"].close()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from rfsn_b200 import _native as native

    # 1024 query rows x 4 heads per KV head on the CUDA-core kernel (float32 K/V):
    # its per-row partials alone exceed the built-in array.
    layout = make_layout("float32", 1, 8, 128, [64, 64], 2048, 1024, 0, seed=22)
    q = np.zeros((1, 32, 1024, 128), np.float32)
    c = _device_case(layout, q)
    status, _, _ = _no_alloc(c, layout)
    assert status == native.RFSN_ERR_OVERFLOW
    assert "built-in scratch" in native.last_error()
    c["arena"].close()
