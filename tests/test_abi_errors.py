"""Argument checking at the C-ABI boundary (no GPU needed).

Every entry point validates its pointers and sizes on the host before it
touches the CUDA runtime, returns RFSN_ERR_INVALID_ARG with a message that
names the function, and the Python layer maps that code to ValueError, the
exception the reference raises for bad positions, shapes and head counts
(rfsn_v10_5/config.py:88-129, rfsn_v10_5/model.py:77-99). Only invalid
arguments are passed here, so no call reaches a kernel launch.
"""

import ctypes

import pytest

from rfsn_b200 import _native as native

BAD = native.RFSN_ERR_INVALID_ARG
FAKE = 0x10000  # a non-NULL, 16-byte aligned address that is never dereferenced


@pytest.fixture(scope="module")
def lib():
    return native.load_library()


def _expect_bad(status, fragment):
    assert status == BAD, (status, native.last_error())
    assert fragment in native.last_error()


def test_device_and_arena_arguments(lib):
    _expect_bad(lib.rfsn_device_sm_count(None), "rfsn_device_sm_count")
    out = ctypes.c_void_p()
    _expect_bad(lib.rfsn_arena_create(None, FAKE, native.RFSN_BF16, 8, 64, 128, ctypes.byref(out)), "NULL arena")
    _expect_bad(lib.rfsn_arena_create(FAKE, FAKE, 7, 8, 64, 128, ctypes.byref(out)), "unknown dtype")
    _expect_bad(lib.rfsn_arena_create(FAKE, FAKE, native.RFSN_BF16, 8, 0, 128, ctypes.byref(out)), "non-positive")
    _expect_bad(lib.rfsn_arena_create(FAKE, FAKE, native.RFSN_BF16, 8, 64, 127, ctypes.byref(out)), "even")
    _expect_bad(lib.rfsn_arena_create(FAKE + 8, FAKE, native.RFSN_BF16, 8, 64, 128, ctypes.byref(out)), "aligned")
    _expect_bad(lib.rfsn_arena_create(FAKE, FAKE, native.RFSN_BF16, 8, 64, 128, None), "out is NULL")
    assert out.value is None


def test_ring_and_block_copy_arguments(lib):
    f32 = native.RFSN_F32
    # (q, k, v, dtype, inv_freq, pos0, batch, heads, kv heads, len, d, q_out, arena, ring row0, capacity, write, stream)
    _expect_bad(lib.rfsn_rope_append(FAKE, FAKE, FAKE, f32, FAKE, 0, 1, 32, 8, 1, 128, FAKE, None, 0, 64, 0, None),
                "NULL arena")
    _expect_bad(lib.rfsn_rope_append(FAKE, FAKE, None, f32, FAKE, 0, 1, 32, 8, 1, 128, FAKE, FAKE, 0, 64, 0, None),
                "both")
    # (q, k, v, dtype, inv_freq, state, state copy, batch, heads, kv heads, len, d, q_out, arena, row0, capacity, stream)
    _expect_bad(lib.rfsn_rope_append_step(FAKE, FAKE, FAKE, f32, FAKE, None, None, 1, 32, 8, 1, 128, FAKE, FAKE, 0, 64,
                                          None), "NULL step state")
    _expect_bad(lib.rfsn_rope_append_step(FAKE, FAKE, FAKE, f32, FAKE, FAKE, None, 1, 32, 8, 1, 128, FAKE, None, 0, 64,
                                          None), "NULL arena")
    # (q, k, v, dtype, cos, sin, table dtype, inv_freq, pos0, batch, heads, kv heads, len, d, q_out, arena,
    #  row0, capacity, write index, stream)
    _expect_bad(lib.rfsn_rope_append_tables(FAKE, FAKE, FAKE, f32, FAKE, FAKE, f32, FAKE, 0, 1, 32, 8, 1, 128, FAKE,
                                            None, 0, 64, 0, None), "NULL arena")
    _expect_bad(lib.rfsn_rope_append_tables(FAKE, FAKE, FAKE, f32, FAKE, None, f32, FAKE, 0, 1, 32, 8, 1, 128, FAKE,
                                            FAKE, 0, 64, 0, None), "go together")
    _expect_bad(lib.rfsn_rope_append_tables(FAKE, FAKE, FAKE, f32, None, None, f32, None, 0, 1, 32, 8, 1, 128, FAKE,
                                            FAKE, 0, 64, 0, None), "no tables and no inv_freq")
    _expect_bad(lib.rfsn_rope_append_tables(FAKE, None, FAKE, f32, FAKE, FAKE, f32, FAKE, 0, 1, 32, 8, 1, 128, FAKE,
                                            FAKE, 0, 64, 0, None), "NULL q/k/v/q_out")
    _expect_bad(lib.rfsn_arena_copy_rows(None, 0, 0, 0, 0, 1, None), "NULL arena")
    _expect_bad(lib.rfsn_block_upload(None, 0, 1, FAKE, FAKE, None, None), "NULL arena")
    _expect_bad(lib.rfsn_block_download(None, 0, 1, FAKE, FAKE, None, None), "NULL arena")
    _expect_bad(lib.rfsn_event_wait(None, 1000), "NULL event")
    _expect_bad(lib.rfsn_workspace_check(None, None, 1000), "NULL workspace")
    dev = ctypes.c_void_p()
    _expect_bad(lib.rfsn_host_device_pointer(None, ctypes.byref(dev)), "NULL pointer")


def test_attention_arguments(lib):
    table, hot = native.PageTableC(), native.HotWindowC()
    _expect_bad(lib.rfsn_paged_attention(None, FAKE, 1, 32, 8, 1, 0, ctypes.byref(table), ctypes.byref(hot), FAKE,
                                         None, FAKE, 1 << 20, 0, None), "NULL arena")
    _expect_bad(lib.rfsn_paged_attention_noalloc(None, FAKE, 1, 32, 8, 1, 0, ctypes.byref(table), ctypes.byref(hot),
                                                 FAKE, None, 0, None), "rfsn_paged_attention")
    # (arena, q, batch, heads, kv heads, q_len, q_pos0, table, hot, peers, out, lse, workspace, bytes, splits, stream)
    _expect_bad(lib.rfsn_paged_attention_peer(FAKE, FAKE, 1, 32, 8, 1, 0, ctypes.byref(table), ctypes.byref(hot),
                                              None, FAKE, None, FAKE, 1 << 20, 0, None), "not connected")
    _expect_bad(lib.rfsn_lse_merge(None, FAKE, 2, 32, 128, FAKE, None, None), "rfsn_lse_merge")
    _expect_bad(lib.rfsn_lse_merge(FAKE, FAKE, 0, 32, 128, FAKE, None, None), "non-positive")
    n = ctypes.c_size_t()
    _expect_bad(lib.rfsn_attention_workspace_size(1, 32, 8, 1, 128, 0, None), "bytes is NULL")
    _expect_bad(lib.rfsn_attention_workspace_size(1, 32, 0, 1, 128, 0, ctypes.byref(n)), "rfsn_attention_workspace_size")
    with pytest.raises(ValueError, match="divisible"):
        native.check(lib.rfsn_attention_workspace_size(1, 32, 6, 1, 128, 0, ctypes.byref(n)), "workspace")


def test_model_op_arguments(lib):
    bf16 = native.RFSN_BF16
    _expect_bad(lib.rfsn_rms_norm(None, None, FAKE, None, FAKE, 1, 4096, bf16, 1e-5, None), "NULL pointer")
    _expect_bad(lib.rfsn_rms_norm(FAKE, FAKE, FAKE, None, FAKE, 1, 4096, bf16, 1e-5, None), "go together")
    _expect_bad(lib.rfsn_rms_norm(FAKE, None, FAKE, None, FAKE, 1, 0, bf16, 1e-5, None), "bad shape")
    _expect_bad(lib.rfsn_silu_mul(None, FAKE, 1, 14336, bf16, None), "NULL pointer")
    _expect_bad(lib.rfsn_silu_mul(FAKE, FAKE, 1, 14336, 9, None), "bad shape or dtype")
    _expect_bad(lib.rfsn_gemv(FAKE, FAKE, None, 4096, 4096, 1, bf16, None), "NULL pointer")
    _expect_bad(lib.rfsn_gemv(FAKE, FAKE, FAKE, 4096, 4096, 0, bf16, None), "rows of x")
    _expect_bad(lib.rfsn_gemv(FAKE, FAKE, FAKE, 4096, 4100, 1, bf16, None), "16-byte aligned")
    _expect_bad(lib.rfsn_gemv(FAKE + 4, FAKE, FAKE, 4096, 4096, 1, bf16, None), "16-byte aligned")
    _expect_bad(lib.rfsn_gemv(FAKE, FAKE, FAKE, 4096, 65536, 1, bf16, None), "shared memory")


def test_peer_group_arguments(lib):
    group, handle = ctypes.c_void_p(), ctypes.create_string_buffer(max(64, lib.rfsn_peer_ipc_handle_bytes()))
    _expect_bad(lib.rfsn_peer_group_create(2, 0, 8, 128, None, handle), "NULL output")
    _expect_bad(lib.rfsn_peer_group_create(0, 0, 8, 128, ctypes.byref(group), handle), "world 0")
    _expect_bad(lib.rfsn_peer_group_create(2, 2, 8, 128, ctypes.byref(group), handle), "rank 2")
    _expect_bad(lib.rfsn_peer_group_create(2, 0, 8, 126, ctypes.byref(group), handle), "bad shape")
    _expect_bad(lib.rfsn_peer_group_connect(None, handle), "NULL argument")
    _expect_bad(lib.rfsn_peer_group_set_timeout(None, 1000), "bad argument")
    assert group.value is None
