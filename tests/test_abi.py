"""The C-ABI library loads here (no GPU) and exports every declared symbol."""

import ctypes
import re
from pathlib import Path

import pytest

from rfsn_b200 import _native as native

HEADER = Path(__file__).resolve().parent.parent / "include" / "rfsn_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^RFSN_API\s+[\w\s\*]+?\b(rfsn_\w+)\s*\(", text, flags=re.M)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = native.load_library()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_error_string():
    lib = native.load_library()
    assert lib.rfsn_abi_version() == 1
    assert isinstance(native.last_error(), str)


def test_workspace_size_is_host_only_and_validates():
    n = native.workspace_bytes(1, 32, 8, 1, 128)
    assert n > 256
    with pytest.raises(ValueError, match="divisible"):
        native.workspace_bytes(1, 30, 8, 1, 128)


def test_workspace_size_follows_the_split_counts_the_kernels_choose():
    # decode: at most 2 CTAs per SM of the tensor-core kernel or 4 of the CUDA-core
    # one; a 2048-token prefill chunk: split parts of the tensor-core kernel
    assert native.workspace_bytes(1, 32, 8, 1, 128) < 4 << 20
    prefill = native.workspace_bytes(1, 32, 8, 2048, 128)
    assert prefill >= 4 * 148 * 128 * 129 * 4 and prefill < 64 << 20
    # an explicit split cap never asks for more
    assert native.workspace_bytes(1, 32, 8, 1, 128, 8) <= native.workspace_bytes(1, 32, 8, 1, 128)


def test_prefill_plan_fills_the_last_wave():
    chunk = 2048
    units = (chunk // 32) * 8  # 32 positions x 8 KV heads per unit
    for c in range(16):  # 32K prompt in 2048-token chunks, 4096-token hot ring
        nb = max(0, c - 1)
        whole, splits, ctas = native.prefill_plan(1, 32, 8, chunk, c * chunk, nb * chunk, nb * chunk, min(c + 1, 2) * chunk)
        assert 1 <= splits <= 4 and 0 <= whole <= units
        assert ctas == whole + (units - whole) * splits
        assert (units - whole) * splits <= 4 * 148 or splits == 1
        if c >= 4:  # near-equal units: 3 full waves run whole, the 68 of the last wave in halves
            assert (whole, splits) == (units - units % 148, 2), (c, whole, splits)
    assert native.prefill_plan(1, 32, 8, chunk, 0, 0, 0, chunk)[1] == 1  # first chunk: short units, no split
    # few units over a long context: every unit split
    whole, splits, ctas = native.prefill_plan(1, 16, 4, 320, 6000 + 512 - 320, 6000, 6000, 512)
    assert whole == 0 and splits > 1
    with pytest.raises(ValueError):
        native.prefill_plan(1, 30, 8, 64, 0, 0, 0, 64)


def test_struct_layouts_match_header():
    assert ctypes.sizeof(native.PageTableC) == 24
    assert ctypes.sizeof(native.HotWindowC) == 32
    assert ctypes.sizeof(native.SegmentDescC) == 80


def test_prefill_plan_invariants_over_random_shapes():
    """The planner's answer is always a launchable split: 1-4 parts per split
    unit, split units only at the end of the unit order, at most 4 parts per SM
    and one arrival counter per split unit, the same answer for the same shape."""
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=300, deadline=None, derandomize=True)
    @hyp.given(batch=st.integers(1, 2), kv_heads=st.sampled_from([1, 2, 4, 8]), G=st.sampled_from([1, 2, 4, 8, 16]),
               q_len=st.integers(64, 4096), archived=st.integers(0, 200_000), hot_len=st.integers(0, 8192),
               back=st.integers(0, 8192))
    def check(batch, kv_heads, G, q_len, archived, hot_len, back):
        hot_start = archived
        q_pos0 = hot_start + max(0, hot_len - min(back, hot_len))
        whole, splits, ctas = native.prefill_plan(batch, G * kv_heads, kv_heads, q_len, q_pos0, archived, hot_start,
                                                  hot_len)
        ppc = 128 // G
        units = -(-q_len // ppc) * batch * kv_heads
        assert 1 <= splits <= 4 and 0 <= whole <= units
        assert ctas == whole + (units - whole) * splits
        if splits > 1:
            assert units - whole >= 1
            assert (units - whole) * splits <= 4 * 148  # 148 SMs (the host-side default without a device)
            assert units - whole <= 16384
        else:
            assert ctas == units
        assert native.prefill_plan(batch, G * kv_heads, kv_heads, q_len, q_pos0, archived, hot_start,
                                   hot_len) == (whole, splits, ctas)

    check()
