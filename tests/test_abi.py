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


def test_struct_layouts_match_header():
    assert ctypes.sizeof(native.PageTableC) == 24
    assert ctypes.sizeof(native.HotWindowC) == 32
    assert ctypes.sizeof(native.SegmentDescC) == 80
