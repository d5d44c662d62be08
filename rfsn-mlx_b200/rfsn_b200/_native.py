"""ctypes binding of the C ABI in ``include/rfsn_b200.h``.

This is the only module that talks to ``librfsn_b200.so``. Tensors cross the
boundary as raw device pointers (``tensor.data_ptr()``) plus sizes; streams as
``torch.cuda.current_stream().cuda_stream``. Status codes become the exception
types the reference raises for the same condition (ValueError for bad
arguments, RuntimeError for overflow / device failures, TimeoutError for an
expired bounded wait).

There is no CPU fallback: if the library or a CUDA device is missing, every
compute call raises ``NativeUnavailable``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

import torch

_LIB_NAME = "librfsn_b200.so"
_LIB_PATH = Path(__file__).resolve().parent / _LIB_NAME

RFSN_OK = 0
RFSN_ERR_INVALID_ARG = 1
RFSN_ERR_UNSUPPORTED = 2
RFSN_ERR_OVERFLOW = 3
RFSN_ERR_TIMEOUT = 4
RFSN_ERR_CUDA = 5
RFSN_ERR_DEVICE = 6

RFSN_F32 = 0
RFSN_F16 = 1
RFSN_BF16 = 2
TILE_KEYS = 64

DTYPE_CODE = {torch.float32: RFSN_F32, torch.float16: RFSN_F16, torch.bfloat16: RFSN_BF16}

# Every symbol declared in include/rfsn_b200.h.
EXPORTED_SYMBOLS = (
    "rfsn_last_error",
    "rfsn_abi_version",
    "rfsn_device_sm_count",
    "rfsn_arena_create",
    "rfsn_arena_destroy",
    "rfsn_rope_append",
    "rfsn_rope_append_step",
    "rfsn_rope_append_tables",
    "rfsn_arena_copy_rows",
    "rfsn_block_upload",
    "rfsn_block_download",
    "rfsn_event_wait",
    "rfsn_attention_workspace_size",
    "rfsn_paged_attention",
    "rfsn_segmented_attention",
    "rfsn_lse_merge",
    "rfsn_workspace_check",
    "rfsn_launch_count",
    "rfsn_paged_attention_noalloc",
    "rfsn_noalloc_check",
    "rfsn_peer_ipc_handle_bytes",
    "rfsn_peer_group_create",
    "rfsn_peer_group_connect",
    "rfsn_peer_group_set_timeout",
    "rfsn_peer_group_destroy",
    "rfsn_paged_attention_peer",
    "rfsn_host_device_pointer",
    "rfsn_prefill_plan",
    "rfsn_rms_norm",
    "rfsn_silu_mul",
    "rfsn_gemv",
)


class NativeUnavailable(RuntimeError):
    """The CUDA library or device needed by the B200 path is not available."""


class PageTableC(ctypes.Structure):
    _fields_ = [
        ("records", ctypes.c_void_p),
        ("n_blocks", ctypes.c_int32),
        ("archived_tokens", ctypes.c_int32),
        ("archived_tiles", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class HotWindowC(ctypes.Structure):
    _fields_ = [
        ("ring_row0", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("head_index", ctypes.c_int32),
        ("length", ctypes.c_int32),
        ("start_pos", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("step_state", ctypes.c_void_p),  # optional device int32[8] (RFSN_STEP_*), read when the kernel runs
    ]


# Device step state layout (int32 indices), include/rfsn_b200.h RFSN_STEP_*
STEP_POS, STEP_WRITE_INDEX, STEP_HEAD, STEP_LENGTH, STEP_START, STEP_STATE_LEN = 0, 1, 2, 3, 4, 8


class SegmentDescC(ctypes.Structure):
    _fields_ = [
        ("k_ptr", ctypes.c_uint64),
        ("v_ptr", ctypes.c_uint64),
        ("k_stride_b", ctypes.c_int64),
        ("k_stride_h", ctypes.c_int64),
        ("k_stride_t", ctypes.c_int64),
        ("v_stride_b", ctypes.c_int64),
        ("v_stride_h", ctypes.c_int64),
        ("v_stride_t", ctypes.c_int64),
        ("pos", ctypes.c_int32),
        ("len", ctypes.c_int32),
        ("tile_begin", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_lib: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    return Path(os.environ.get("RFSN_B200_LIB", str(_LIB_PATH)))


def load_library() -> ctypes.CDLL:
    """Load the shared library (no CUDA device needed just to load it)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not path.exists():
        raise NativeUnavailable(
            f"{path} is missing; build it with `make -C rfsn-mlx_b200/csrc` (or __graft_entry__.build())"
        )
    lib = ctypes.CDLL(str(path))
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "rfsn_last_error": (ctypes.c_char_p, []),
        "rfsn_abi_version": (i32, []),
        "rfsn_device_sm_count": (i32, [ctypes.POINTER(i32)]),
        "rfsn_arena_create": (i32, [vp, vp, i32, i32, i32, i32, ctypes.POINTER(vp)]),
        "rfsn_arena_destroy": (i32, [vp]),
        "rfsn_rope_append": (i32, [vp, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp, i32, i32, i32, vp]),
        "rfsn_rope_append_step": (i32, [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, vp, vp, i32, i32, vp]),
        "rfsn_rope_append_tables": (i32, [vp, vp, vp, i32, vp, vp, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp, i32,
                                          i32, i32, vp]),
        "rfsn_host_device_pointer": (i32, [vp, ctypes.POINTER(ctypes.c_void_p)]),
        "rfsn_prefill_plan": (i32, [i32] * 8 + [ctypes.POINTER(ctypes.c_int)] * 3),
        "rfsn_rms_norm": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, ctypes.c_float, vp]),
        "rfsn_silu_mul": (i32, [vp, vp, i32, i32, i32, vp]),
        "rfsn_gemv": (i32, [vp, vp, vp, i32, i32, i32, i32, vp]),
        "rfsn_arena_copy_rows": (i32, [vp, i32, i32, i32, i32, i32, vp]),
        "rfsn_block_upload": (i32, [vp, i32, i32, vp, vp, vp, vp]),
        "rfsn_block_download": (i32, [vp, i32, i32, vp, vp, vp, vp]),
        "rfsn_event_wait": (i32, [vp, i64]),
        "rfsn_attention_workspace_size": (i32, [i32, i32, i32, i32, i32, i32, ctypes.POINTER(sz)]),
        "rfsn_paged_attention": (
            i32,
            [vp, vp, i32, i32, i32, i32, i32, ctypes.POINTER(PageTableC), ctypes.POINTER(HotWindowC), vp, vp, vp, sz, i32, vp],
        ),
        "rfsn_segmented_attention": (
            i32,
            [vp, i32, i32, i32, i32, i32, i32, i32, vp, i32, i32, vp, vp, vp, sz, i32, vp],
        ),
        "rfsn_lse_merge": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "rfsn_workspace_check": (i32, [vp, vp, i64]),
        "rfsn_launch_count": (ctypes.c_uint64, []),
        "rfsn_peer_ipc_handle_bytes": (i32, []),
        "rfsn_peer_group_create": (i32, [i32, i32, i32, i32, ctypes.POINTER(vp), vp]),
        "rfsn_peer_group_connect": (i32, [vp, vp]),
        "rfsn_peer_group_set_timeout": (i32, [vp, i64]),
        "rfsn_peer_group_destroy": (i32, [vp]),
        "rfsn_paged_attention_peer": (
            i32,
            [vp, vp, i32, i32, i32, i32, i32, ctypes.POINTER(PageTableC), ctypes.POINTER(HotWindowC), vp, vp, vp, vp,
             sz, i32, vp],
        ),
        "rfsn_paged_attention_noalloc": (
            i32,
            [vp, vp, i32, i32, i32, i32, i32, ctypes.POINTER(PageTableC), ctypes.POINTER(HotWindowC), vp, vp, i32, vp],
        ),
        "rfsn_noalloc_check": (i32, [vp, i64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


_device_seen = False


def lib() -> ctypes.CDLL:
    """The loaded library, after checking (once per process) that a CUDA device is visible."""
    global _device_seen
    lib_ = load_library()
    if not _device_seen:
        if not torch.cuda.is_available():
            raise NativeUnavailable("the B200 attention path needs a CUDA device; none is visible")
        _device_seen = True
    return lib_


def launch_count() -> int:
    """Kernels launched by the native library so far in this process."""
    return int(load_library().rfsn_launch_count())


def last_error() -> str:
    return load_library().rfsn_last_error().decode("utf-8", "replace")


def check(status: int, what: str) -> None:
    if status == RFSN_OK:
        return
    msg = last_error()
    if status == RFSN_ERR_INVALID_ARG:
        raise ValueError(f"{what}: {msg}")
    if status == RFSN_ERR_TIMEOUT:
        raise TimeoutError(f"{what}: {msg}")
    if status == RFSN_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg}")


_raw_current_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_current_device = getattr(torch._C, "_cuda_getDevice", None)


def stream_ptr(stream: Optional[torch.cuda.Stream] = None) -> int:
    """cudaStream_t of ``stream``, else of the current stream of the current
    device (one call into torch's C layer: this runs on every decode step)."""
    if stream is not None:
        return int(stream.cuda_stream)
    if _raw_current_stream is not None and _current_device is not None:
        return int(_raw_current_stream(_current_device()))
    return int(torch.cuda.current_stream().cuda_stream)


def host_device_pointer(t: torch.Tensor) -> int:
    """Device address of a pinned CPU tensor's data, for kernels that read or
    write it across the bus; raises ValueError when it is not page-locked
    memory mapped for the current device."""
    if t.device.type != "cpu" or not t.is_pinned():
        raise ValueError("expected a pinned CPU tensor")
    out = ctypes.c_void_p()
    status = lib().rfsn_host_device_pointer(t.data_ptr(), ctypes.byref(out))
    if status != RFSN_OK or not out.value:
        raise ValueError(f"pinned tensor is not mapped for the device: {last_error()}")
    return int(out.value)


def prefill_plan(batch: int, q_heads: int, kv_heads: int, q_len: int, q_pos0: int, archived_tokens: int,
                 hot_start: int, hot_length: int) -> tuple[int, int, int]:
    """(units run whole, key-range splits of the later units, CTAs) of a
    tensor-core prefill call of this shape (``rfsn_prefill_plan``)."""
    whole, splits, ctas = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(load_library().rfsn_prefill_plan(batch, q_heads, kv_heads, q_len, q_pos0, archived_tokens, hot_start,
                                           hot_length, ctypes.byref(whole), ctypes.byref(splits), ctypes.byref(ctas)),
          "rfsn_prefill_plan")
    return whole.value, splits.value, ctas.value


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype {dtype}") from exc


class Arena:
    """Owns the native descriptor (incl. TMA maps) of one layer's K/V arena."""

    def __init__(self, k: torch.Tensor, v: torch.Tensor) -> None:
        if k.shape != v.shape or k.dtype != v.dtype or k.dim() != 3:
            raise ValueError("arena K/V must be matching [groups, rows, head_dim] tensors")
        if not (k.is_cuda and k.is_contiguous() and v.is_contiguous()):
            raise ValueError("arena K/V must be contiguous CUDA tensors")
        self.k, self.v = k, v
        self.groups, self.rows, self.head_dim = (int(x) for x in k.shape)
        self.dtype = k.dtype
        handle = ctypes.c_void_p()
        check(
            lib().rfsn_arena_create(
                k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), self.groups, self.rows, self.head_dim,
                ctypes.byref(handle),
            ),
            "rfsn_arena_create",
        )
        self.handle = handle

    def close(self) -> None:
        if self.handle:
            _lib.rfsn_arena_destroy(self.handle)  # type: ignore[union-attr]
            self.handle = ctypes.c_void_p()

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def workspace_bytes(batch: int, q_heads: int, kv_heads: int, q_len: int, head_dim: int, max_splits: int = 0) -> int:
    out = ctypes.c_size_t()
    check(
        load_library().rfsn_attention_workspace_size(batch, q_heads, kv_heads, q_len, head_dim, max_splits, ctypes.byref(out)),
        "rfsn_attention_workspace_size",
    )
    return int(out.value)


class Workspace:
    """Zero-initialised device scratch for the split-KV attention kernels.

    The kernels leave their arrival counters at zero after every call, so a
    workspace is zeroed once and reused by calls ordered on one stream. It
    grows when a call needs more room.
    """

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.buf = torch.zeros(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 2 * self.buf.numel()), dtype=torch.uint8, device=self.device)
        return self.buf

    def check(self, timeout_s: float = 10.0) -> None:
        if self.buf.numel():
            check(
                lib().rfsn_workspace_check(self.buf.data_ptr(), stream_ptr(), int(timeout_s * 1e6)),
                "rfsn_workspace_check",
            )


_workspaces: dict[int, Workspace] = {}


def default_workspace(device: torch.device) -> Workspace:
    """The per-device workspace of calls that pass none. Its arrival counters
    are shared, so attention calls that may run concurrently (on different
    streams) must each pass their own ``Workspace``."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None:
        ws = Workspace(torch.device("cuda", idx))
        _workspaces[idx] = ws
    return ws
