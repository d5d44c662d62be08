"""Exact attention entry points (drop-in for ``rfsn_v10_5.attention_exact``).

Same functions, arguments, semantics and errors as the reference
(attention_exact.py:24-195): scaled dot products with scale 1/sqrt(D),
additive-causal masking by absolute positions (key pos <= query pos), one
softmax over all segments, float32 accumulation, result cast to q's dtype.

Both the single-segment path (``run_exact_attention``; MLX's fused SDPA in
the reference) and the multi-segment path (``run_segmented_attention``; two
fp32 passes in the reference) run one split-KV CUDA kernel:

* segments coming from ``LayerKVCache.get_*_attention_segments`` carry the
  layer's device page table and go to ``rfsn_paged_attention`` (TMA-streamed
  tiles, tensor-core contraction) without materialising per-segment tensors;
* any other list of CUDA tensors is described to ``rfsn_segmented_attention``
  by address and strides.

K/V segments may carry fewer heads than q (GQA); query head h then reads KV
head h // (H / Hkv), which is what the reference's ``mx.repeat`` expansion
(layer.py:140-150) produces, so pre-expanded and compact segments agree.
"""

from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import numpy as np
import torch

from . import _native as native
from .cache import PagedSegments, paged_attention

AttentionSegment = Tuple[torch.Tensor, torch.Tensor, int]


def build_causal_mask(q_len: int, k_len: int, q_start_pos: int, k_start_pos: int, *, device=None) -> torch.Tensor:
    """attention_exact.py:27-61: float32 (1, 1, q_len, k_len), 0 allowed / -1e9 masked."""
    q_pos = torch.arange(q_start_pos, q_start_pos + q_len, device=device)[:, None]
    k_pos = torch.arange(k_start_pos, k_start_pos + k_len, device=device)[None, :]
    mask = torch.where(k_pos <= q_pos, 0.0, -1e9).to(torch.float32)
    return mask[None, None]


def _segment_table(segments: Sequence[AttentionSegment], batch: int, head_dim: int, device: torch.device):
    descs = (native.SegmentDescC * len(segments))()
    dtype = None
    kv_heads = None
    tile = 0
    keep: List[torch.Tensor] = []
    for i, (k, v, start) in enumerate(segments):
        if k.dim() != 4 or k.shape != v.shape:
            raise ValueError("each segment must be (k, v, start) with k, v shaped [B, Hkv, n, D]")
        if k.shape[0] != batch or k.shape[3] != head_dim:
            raise ValueError(f"segment {i} shape {tuple(k.shape)} does not match q (batch {batch}, head_dim {head_dim})")
        if kv_heads is None:
            kv_heads, dtype = int(k.shape[1]), k.dtype
        if int(k.shape[1]) != kv_heads or k.dtype != dtype or v.dtype != dtype:
            raise ValueError("all segments must share kv head count and dtype")
        if not (k.is_cuda and v.is_cuda):
            raise ValueError("segments must be CUDA tensors")
        if k.stride(3) != 1:
            k = k.contiguous()
        if v.stride(3) != 1:
            v = v.contiguous()
        keep += [k, v]
        n = int(k.shape[2])
        if n <= 0:
            raise ValueError(f"segment {i} is empty")
        d = descs[i]
        d.k_ptr, d.v_ptr = k.data_ptr(), v.data_ptr()
        d.k_stride_b, d.k_stride_h, d.k_stride_t = k.stride(0), k.stride(1), k.stride(2)
        d.v_stride_b, d.v_stride_h, d.v_stride_t = v.stride(0), v.stride(1), v.stride(2)
        d.pos, d.len, d.tile_begin = int(start), n, tile
        tile += (n + native.TILE_KEYS - 1) // native.TILE_KEYS
    raw = np.frombuffer(bytes(descs), dtype=np.uint8)
    dev = torch.from_numpy(raw.copy()).to(device)
    return dev, kv_heads, dtype, tile, keep


def segmented_attention(q: torch.Tensor, segments: Sequence[AttentionSegment], q_start_pos: int,
                        *, want_lse: bool = False, max_splits: int = 0):
    """float32 result (and optionally the natural-log LSE) of exact attention
    of q [B, H, Lq, D] over arbitrary CUDA K/V segments."""
    if len(segments) == 0:
        raise RuntimeError("run_segmented_attention requires at least one KV segment")
    if q.dim() != 4:
        raise ValueError("q must be [B, H, Lq, D]")
    device = segments[0][0].device
    qf = q.to(device=device, dtype=torch.float32).contiguous()
    B, H, Lq, D = (int(x) for x in qf.shape)
    table, kv_heads, dtype, tiles, keep = _segment_table(segments, B, D, device)
    if H % kv_heads != 0:
        raise ValueError(f"num_heads ({H}) must be divisible by num_kv_heads ({kv_heads})")
    out = torch.empty((B, H, Lq, D), dtype=torch.float32, device=device)
    lse = torch.empty((B, H, Lq), dtype=torch.float32, device=device) if want_lse else None
    ws = native.default_workspace(device)
    buf = ws.get(native.workspace_bytes(B, H, kv_heads, Lq, D, max_splits))
    native.check(
        native.lib().rfsn_segmented_attention(
            qf.data_ptr(), B, H, kv_heads, Lq, int(q_start_pos), D, native.dtype_code(dtype), table.data_ptr(),
            len(segments), tiles, out.data_ptr(), lse.data_ptr() if lse is not None else None, buf.data_ptr(),
            buf.numel(), max_splits, native.stream_ptr(),
        ),
        "rfsn_segmented_attention",
    )
    del keep
    return (out, lse) if want_lse else out


def run_exact_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_start_pos: int, k_start_pos: int) -> torch.Tensor:
    """attention_exact.py:64-108."""
    out = segmented_attention(q, [(k, v, k_start_pos)], q_start_pos)
    return out if q.dtype == torch.float32 else out.to(q.dtype)


def exact_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_start_pos: int, k_start_pos: int) -> torch.Tensor:
    """attention_exact.py:111-119."""
    return run_exact_attention(q, k, v, q_start_pos, k_start_pos)


def run_segmented_attention(q: torch.Tensor, segments: Sequence[AttentionSegment], q_start_pos: int) -> torch.Tensor:
    """attention_exact.py:122-164 (one segment: the exact path, :135-137)."""
    if len(segments) == 0:
        raise RuntimeError("run_segmented_attention requires at least one KV segment")
    if isinstance(segments, PagedSegments):
        out = paged_attention(segments.cache, q, q_start_pos, segments)
    else:
        out = segmented_attention(q, segments, q_start_pos)
    return out if q.dtype == torch.float32 else out.to(q.dtype)


def exact_prefill_attention(q, k, v, q_start_pos: int, k_start_pos: int) -> torch.Tensor:
    """attention_exact.py:167-178."""
    return run_exact_attention(q, k, v, q_start_pos, k_start_pos)


def exact_decode_attention(q, k, v, q_abs_pos: int, k_start_pos: int) -> torch.Tensor:
    """attention_exact.py:181-195."""
    return run_exact_attention(q, k, v, q_abs_pos, k_start_pos)


__all__ = [
    "AttentionSegment",
    "build_causal_mask",
    "run_exact_attention",
    "exact_attention",
    "run_segmented_attention",
    "exact_prefill_attention",
    "exact_decode_attention",
    "segmented_attention",
]

del ctypes
