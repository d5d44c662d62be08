"""Attention step of a transformer layer (the hot part of
``rfsn_v10_5.layer.RFSNLayerMLX.__call__``, layer.py:131-162).

``attention_step`` performs, for one layer and one chunk of L tokens:
RoPE on q and k (layer.py:131-132), the seal rule (``evict_for_append``,
layer.py:134), the ring append (layer.py:135), the decode-time prefetch hook
(layer.py:136-137) and exact attention over archived blocks + hot window
(layer.py:139-162). RoPE and the append are one fused kernel; the GQA
expansion of layer.py:140-150 is not materialised (the attention kernel maps
query head h to KV head h // groups).
"""

from __future__ import annotations

from typing import Tuple

import numpy as np
import torch

from .cache import LayerKVCache, paged_attention


def build_rope_tables(head_dim: int, rope_base: float, seq_len: int, start_pos: int = 0,
                      dtype: torch.dtype = torch.float32, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """layer.py:20-35: float32 cos/sin tables [seq_len, head_dim] for positions
    start_pos .. start_pos + seq_len (freqs duplicated over both halves)."""
    half = head_dim // 2
    exponent = np.arange(0, half, dtype=np.float32) / np.float32(half)
    inv_freq = (np.float32(1.0) / np.power(np.float32(rope_base), exponent, dtype=np.float32)).astype(np.float32)
    positions = np.arange(start_pos, start_pos + seq_len, dtype=np.float64).astype(np.float32)
    freqs = torch.from_numpy(positions[:, None] * inv_freq[None, :])
    emb = torch.cat([freqs, freqs], dim=-1)
    cos_t, sin_t = torch.cos(emb).to(dtype), torch.sin(emb).to(dtype)
    if device is not None:
        cos_t, sin_t = cos_t.to(device), sin_t.to(device)
    return cos_t, sin_t


def attention_step(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache: LayerKVCache, start_pos: int) -> torch.Tensor:
    """q [B, H, L, D], k/v [B, Hkv, L, D] (pre-RoPE, any float dtype) at
    absolute positions start_pos .. start_pos + L. Returns the float32
    attention output [B, H, L, D]."""
    seq_len = int(k.shape[2])
    cache.evict_for_append(seq_len)
    q_rot = cache.append_rope(q, k, v, start_pos)
    if seq_len == 1:
        cache.maybe_prefetch_for_decode(start_pos)
    segments = cache.get_attention_segments()
    return paged_attention(cache, q_rot, start_pos, segments)
