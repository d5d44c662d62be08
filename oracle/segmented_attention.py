"""Exact segmented attention, restated in numpy float32 (test infrastructure).

Follows ``rfsn_v10_5/attention_exact.py`` of the reference:

* ``build_causal_mask``      -> attention_exact.py:27-61 (0 / -1e9 additive,
  by absolute positions, float32, shape (1, 1, q_len, k_len)).
* ``run_segmented_attention`` -> attention_exact.py:122-164 (empty list raises
  RuntimeError; one segment goes to the exact path; otherwise float32 logits per
  segment, one global max over all segments, then
  sum(exp(logits - max) @ v) / max(sum(exp(logits - max)), 1e-9), cast to
  q's dtype).
* ``run_exact_attention``     -> attention_exact.py:64-108: MLX's fused SDPA
  with scale 1/sqrt(D) and the same mask; restated as the same two-pass
  formula over a single segment, which is what that fused kernel computes.
* GQA expansion               -> layer.py:140-150 (``mx.repeat`` of each K/V
  segment by ``kv_groups`` on the head axis, so query head h reads KV head
  h // groups). The reference does this in the layer before calling the
  attention; here it is done inside when K/V carry fewer heads than q.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np

Segment = Tuple[np.ndarray, np.ndarray, int]


def build_causal_mask(q_len: int, k_len: int, q_start_pos: int, k_start_pos: int) -> np.ndarray:
    """attention_exact.py:27-61."""
    q_positions = np.arange(q_start_pos, q_start_pos + q_len)[:, None]
    k_positions = np.arange(k_start_pos, k_start_pos + k_len)[None, :]
    mask = np.where(k_positions <= q_positions, 0.0, -1e9).astype(np.float32)
    return mask[None, None, :, :]


def _expand_gqa(x: np.ndarray, num_heads: int) -> np.ndarray:
    """layer.py:140-150: repeat each KV head ``groups`` times on axis 1."""
    groups = num_heads // x.shape[1]
    if groups == 1:
        return x
    return np.repeat(x, groups, axis=1)


def run_segmented_attention(
    q: np.ndarray,
    segments: Sequence[Segment],
    q_start_pos: int,
    *,
    return_lse: bool = False,
    grouped: bool = False,
    q_positions=None,
):
    """attention_exact.py:122-164 (with the single-segment branch of :135-137).

    ``q`` is (B, H, Lq, D) float32 (the reference's q is float32 after RoPE
    promotion, layer.py:131-132). Segment K/V are float arrays (already decoded
    from their storage dtype) shaped (B, Hkv, n, D) with H % Hkv == 0.
    With ``return_lse`` the natural-log log-sum-exp of the scaled, masked
    logits, shape (B, H, Lq), is returned too (used to check split merges).
    ``grouped=True`` evaluates the same formula without materialising the GQA
    repeat (each KV head's query group is stacked along the query axis), which
    keeps 128K-token cases within memory.
    ``q_positions`` (grouped evaluation) gives each query row its own absolute
    position instead of ``q_start_pos + row``: sampled rows of a long chunk are
    checked without evaluating every row. The mask rule is the same (key
    position <= query position, build_causal_mask).
    """
    if not segments:
        raise RuntimeError("run_segmented_attention requires at least one KV segment")
    if grouped or q_positions is not None:
        return _grouped(q, segments, q_start_pos, return_lse, q_positions)
    q_f32 = np.asarray(q, dtype=np.float32)
    num_heads = q_f32.shape[1]
    scale = np.float32(1.0 / (q_f32.shape[-1] ** 0.5))

    global_max = None
    segment_logits = []
    for k, v, k_start in segments:
        k32 = _expand_gqa(np.asarray(k, dtype=np.float32), num_heads)
        v32 = _expand_gqa(np.asarray(v, dtype=np.float32), num_heads)
        logits = np.matmul(q_f32, np.swapaxes(k32, -1, -2)) * scale
        logits = logits + build_causal_mask(q_f32.shape[2], k32.shape[2], q_start_pos, k_start)
        segment_logits.append((logits, v32))
        local_max = logits.max(axis=-1, keepdims=True)
        global_max = local_max if global_max is None else np.maximum(global_max, local_max)

    numerator = None
    denominator = None
    for logits, v32 in segment_logits:
        weights = np.exp(logits - global_max)
        weighted_v = np.matmul(weights, v32)
        weight_sum = weights.sum(axis=-1, keepdims=True)
        numerator = weighted_v if numerator is None else numerator + weighted_v
        denominator = weight_sum if denominator is None else denominator + weight_sum

    out = (numerator / np.maximum(denominator, np.float32(1e-9))).astype(np.float32)
    if return_lse:
        lse = (global_max + np.log(denominator))[..., 0]
        return out, lse.astype(np.float32)
    return out


def _grouped(q: np.ndarray, segments: Sequence[Segment], q_start_pos: int, return_lse: bool, q_positions=None):
    q_f32 = np.asarray(q, dtype=np.float32)
    B, H, Lq, D = q_f32.shape
    Hkv = segments[0][0].shape[1]
    G = H // Hkv
    qg = q_f32.reshape(B, Hkv, G * Lq, D)
    scale = np.float32(1.0 / (D ** 0.5))
    logits_all = []
    global_max = None
    for k, v, k_start in segments:
        k32 = np.asarray(k, dtype=np.float32)
        logits = np.matmul(qg, np.swapaxes(k32, -1, -2)) * scale
        if q_positions is None:
            mask = build_causal_mask(Lq, k32.shape[2], q_start_pos, k_start)
        else:
            k_positions = np.arange(k_start, k_start + k32.shape[2])[None, :]
            qp = np.asarray(q_positions, dtype=np.int64)[:, None]
            mask = np.where(k_positions <= qp, 0.0, -1e9).astype(np.float32)[None, None]
        logits = logits + np.tile(mask, (1, 1, G, 1))
        local_max = logits.max(axis=-1, keepdims=True)
        global_max = local_max if global_max is None else np.maximum(global_max, local_max)
        logits_all.append((logits, v))
    num = None
    den = None
    for logits, v in logits_all:
        w = np.exp(logits - global_max)
        wv = np.matmul(w, np.asarray(v, dtype=np.float32))
        ws = w.sum(axis=-1, keepdims=True)
        num = wv if num is None else num + wv
        den = ws if den is None else den + ws
    out = (num / np.maximum(den, np.float32(1e-9))).astype(np.float32).reshape(B, H, Lq, D)
    if return_lse:
        lse = (global_max + np.log(den))[..., 0].reshape(B, H, Lq).astype(np.float32)
        return out, lse
    return out


def run_exact_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, q_start_pos: int, k_start_pos: int) -> np.ndarray:
    """attention_exact.py:64-108 (one contiguous K/V segment)."""
    return run_segmented_attention(q, [(k, v, k_start_pos)], q_start_pos)


def merge_partials(outs: Sequence[np.ndarray], lses: Sequence[np.ndarray]) -> np.ndarray:
    """Combine attention results over disjoint key sets by log-sum-exp.

    Given per-part outputs O_r (normalised) and natural-log LSE_r, the exact
    result over the union is sum_r exp(LSE_r - LSE*) O_r / sum_r exp(LSE_r - LSE*).
    This is the associative form of the global-max merge at
    attention_exact.py:141-164, used to check sharded/split results.
    """
    lse_stack = np.stack([np.asarray(x, dtype=np.float64) for x in lses])
    m = lse_stack.max(axis=0)
    w = np.exp(lse_stack - m)
    num = sum(wi[..., None] * np.asarray(o, dtype=np.float64) for wi, o in zip(w, outs))
    return (num / w.sum(axis=0)[..., None]).astype(np.float32)
