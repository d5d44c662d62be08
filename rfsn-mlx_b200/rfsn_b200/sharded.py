"""Context-sharded exact decode attention over the GPUs of one node.

The reference has no parallelism. Long contexts shard naturally by archived
block: attention over the segment list is an associative merge of per-part
(max, sum, output) states (attention_exact.py:141-164 is that merge done in
two passes). Rank r of P holds the archived blocks
[r * N / P, (r + 1) * N / P) of each layer in its own HBM and the last rank
also holds the hot window; no rank reads another rank's K/V.

A decode step on every rank: rotate q (the rank that owns the hot window also
appends the new token's K/V), attend over the local blocks with the paged
kernel, which also returns the natural-log LSE of each query row, all-gather
the (output, LSE) pairs (fp32, ~16.6 KB per rank for 32 heads x 128) with
NCCL, and combine them in rank order with ``rfsn_lse_merge``.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _native as native
from .cache import LayerKVCache


def shard_range(n_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) owned by ``rank`` (page-table order)."""
    return n_blocks * rank // world, n_blocks * (rank + 1) // world


def gather_parts(out: torch.Tensor, lse: torch.Tensor, group: Optional[dist.ProcessGroup] = None):
    """All-gather every rank's (out [B,H,Lq,D], lse [B,H,Lq]) in rank order.

    Returns (parts_out [P, rows, D], parts_lse [P, rows]) with rows = B*H*Lq.
    One collective of P x rows x (D + 1) float32 values: the output and LSE
    of a rank travel packed in one buffer.
    """
    world = dist.get_world_size(group)
    B, H, Lq, D = out.shape
    rows = B * H * Lq
    packed = torch.cat([out.reshape(-1).float(), lse.reshape(-1).float()])
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world, packed.numel()), dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(gathered, packed, group=group)
    else:
        chunks = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(chunks, packed, group=group)
        gathered = torch.stack(chunks)
    return gathered[:, : rows * D].reshape(world, rows, D), gathered[:, rows * D:].reshape(world, rows)


def merge_parts(parts_out: torch.Tensor, parts_lse: torch.Tensor, shape) -> torch.Tensor:
    """LSE-merge gathered parts on the device (rfsn_lse_merge, rank order)."""
    world, rows, D = parts_out.shape
    po, pl = parts_out.contiguous(), parts_lse.contiguous()
    merged = torch.empty(shape, dtype=torch.float32, device=po.device)
    native.check(
        native.lib().rfsn_lse_merge(po.data_ptr(), pl.data_ptr(), world, rows, D, merged.data_ptr(), None,
                                    native.stream_ptr()),
        "rfsn_lse_merge",
    )
    return merged


def merge_across_ranks(out: torch.Tensor, lse: torch.Tensor, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather per-rank (out, lse) and LSE-merge them; every rank returns
    the merged result. With one rank (or no process group) this is the identity."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return out
    parts_out, parts_lse = gather_parts(out, lse, group)
    return merge_parts(parts_out, parts_lse, out.shape)


def sharded_decode_step(cache: LayerKVCache, q: torch.Tensor, k: Optional[torch.Tensor], v: Optional[torch.Tensor],
                        pos: int, *, owns_hot: bool, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """One decode token of one layer on this rank's shard; returns the merged
    float32 output [B, H, 1, D] on every rank."""
    if owns_hot:
        cache.evict_for_append(int(k.shape[2]))
        q_rot = cache.append_rope(q, k, v, pos)
    else:
        q_rot = cache.rope_query(q, pos)
    segments = cache.get_attention_segments()
    if len(segments) == 0:
        # a rank with nothing to attend contributes an empty part (lse = -inf)
        out = torch.zeros(q_rot.shape, dtype=torch.float32, device=q_rot.device)
        lse = torch.full(q_rot.shape[:3], float("-inf"), dtype=torch.float32, device=q_rot.device)
    else:
        out, lse = cache.attend(q_rot, pos, segments, want_lse=True)
    return merge_across_ranks(out, lse, group)
