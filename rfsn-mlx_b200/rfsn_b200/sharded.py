"""Context-sharded exact decode attention over the GPUs of one node.

The reference has no parallelism. Long contexts shard naturally by archived
block: attention over the segment list is an associative merge of per-part
(max, sum, output) states (attention_exact.py:141-164 is that merge done in
two passes). Rank r of P holds the archived blocks
[r * N / P, (r + 1) * N / P) of each layer in its own HBM and the last rank
also holds the hot window; no rank reads another rank's K/V.

A decode step on every rank: rotate q (the rank that owns the hot window also
appends the new token's K/V), attend over the local blocks, and combine the
ranks' (output, LSE) pairs in rank order. Two exchange paths:

* ``PeerGroup`` (default for the tensor-core decode shape): the merge is fused
  into the attention kernel. Each rank's mailbox is mapped into every peer
  with CUDA IPC; the last CTA of each KV head stores its part into every
  mailbox over NVLink, waits (bounded) for the peers' parts and merges them,
  so one kernel per step produces the merged result on every rank.
* NCCL: the paged kernel returns (output, LSE), ``gather_parts`` all-gathers
  them (fp32, ~16.6 KB per rank for 32 heads x 128) and ``rfsn_lse_merge``
  combines them.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _native as native
from .cache import LayerKVCache


def shard_range(n_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) owned by ``rank`` (page-table order)."""
    return n_blocks * rank // world, n_blocks * (rank + 1) // world


def balanced_shards(block_lens: list[int], hot_len: int, world: int) -> list[tuple[int, int]]:
    """Contiguous block ranges [lo, hi) per rank (page-table order) that
    balance tokens, counting the hot window on the last rank: each rank's
    range ends at the block boundary closest to its share of the total."""
    total = sum(block_lens) + hot_len
    cum = [0]
    for n in block_lens:
        cum.append(cum[-1] + n)
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        # boundary index b in [bounds[-1], len(block_lens)] with cum[b] closest to target
        best = bounds[-1]
        for b in range(bounds[-1], len(block_lens) + 1):
            if abs(cum[b] - target) < abs(cum[best] - target):
                best = b
        bounds.append(best)
    bounds.append(len(block_lens))
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


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


class PeerGroup:
    """NVLink mailboxes of one sharded layer shape (batch * kv_heads groups,
    head_dim) across the ranks of ``group`` (one process per GPU).

    Collective to construct and to close: every rank must create it, and
    closing waits on a barrier so no peer still writes into a mailbox that is
    being released."""

    def __init__(self, groups: int, head_dim: int, group: Optional[dist.ProcessGroup] = None,
                 timeout_s: float = 2.0) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        lib = native.lib()
        nbytes = lib.rfsn_peer_ipc_handle_bytes()
        mine = (ctypes.c_ubyte * nbytes)()
        handle = ctypes.c_void_p()
        native.check(lib.rfsn_peer_group_create(self.world, self.rank, groups, head_dim, ctypes.byref(handle), mine),
                     "rfsn_peer_group_create")
        self.handle = handle
        raw = bytes(mine)
        if self.world > 1:
            t = torch.tensor(list(raw), dtype=torch.uint8, device=torch.device("cuda", torch.cuda.current_device()))
            if dist.get_backend(group) == "nccl":
                out = torch.empty(self.world * nbytes, dtype=torch.uint8, device=t.device)
                dist.all_gather_into_tensor(out, t, group=group)
            else:  # gloo exchanges host tensors
                tc = t.cpu()
                parts = [torch.empty_like(tc) for _ in range(self.world)]
                dist.all_gather(parts, tc, group=group)
                out = torch.cat(parts)
            raw = bytes(out.cpu().numpy().tobytes())
        table = (ctypes.c_ubyte * len(raw)).from_buffer_copy(raw)
        native.check(lib.rfsn_peer_group_connect(self.handle, table), "rfsn_peer_group_connect")
        native.check(lib.rfsn_peer_group_set_timeout(self.handle, int(timeout_s * 1e6)), "rfsn_peer_group_set_timeout")
        if self.world > 1:
            dist.barrier(group=group)

    def close(self) -> None:
        if self.handle:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            native.lib().rfsn_peer_group_destroy(self.handle)
            self.handle = ctypes.c_void_p()


def sharded_decode_step(cache: LayerKVCache, q: torch.Tensor, k: Optional[torch.Tensor], v: Optional[torch.Tensor],
                        pos: int, *, owns_hot: bool, group: Optional[dist.ProcessGroup] = None,
                        peers: Optional[PeerGroup] = None) -> torch.Tensor:
    """One decode token of one layer on this rank's shard; returns the merged
    float32 output [B, H, 1, D] on every rank. With ``peers`` the merge is
    fused into the attention kernel (NVLink); otherwise it goes through NCCL."""
    if owns_hot:
        cache.evict_for_append(int(k.shape[2]))
        q_rot = cache.append_rope(q, k, v, pos)
    else:
        q_rot = cache.rope_query(q, pos)
    segments = cache.get_attention_segments()
    if peers is not None:
        from .cache import paged_attention

        return paged_attention(cache, q_rot, pos, segments, peers=peers)
    if len(segments) == 0:
        # a rank with nothing to attend contributes an empty part (lse = -inf)
        out = torch.zeros(q_rot.shape, dtype=torch.float32, device=q_rot.device)
        lse = torch.full(q_rot.shape[:3], float("-inf"), dtype=torch.float32, device=q_rot.device)
    else:
        out, lse = cache.attend(q_rot, pos, segments, want_lse=True)
    return merge_across_ranks(out, lse, group)


class GraphedShardedDecodeStep:
    """``sharded_decode_step`` with a peer group, host buffers in and out, as one
    CUDA graph replay per token on every rank.

    Fill ``q_host`` (and, on the hot-window owner, ``k_host`` / ``v_host``) and
    call ``step(pos)`` on every rank for every token, in the same order. The
    host runs this rank's cache bookkeeping (the owner's seal rule and append
    counters, the segment walk) and writes the step state; the graph applies
    RoPE (and the ring append on the owner) reading the pinned staging buffer
    across the bus, and runs the decode kernel that merges all ranks' parts
    over NVLink and writes the merged output into the pinned ``out_host``. A rank captures its graph again when
    its own page table or arena changes (a seal on the owner); the kernels'
    call stamps live on the device, so replays and re-captures stay matched
    across ranks. Needs bf16/f16 K/V, head_dim 128 and <= 4 query heads per KV
    head."""

    def __init__(self, cache: LayerKVCache, q_heads: int, *, owns_hot: bool, peers: PeerGroup) -> None:
        from .layer import GraphedDecodeStep  # staging layout and capture helper

        self.cache = cache
        self.owns_hot = owns_hot
        self.peers = peers
        self._inner = GraphedDecodeStep(cache, q_heads)  # buffers, workspace, stream
        self.q_host, self.k_host, self.v_host = self._inner.q_host, self._inner.k_host, self._inner.v_host
        self.out_host = self._inner.out_host
        self.stage_host = self._inner.stage_host  # what one replay copies in (step state + q/k/v)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.key = None
        self.replays = self.captures = 0
        self.graph_kernels = 0

    def _body(self, segs) -> torch.Tensor:
        from .cache import paged_attention

        c, inner = self.cache, self._inner
        B, H, L, D = inner.shape_q
        q_rot = inner.q_rot
        # the kernels read the pinned staging buffer and write the pinned output across the bus
        native.check(
            native.lib().rfsn_rope_append_step(
                inner._dptr_q, inner._dptr_k if self.owns_hot else None, inner._dptr_v if self.owns_hot else None,
                native.dtype_code(c.dtype), c.inv_freq().data_ptr(), inner._dptr_state, inner.state_dev.data_ptr(),
                B, H, c.num_kv_heads if self.owns_hot else 0, 1, D, q_rot.data_ptr(), c.arena.handle, 0,
                c.config.hot_capacity, native.stream_ptr()),
            "rfsn_rope_append_step",
        )
        return paged_attention(c, q_rot, 0, segs, workspace=inner.workspace, step_state=inner.state_dev,
                               peers=self.peers, out=self.out_host)

    def step(self, pos: int) -> torch.Tensor:
        from .layer import capture_graph

        c, inner = self.cache, self._inner
        if self.owns_hot:
            c.evict_for_append(1)
            write_index = c.hot_write_index
            c._check_append(1)
            c.hot_seq_len += 1
        else:
            write_index = 0
        segs = c.get_attention_segments()
        head, hlen, hstart = segs.hot_state if segs.hot_state is not None else (0, 0, c.hot_start)
        st = inner._state_np
        st[0], st[1], st[2], st[3], st[4] = pos, write_index, head, hlen, hstart
        key = (c.arena.handle.value, c._arena_k.data_ptr(),
               (segs.table[0].data_ptr(),) + tuple(segs.table[1:]) if segs.table is not None else None)
        if key != self.key or self.graph is None:
            # this token runs op by op on the side stream (it takes part in the peers'
            # exchange for this call), then the graph is captured without running it
            inner.stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(inner.stream):
                self._body(segs)
            torch.cuda.current_stream().wait_stream(inner.stream)
            self.graph = None
            before = native.launch_count()
            self.graph = capture_graph(lambda: self._body(segs), inner.stream)
            self.graph_kernels = native.launch_count() - before  # this library's kernels per replay
            self.key = key
            self.captures += 1
            torch.cuda.current_stream().synchronize()
            return self.out_host
        self.graph.replay()
        self.replays += 1
        torch.cuda.current_stream().synchronize()
        return self.out_host
