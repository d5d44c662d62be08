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

from typing import Optional, Tuple

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


def attention_step_tables(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cache: LayerKVCache, start_pos: int,
                          rope_tables=None) -> torch.Tensor:
    """``attention_step`` with the RoPE of a stand-alone layer call
    (layer.py:118-135): the given (cos, sin) tables, or tables built in the
    model dtype when ``rope_tables`` is None, with the reference's per-op
    rounding. Returns the float32 attention output [B, H, L, D]."""
    seq_len = int(k.shape[2])
    cache.evict_for_append(seq_len)
    q_rot = cache.append_rope_tables(q, k, v, start_pos, rope_tables)
    if seq_len == 1:
        cache.maybe_prefetch_for_decode(start_pos)
    segments = cache.get_attention_segments()
    return paged_attention(cache, q_rot, start_pos, segments)


def capture_graph(fn, stream: torch.cuda.Stream) -> torch.cuda.CUDAGraph:
    """Capture ``fn()`` into a new CUDA graph on ``stream``. Unlike the
    ``torch.cuda.graph`` context manager this runs no garbage collection or
    cache release first, which would cost tens to hundreds of milliseconds at
    every re-capture of a decode step."""
    graph = torch.cuda.CUDAGraph()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        graph.capture_begin()
        try:
            fn()
        finally:
            graph.capture_end()
    torch.cuda.current_stream().wait_stream(stream)
    return graph


class GraphedDecodeStep:
    """One decode token of one layer, host buffers in and out, as one CUDA graph.

    Fill ``q_host`` [B, H, 1, D], ``k_host`` / ``v_host`` [B, Hkv, 1, D]
    (pinned, cache dtype) and call ``step(pos)``: the host runs the cache
    bookkeeping of ``attention_step`` (seal rule, append counters, prefetch
    hook, segment walk), writes the step state, and replays a graph of two
    kernels: the fused RoPE/append reads the step state, q, k and v straight
    from the pinned staging buffer across the bus (no copy operation) and
    leaves a device copy of the state, and the paged decode kernel reads that
    state and writes the float32 output straight into the pinned
    ``out_host``, which is returned after the step completes. The graph is captured again when the
    page table or the arena changes; when archived blocks are cold or a
    prefetch is in flight the step runs ``attention_step`` op by op instead.
    Needs bf16/f16 K/V, head_dim 128 and <= 4 query heads per KV head (the
    tensor-core decode kernel)."""

    def __init__(self, cache: LayerKVCache, q_heads: int) -> None:
        from . import _native as native

        self.cache = cache
        B, Hkv, D = cache.batch_size, cache.num_kv_heads, cache.config.head_dim
        self.shape_q = (B, q_heads, 1, D)
        shape_kv = (B, Hkv, 1, D)
        self.supported = (cache.dtype in (torch.bfloat16, torch.float16) and D == 128 and q_heads % Hkv == 0
                          and q_heads // Hkv <= 4)
        dev = cache.device
        es = torch.empty((), dtype=cache.dtype).element_size()
        align = lambda n: (n + 255) // 256 * 256  # noqa: E731
        n_state = align(4 * native.STEP_STATE_LEN)
        n_q = align(B * q_heads * D * es)
        n_kv = align(B * Hkv * D * es)
        total = n_state + n_q + 2 * n_kv
        self.stage_host = torch.zeros(total, dtype=torch.uint8).pin_memory()

        def views(buf):
            st = buf[:4 * native.STEP_STATE_LEN].view(torch.int32)
            o = n_state
            q = buf[o:o + B * q_heads * D * es].view(cache.dtype).view(self.shape_q)
            o += n_q
            k = buf[o:o + B * Hkv * D * es].view(cache.dtype).view(shape_kv)
            o += n_kv
            v = buf[o:o + B * Hkv * D * es].view(cache.dtype).view(shape_kv)
            return st, q, k, v

        self.state_host, self.q_host, self.k_host, self.v_host = views(self.stage_host)
        self._state_np = self.state_host.numpy()  # element writes without torch indexing
        self.state_dev = torch.zeros(native.STEP_STATE_LEN, dtype=torch.int32, device=dev)
        self.out_host = torch.zeros(self.shape_q, dtype=torch.float32).pin_memory()
        # device addresses of the pinned buffers (the kernels read and write them across the bus)
        base = native.host_device_pointer(self.stage_host) if self.supported else 0
        self._dptr_state, self._dptr_q = base, base + n_state
        self._dptr_k, self._dptr_v = base + n_state + n_q, base + n_state + n_q + n_kv
        self.workspace = native.Workspace(dev)
        self.workspace.get(native.workspace_bytes(B, q_heads, Hkv, 1, D, 0))
        # rotated q: allocated here, so a capture allocates nothing (a device
        # allocation inside a capture can cost tens of milliseconds)
        self.q_rot = torch.empty(self.shape_q, dtype=torch.float32, device=dev)
        self.stream = torch.cuda.Stream(device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.key = None
        self.replays = self.captures = self.fallbacks = 0
        self.graph_kernels = 0

    def _eligible(self) -> bool:
        c = self.cache
        return self.supported and not c.residency_manager.has_pending and c.all_blocks_resident()

    def _body(self, segs) -> torch.Tensor:
        from . import _native as native
        from .cache import paged_attention

        c = self.cache
        B, H, L, D = self.shape_q
        q_rot = self.q_rot
        native.check(
            native.lib().rfsn_rope_append_step(
                self._dptr_q, self._dptr_k, self._dptr_v, native.dtype_code(c.dtype), c.inv_freq().data_ptr(),
                self._dptr_state, self.state_dev.data_ptr(), B, H, c.num_kv_heads, 1, D, q_rot.data_ptr(),
                c.arena.handle, 0, c.config.hot_capacity, native.stream_ptr()),
            "rfsn_rope_append_step",
        )
        return paged_attention(c, q_rot, 0, segs, workspace=self.workspace, step_state=self.state_dev,
                               out=self.out_host)

    def step(self, pos: int) -> torch.Tensor:
        from . import _native as native

        c = self.cache
        if not self._eligible():
            self.fallbacks += 1
            out = attention_step(self.q_host.to(c.device, non_blocking=True),
                                 self.k_host.to(c.device, non_blocking=True),
                                 self.v_host.to(c.device, non_blocking=True), c, pos)
            self.out_host.copy_(out, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            return self.out_host
        # attention_step's host part for one token (layer.py:134-139)
        c.evict_for_append(1)
        write_index = c.hot_write_index
        c._check_append(1)
        c.hot_seq_len += 1
        c.maybe_prefetch_for_decode(pos)
        segs = c.get_attention_segments()
        head, hlen, hstart = segs.hot_state
        st = self._state_np
        st[0], st[1], st[2], st[3], st[4] = pos, write_index, head, hlen, hstart
        key = (c.arena.handle.value, c._arena_k.data_ptr(),
               (segs.table[0].data_ptr(),) + tuple(segs.table[1:]) if segs.table is not None else None)
        if key != self.key or self.graph is None:
            # run this step op by op on the side stream first (the warm-up a
            # capture wants; it also produces this step's result), then capture
            self.stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.stream):
                self._body(segs)
            torch.cuda.current_stream().wait_stream(self.stream)
            self.graph = None
            before = native.launch_count()
            graph = capture_graph(lambda: self._body(segs), self.stream)
            self.graph_kernels = native.launch_count() - before  # this library's kernels per replay
            self.graph, self.key = graph, key
            self.captures += 1
            torch.cuda.current_stream().synchronize()
            return self.out_host
        self.graph.replay()
        self.replays += 1
        torch.cuda.current_stream().synchronize()
        return self.out_host


def __getattr__(name: str):
    """The reference's ``layer`` module also holds the layer and its RMS norm
    (``RFSNLayerMLX``, ``RFSNLayerNorm``); they live in ``model`` here and
    are resolved on first use (``model`` imports this module)."""
    if name in ("RFSNLayerMLX", "RFSNLayerNorm", "RFSNLayer"):
        from . import model

        return getattr(model, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
