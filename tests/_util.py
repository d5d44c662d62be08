"""Test helpers: seeded paged-attention layouts and golden-fixture access."""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from oracle.numerics import from_storage, to_storage

GOLDEN = Path(__file__).resolve().parent / "golden"
TILE = 64


def load_json(name: str):
    return json.loads((GOLDEN / name).read_text())


def golden_attention_cases():
    data = np.load(GOLDEN / "segattn_golden.npz")
    out = []
    for name in data["__cases__"]:
        name = str(name)
        B, Hq, Hkv, D, Lq, q_start, nseg = (int(x) for x in data[f"{name}/meta"])
        dtype = str(data[f"{name}/dtype"])
        starts = [int(x) for x in data[f"{name}/starts"]]
        segs = [(data[f"{name}/k{i}"], data[f"{name}/v{i}"], starts[i]) for i in range(nseg)]
        out.append(dict(name=name, dtype=dtype, q=data[f"{name}/q"], segs=segs, q_start=q_start,
                        out=data[f"{name}/out"], Hkv=Hkv))
    return out


@dataclass
class PagedLayout:
    """Synthetic layer storage: archived blocks at scattered arena rows plus a ring."""

    dtype: str
    batch: int
    kv_heads: int
    head_dim: int
    rows: int
    ring_cap: int
    hot_head: int
    hot_len: int
    hot_start: int
    k_store: np.ndarray     # [groups, rows, D] storage dtype
    v_store: np.ndarray
    records: np.ndarray     # [n_blocks + 1, 4] int32
    block_lens: list
    block_starts: list

    def oracle_segments(self):
        """Segments in the reference order (archived by logical_start, then hot pieces), float32."""
        groups, D = self.batch * self.kv_heads, self.head_dim
        kf = from_storage(self.k_store, self.dtype)
        vf = from_storage(self.v_store, self.dtype)
        shape = lambda x, n: x.reshape(self.batch, self.kv_heads, n, D)  # noqa: E731
        segs = []
        for row, start, n, _ in self.records[:-1]:
            segs.append((shape(kf[:, row:row + n], n), shape(vf[:, row:row + n], n), int(start)))
        first = min(self.hot_len, self.ring_cap - self.hot_head)
        if first > 0:
            segs.append((shape(kf[:, self.hot_head:self.hot_head + first], first),
                         shape(vf[:, self.hot_head:self.hot_head + first], first), self.hot_start))
        rest = self.hot_len - first
        if rest > 0:
            segs.append((shape(kf[:, :rest], rest), shape(vf[:, :rest], rest), self.hot_start + first))
        return segs

    @property
    def total_tokens(self):
        return sum(self.block_lens) + self.hot_len


def make_layout(dtype: str, batch: int, kv_heads: int, head_dim: int, block_lens, ring_cap: int, hot_len: int,
                hot_head: int, seed: int, *, shuffle: bool = True, gap: int = 3) -> PagedLayout:
    rng = np.random.default_rng(seed)
    groups = batch * kv_heads
    n_blocks = len(block_lens)
    # place blocks in the pool at scattered rows (random order, small gaps)
    order = rng.permutation(n_blocks) if shuffle else np.arange(n_blocks)
    rows_of = [0] * n_blocks
    cursor = ring_cap
    for idx in order:
        cursor += int(rng.integers(0, gap + 1)) if gap else 0
        rows_of[idx] = cursor
        cursor += block_lens[idx]
    rows = cursor + 5
    k = rng.standard_normal((groups, rows, head_dim), dtype=np.float32)
    v = rng.standard_normal((groups, rows, head_dim), dtype=np.float32)
    records = np.zeros((n_blocks + 1, 4), np.int32)
    pos, tile = 0, 0
    starts = []
    for i, n in enumerate(block_lens):
        records[i] = (rows_of[i], pos, n, tile)
        starts.append(pos)
        pos += n
        tile += (n + TILE - 1) // TILE
    records[n_blocks, 3] = tile
    return PagedLayout(dtype, batch, kv_heads, head_dim, rows, ring_cap, hot_head, hot_len, pos,
                       to_storage(k, dtype), to_storage(v, dtype), records, list(block_lens), starts)


def torch_dtype(name: str):
    import torch

    return {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[name]


def to_device_storage(x: np.ndarray, dtype: str):
    """numpy storage array (uint16 bits for bf16) -> CUDA tensor of that dtype."""
    import torch

    if dtype == "bfloat16":
        return torch.from_numpy(x.view(np.int16).copy()).cuda().view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_paged(layout: PagedLayout, q: np.ndarray, q_pos0: int, *, max_splits: int = 0, want_lse: bool = True,
              step_state=None):
    """Run rfsn_paged_attention on the layout through the C ABI; returns numpy out (and lse).

    ``step_state`` (RFSN_STEP_* int32 values, or True for the layout's own
    window and q_pos0) passes the query position and hot window through a
    device step state instead of the call's arguments, which then carry zeros."""
    import torch

    from rfsn_b200 import _native as native

    k = to_device_storage(layout.k_store, layout.dtype)
    v = to_device_storage(layout.v_store, layout.dtype)
    arena = native.Arena(k, v)
    rec = torch.from_numpy(layout.records).cuda()
    B, H, Lq, D = q.shape
    qd = torch.from_numpy(np.ascontiguousarray(q, dtype=np.float32)).cuda()
    out = torch.empty_like(qd)
    lse = torch.empty((B, H, Lq), dtype=torch.float32, device="cuda")
    nblk = len(layout.block_lens)
    table = native.PageTableC(rec.data_ptr(), nblk, int(sum(layout.block_lens)), int(layout.records[nblk, 3]), 0)
    if step_state is None:
        hot = native.HotWindowC(0, layout.ring_cap, layout.hot_head, layout.hot_len, layout.hot_start)
    else:
        if step_state is True:
            step_state = [q_pos0, 0, layout.hot_head, layout.hot_len, layout.hot_start, 0, 0, 0]
        state = torch.tensor(list(step_state) + [0] * (native.STEP_STATE_LEN - len(step_state)), dtype=torch.int32,
                             device="cuda")
        # decoy window in the arguments: the kernel must take the state's
        hot = native.HotWindowC(0, layout.ring_cap, 0, 1, 0, 0, state.data_ptr())
        q_pos0 = 0
    nbytes = native.workspace_bytes(B, H, layout.kv_heads, Lq, D, max_splits)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    native.check(
        native.lib().rfsn_paged_attention(
            arena.handle, qd.data_ptr(), B, H, layout.kv_heads, Lq, q_pos0, ctypes.byref(table), ctypes.byref(hot),
            out.data_ptr(), lse.data_ptr() if want_lse else None, ws.data_ptr(), nbytes, max_splits,
            native.stream_ptr(),
        ),
        "rfsn_paged_attention",
    )
    native.check(native.lib().rfsn_workspace_check(ws.data_ptr(), native.stream_ptr(), 30_000_000), "workspace")
    torch.cuda.synchronize()
    # counters must be back at zero for the next call
    G = H // layout.kv_heads
    qblocks = (Lq * G + 7) // 8
    counters = ws[256:256 + 4 * B * layout.kv_heads * qblocks].view(torch.int32)
    assert int(counters.abs().sum().item()) == 0, "split counters not reset"
    res = out.cpu().numpy()
    arena.close()
    return (res, lse.cpu().numpy()) if want_lse else res
