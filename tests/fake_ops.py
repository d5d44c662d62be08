"""Test double for ``rfsn_b200.cache.DeviceOps``.

Moves rows between CPU tensors so that the cache's host bookkeeping (ring
indices, seal rule, page table, warm/cold residency, disk round trips) can be
checked against the reference traces without a GPU. It performs no attention
and no RoPE, and nothing in the product can construct it: tests pass it to
``LayerKVCache(ops=...)`` explicitly.
"""

from __future__ import annotations

from types import SimpleNamespace

import torch


class FakeDeviceOps:
    def __init__(self) -> None:
        self.device = torch.device("cpu")
        self.arena = None
        self.k = self.v = None
        self.calls: list[tuple] = []

    def new_arena(self, groups, rows, head_dim, dtype):
        self.k = torch.zeros((groups, rows, head_dim), dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.arena = SimpleNamespace(handle=None, groups=groups, rows=rows, head_dim=head_dim, dtype=dtype)
        return self.k, self.v

    def copy_rows(self, src_row0, src_offset, src_wrap, dst_row0, count):
        self.calls.append(("copy_rows", src_row0, src_offset, src_wrap, dst_row0, count))
        for i in range(count):
            s = src_offset + i
            if src_wrap:
                s %= src_wrap
            self.k[:, dst_row0 + i] = self.k[:, src_row0 + s]
            self.v[:, dst_row0 + i] = self.v[:, src_row0 + s]

    def append(self, q, k, v, inv_freq, start_pos, capacity, write_index):
        if inv_freq is not None or q is not None:
            raise NotImplementedError("the CPU test double does not rotate")
        self.calls.append(("append", int(k.shape[2]), write_index))
        groups = k.shape[0] * k.shape[1]
        kk = k.reshape(groups, k.shape[2], k.shape[3])
        vv = v.reshape(groups, v.shape[2], v.shape[3])
        for i in range(kk.shape[1]):
            slot = (write_index + i) % capacity
            self.k[:, slot] = kk[:, i]
            self.v[:, slot] = vv[:, i]
        return None

    def rotate_q(self, q, inv_freq, start_pos):
        raise NotImplementedError("the CPU test double does not rotate")

    def download(self, row, n, out_dtype):
        self.calls.append(("download", row, n))
        return self.k[:, row:row + n].to(out_dtype).clone(), self.v[:, row:row + n].to(out_dtype).clone()

    def download_pinned(self, row, n):
        self.calls.append(("download_pinned", row, n))
        return self.k[:, row:row + n].clone(), self.v[:, row:row + n].clone()

    def upload(self, row, n, k_host, v_host):
        self.calls.append(("upload", row, n))
        self.k[:, row:row + n] = k_host.to(self.k.dtype)
        self.v[:, row:row + n] = v_host.to(self.v.dtype)

    def new_table(self, rows):
        return torch.zeros((rows, 4), dtype=torch.int32)
