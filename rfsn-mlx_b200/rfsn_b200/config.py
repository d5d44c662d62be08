"""Runtime configuration (drop-in for ``rfsn_v10_5.config``).

Same fields, defaults, validation rules and error messages as the reference
(config.py:24-129); dtypes resolve to torch dtypes instead of MLX dtypes.
"""

from __future__ import annotations

import re
from dataclasses import dataclass
from enum import Enum

import torch

_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}
_SESSION_RE = re.compile(r"^[A-Za-z0-9._-]+$")


def resolve_dtype(name: str) -> torch.dtype:
    """config.py:32-39."""
    if name not in _DTYPES:
        raise ValueError(f"model_dtype must be one of {set(_DTYPES)}, got '{name}'")
    return _DTYPES[name]


def validate_session_id(session_id: str) -> str:
    """config.py:42-51: strip; empty stays empty; otherwise [A-Za-z0-9._-]+."""
    cleaned = session_id.strip()
    if cleaned and not _SESSION_RE.fullmatch(cleaned):
        raise ValueError("session_id must contain only letters, numbers, '.', '_' or '-'")
    return cleaned


class RuntimeMode(str, Enum):
    """config.py:54-58."""

    EXACT = "exact"
    ARCHIVED = "archived"


@dataclass
class RFSNConfig:
    """config.py:61-129."""

    hidden_dim: int = 512
    num_heads: int = 8
    num_kv_heads: int = 0
    head_dim: int = 64
    num_layers: int = 4

    hot_capacity: int = 512
    warm_capacity: int = 2048
    cold_capacity: int = 8192
    block_size_seq: int = 64
    runtime_mode: RuntimeMode = RuntimeMode.ARCHIVED

    vocab_size: int = 50000
    max_position_embeddings: int = 0
    disk_cache_dir: str = "./rfsn_disk_cache"
    session_id: str = ""

    rope_base: float = 10000.0
    ffn_multiplier: int = 4
    ffn_dim: int = 0
    norm_eps: float = 1e-5
    model_dtype: str = "bfloat16"

    def __post_init__(self) -> None:
        if self.num_kv_heads <= 0:
            self.num_kv_heads = self.num_heads
        if not isinstance(self.runtime_mode, RuntimeMode):
            self.runtime_mode = RuntimeMode(str(self.runtime_mode))
        checks = [
            (
                self.hidden_dim == self.num_heads * self.head_dim,
                f"hidden_dim ({self.hidden_dim}) must equal num_heads * head_dim ({self.num_heads * self.head_dim})",
            ),
            (
                self.num_heads % self.num_kv_heads == 0,
                f"num_heads ({self.num_heads}) must be divisible by num_kv_heads ({self.num_kv_heads})",
            ),
            (
                self.hot_capacity <= self.warm_capacity <= self.cold_capacity,
                "Cache capacities must satisfy hot_capacity <= warm_capacity <= cold_capacity",
            ),
            (self.block_size_seq > 0, "block_size_seq must be > 0"),
            (self.max_position_embeddings >= 0, "max_position_embeddings must be >= 0"),
            (self.ffn_multiplier > 0, "ffn_multiplier must be > 0"),
            (bool(self.disk_cache_dir and self.disk_cache_dir.strip()), "disk_cache_dir must be a non-empty path"),
        ]
        for ok, message in checks:
            if not ok:
                raise ValueError(message)
        self.session_id = validate_session_id(self.session_id)
        if self.ffn_dim <= 0:
            self.ffn_dim = self.hidden_dim * self.ffn_multiplier
        if self.model_dtype not in _DTYPES:
            raise ValueError(f"model_dtype must be one of {set(_DTYPES)}, got '{self.model_dtype}'")

    @property
    def kv_groups(self) -> int:
        """Query heads per KV head (config.py:126-129)."""
        return self.num_heads // self.num_kv_heads
