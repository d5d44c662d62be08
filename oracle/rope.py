"""Rotary embedding, restated in numpy float32 (test infrastructure).

* ``inv_freq`` / ``rope_tables`` -> ``build_rope_tables`` layer.py:20-35:
  inv_freq = 1 / base ** (arange(0, half, f32) / half), positions are float32
  arange(start, start + L), freqs = positions[:, None] * inv_freq[None, :]
  (one float32 product), emb = [freqs, freqs], cos/sin of emb in float32.
* ``apply_rope`` -> ``_apply_rope`` layer.py:38-51 (NeoX rotate-half:
  [x1 c - x2 s, x1 s + x2 c]); x is promoted to float32 because the tables are
  float32 (model.py:120 builds them in float32), so the result is float32.
* ``rope_tables_in`` / ``apply_rope_in`` -> the same two functions when the
  tables are in another dtype (layer.py:118-126: a layer called without
  tables builds them in the model dtype; tables passed in are used as given):
  cos/sin evaluated in float32 and rounded to the table dtype, and every
  product and sum of the rotation rounded to the promoted dtype of x and the
  tables (the 16-bit type when both are that type, else float32), the way
  MLX's elementwise ops round each result.
"""

from __future__ import annotations

import numpy as np

from .numerics import round_to_dtype


def inv_freq(head_dim: int, base: float) -> np.ndarray:
    half = head_dim // 2
    exponent = np.arange(0, half, dtype=np.float32) / np.float32(half)
    return (np.float32(1.0) / np.power(np.float32(base), exponent, dtype=np.float32)).astype(np.float32)


def rope_tables(head_dim: int, base: float, seq_len: int, start_pos: int = 0) -> tuple[np.ndarray, np.ndarray]:
    inv = inv_freq(head_dim, base)
    positions = np.arange(start_pos, start_pos + seq_len, dtype=np.float64).astype(np.float32)
    freqs = positions[:, None] * inv[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x: np.ndarray, cos_t: np.ndarray, sin_t: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = cos_t[None, None]
    s = sin_t[None, None]
    return np.concatenate(
        [x1 * c[..., :half] - x2 * s[..., :half], x1 * s[..., half:] + x2 * c[..., half:]],
        axis=-1,
    ).astype(np.float32)


def promoted_dtype(x_dtype: str, table_dtype: str) -> str:
    """Result dtype of an elementwise op between the two (float16 with
    bfloat16 promotes to float32, as in MLX)."""
    return x_dtype if x_dtype == table_dtype else "float32"


def rope_tables_in(head_dim: int, base: float, seq_len: int, start_pos: int, dtype: str):
    """build_rope_tables(..., dtype=dtype): float32 tables rounded to dtype."""
    cos_t, sin_t = rope_tables(head_dim, base, seq_len, start_pos)
    return round_to_dtype(cos_t, dtype), round_to_dtype(sin_t, dtype)


def apply_rope_in(x: np.ndarray, cos_t: np.ndarray, sin_t: np.ndarray, dtype: str) -> np.ndarray:
    """_apply_rope with every product and sum rounded to ``dtype`` (float32
    values of x and of the tables, already representable in their dtypes)."""
    r = lambda a: round_to_dtype(a, dtype)  # noqa: E731
    x = np.asarray(x, dtype=np.float32)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = np.asarray(cos_t, dtype=np.float32)[None, None]
    s = np.asarray(sin_t, dtype=np.float32)[None, None]
    lo = r(r(x1 * c[..., :half]) - r(x2 * s[..., :half]))
    hi = r(r(x1 * s[..., half:]) + r(x2 * c[..., half:]))
    return np.concatenate([lo, hi], axis=-1).astype(np.float32)
