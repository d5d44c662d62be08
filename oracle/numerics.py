"""Storage-dtype helpers for the oracle (test infrastructure).

numpy has no bfloat16, so bf16 tensors are carried as ``uint16`` bit patterns.
Conversion fp32 -> bf16 is IEEE round-to-nearest-even on the upper 16 bits
(the rounding torch, MLX and CUDA's ``__float2bfloat16_rn`` all use); NaN
payloads are not special-cased because the oracle never produces NaN.
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return ((u + rounding) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values through ``dtype`` storage and back to float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x.copy()
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    raise ValueError(f"unsupported dtype {dtype!r}")


def to_storage(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> the array the device stores (uint16 bits for bfloat16)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x.copy()
    if dtype == "float16":
        return x.astype(np.float16)
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x)
    raise ValueError(f"unsupported dtype {dtype!r}")


def from_storage(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(x)
    return np.asarray(x).astype(np.float32)
