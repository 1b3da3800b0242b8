"""IEEE-754 half/bfloat16 helpers for the CPU oracle (test infrastructure only).

numpy has no bfloat16, so bf16 tensors travel as ``uint16`` bit patterns.
Conversions implement round-to-nearest-even from the IEEE-754 definition, which
is what ``torch.Tensor.to(torch.bfloat16/float16)`` does on CPU and GPU.
"""
from __future__ import annotations

import numpy as np

F16, BF16, F32 = "f16", "bf16", "f32"


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return b.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even; NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)).astype(np.uint32)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, (u >> np.uint64(16)).astype(np.uint32) | np.uint32(0x40), r)
    return r.astype(np.uint16)


def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    # numpy's float32 -> float16 cast rounds to nearest even, with subnormals.
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def to_f32(bits_or_vals: np.ndarray, dtype: str) -> np.ndarray:
    """Decode a tensor stored as ``dtype`` (bits for f16/bf16) to float32."""
    if dtype == BF16:
        return bf16_bits_to_f32(bits_or_vals)
    if dtype == F16:
        return f16_bits_to_f32(bits_or_vals)
    if dtype == F32:
        return np.asarray(bits_or_vals, dtype=np.float32)
    raise ValueError(dtype)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype``; returns bit patterns for f16/bf16."""
    if dtype == BF16:
        return f32_to_bf16_bits(x)
    if dtype == F16:
        return f32_to_f16_bits(x)
    if dtype == F32:
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dtype)


def quantize(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` and return them as float32 again."""
    return to_f32(round_to(x, dtype), dtype)
