"""RTN uint8-nibble dequant restated in numpy (test infrastructure only).

Restates ``dequant_extra_u8_to_weight`` (reference ``quant_utils.py:72-103``):
the arithmetic runs in the *activation* dtype, so ``q - z`` and ``(q - z) * s``
are each rounded to that dtype (two roundings), exactly like torch's bf16/fp16
elementwise ops (fp32 compute, round to nearest even after every op).
"""
from __future__ import annotations

import numpy as np

from .fp import quantize, round_to, to_f32


def unpack_u8_nibbles(qweight_u8: np.ndarray, in_features: int) -> np.ndarray:
    """uint8 [out, ceil(in/2)] -> int [out, in]: low nibble = even k (quant_utils.py:85-90)."""
    q = np.asarray(qweight_u8, dtype=np.uint8)
    out_f, half = q.shape
    lo = (q & 0x0F).astype(np.int32)
    hi = ((q >> 4) & 0x0F).astype(np.int32)
    inter = np.stack([lo, hi], axis=-1).reshape(out_f, half * 2)
    return inter[:, :in_features]


def dequant_rtn(qweight_u8, scales, scales_dtype, zeros, zeros_dtype, in_features,
                out_features, dtype):
    """Return the weight [out, in] in ``dtype`` (bit patterns for f16/bf16)."""
    w = unpack_u8_nibbles(qweight_u8, in_features).astype(np.float32)  # exact in any dtype
    s = quantize(to_f32(scales, scales_dtype), dtype)                   # scales.to(dtype)
    z = quantize(to_f32(zeros, zeros_dtype), dtype)                     # zeros.to(dtype)
    num_groups = s.shape[1]
    if num_groups == 1:
        d = quantize(w - z, dtype)
        return round_to(d * s, dtype)
    if in_features % num_groups != 0:
        raise RuntimeError(
            f"in_features={in_features} not divisible by num_groups={num_groups}")
    gs = in_features // num_groups
    g = np.arange(in_features) // gs
    d = quantize(w - z[:, g], dtype)
    return round_to(d * s[:, g], dtype)


def pack_u8_nibbles(w_int: np.ndarray) -> np.ndarray:
    """int [out, in] -> uint8 [out, ceil(in/2)] (inverse of ``unpack_u8_nibbles``)."""
    w = np.asarray(w_int, dtype=np.int64) & 0xF
    out_f, in_f = w.shape
    if in_f % 2:
        w = np.concatenate([w, np.zeros((out_f, 1), dtype=np.int64)], axis=1)
    return (w[:, 0::2] | (w[:, 1::2] << 4)).astype(np.uint8)
