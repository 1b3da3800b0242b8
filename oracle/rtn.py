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


def embedding_rtn(ids, qweight_u8, scales, scales_dtype, zeros, zeros_dtype, dim, dtype):
    """PackedEmbedding.forward (reference packed_linear.py:92-104): gather the rows of ``ids``
    (negative ids count from the end, as torch indexing does) and dequantize them like
    ``dequant_rtn`` -> bit patterns [*ids.shape, dim]."""
    ids = np.asarray(ids, dtype=np.int64)
    vocab = qweight_u8.shape[0]
    flat = ids.reshape(-1)
    if ((flat < -vocab) | (flat >= vocab)).any():
        raise IndexError("embedding id out of range")
    flat = np.where(flat < 0, flat + vocab, flat)
    w = dequant_rtn(qweight_u8[flat], np.asarray(scales)[flat], scales_dtype, np.asarray(zeros)[flat], zeros_dtype,
                    dim, flat.shape[0], dtype)
    return w.reshape(*ids.shape, dim)


def quantize_conv_weight_f32(weight: np.ndarray, groupsize: int):
    """RTN encoder of the conv codecs (reference packed_conv.py:63-90) in numpy fp32:
    returns (qweight_u8, scales_f16_bits, zeros_f16_bits, cols). The division and rounding
    steps are the same IEEE fp32 operations torch performs, round-half-to-even."""
    w2 = np.asarray(weight, dtype=np.float32)
    rows, cols = w2.shape
    groups = cols // groupsize if groupsize > 0 and cols % groupsize == 0 else 1
    w = w2.reshape(rows, groups, cols // groups)
    hi = w.max(axis=-1, keepdims=True)
    lo = w.min(axis=-1, keepdims=True)
    empty = (hi == 0) & (lo == 0)
    hi = np.where(empty, np.float32(1), hi)
    lo = np.where(empty, np.float32(-1), lo)
    scale = np.maximum((hi - lo) / np.float32(15), np.float32(1e-8)).astype(np.float32)
    zero = np.round(-lo / scale).astype(np.float32)
    q = np.clip(np.round(w / scale) + zero, 0, 15).astype(np.int64).reshape(rows, cols)
    s16 = scale.reshape(rows, groups).astype(np.float16).view(np.uint16)
    z16 = zero.reshape(rows, groups).astype(np.float16).view(np.uint16)
    return pack_u8_nibbles(q), s16, z16, cols
