"""DSV4 int4/int2 byte-packed dequant restated in numpy (test infrastructure only).

Restates ``dequant_dsv4_packed`` (reference ``layers/dsv4_packed_linear.py:22-56``):
``per = 8 // wbits`` codes per byte along the in-dim, code j at bits ``j*wbits``;
fp32 ``(q - z) * s`` rounded once to the output dtype; ``groupsize <= 0`` means one
scale/zero per output row; scales/zeros given as ``(out, groups)`` are transposed
to ``(groups, out)`` first.
"""
from __future__ import annotations

import numpy as np

from .fp import round_to, to_f32


def unpack_codes(qweight_packed: np.ndarray, wbits: int, in_features: int) -> np.ndarray:
    q = np.asarray(qweight_packed, dtype=np.uint8).astype(np.int32)
    out_f, ncol = q.shape
    per = 8 // wbits
    mask = (1 << wbits) - 1
    codes = np.stack([(q >> (j * wbits)) & mask for j in range(per)], axis=-1)
    return codes.reshape(out_f, ncol * per)[:, :in_features]


def dequant_dsv4(qweight_packed, scales, scales_dtype, qzeros, qzeros_dtype, wbits,
                 groupsize, in_features, dtype):
    q = unpack_codes(qweight_packed, wbits, in_features)
    out_f, in_f = q.shape
    s = to_f32(scales, scales_dtype)
    z = to_f32(qzeros, qzeros_dtype)
    gs = int(groupsize)
    if gs <= 0:
        s = s.reshape(out_f, 1)
        z = z.reshape(out_f, 1)
        w = ((q.astype(np.float32) - z).astype(np.float32) * s).astype(np.float32)
        return round_to(w, dtype)
    num_groups = (in_f + gs - 1) // gs
    if s.shape == (out_f, num_groups):
        s, z = s.T, z.T
    g = np.arange(in_f) // gs
    s_e = s[g, :].T
    z_e = z[g, :].T
    w = ((q.astype(np.float32) - z_e).astype(np.float32) * s_e).astype(np.float32)
    return round_to(w, dtype)


def pack_codes(codes: np.ndarray, wbits: int) -> np.ndarray:
    """int [out, in] -> uint8 [out, ceil(in*wbits/8)] (inverse of ``unpack_codes``)."""
    per = 8 // wbits
    c = np.asarray(codes, dtype=np.int64) & ((1 << wbits) - 1)
    out_f, in_f = c.shape
    ncol = (in_f + per - 1) // per
    pad = np.zeros((out_f, ncol * per), dtype=np.int64)
    pad[:, :in_f] = c
    pad = pad.reshape(out_f, ncol, per)
    acc = np.zeros((out_f, ncol), dtype=np.int64)
    for j in range(per):
        acc |= pad[:, :, j] << (j * wbits)
    return acc.astype(np.uint8)
