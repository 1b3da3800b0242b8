"""AutoGPTQ v1/v2 unpack + dequant restated in numpy (test infrastructure only).

Restates ``onecomp_runtime/quant_utils.py`` (reference):

* ``unpack_rows``       -- ``_unpack_rows`` (quant_utils.py:12-28)
* ``unpack_int_weights``-- quant_utils.py:36-42
* ``unpack_zeros``      -- quant_utils.py:45-47
* ``dequant_gptq``      -- ``dequant_gptq_to_fp`` (quant_utils.py:50-69): fp32
  product ``s * (q - z)`` rounded ONCE to the output dtype
* ``pack_rows``         -- ``_pack_int4_weights`` (layers/fused_int4_linear.py:76-91),
  generalised to any ``wbits`` dividing 32
* ``dequant_gptq_torch``-- the same formula on torch CPU tensors (multi-threaded), for
  preparing the CPU baseline's large weights; checked equal to ``dequant_gptq`` by the tests
"""
from __future__ import annotations

import numpy as np

from .fp import round_to, to_f32


def unpack_rows(packed: np.ndarray, num_rows: int, wbits: int) -> np.ndarray:
    """int32 [R, C] words -> int32 [num_rows, C]; value i of word r is row pf*r+i."""
    if 32 % wbits != 0:
        raise ValueError(f"wbits must divide 32, got {wbits}")
    p = np.ascontiguousarray(packed).astype(np.int64) & 0xFFFFFFFF
    pf = 32 // wbits
    mask = (1 << wbits) - 1
    rows, cols = p.shape
    out = np.empty((rows, pf, cols), dtype=np.int32)
    for i in range(pf):
        out[:, i, :] = (p >> (i * wbits)) & mask
    return out.reshape(rows * pf, cols)[:num_rows]


def unpack_int_weights(packed: np.ndarray, wbits: int, original_shape) -> np.ndarray:
    """qweight [K/pf, N] -> int [N, K] (nn.Linear layout)."""
    in_features = int(original_shape[1])
    return np.ascontiguousarray(unpack_rows(packed, in_features, wbits).T)


def unpack_zeros(packed_zeros: np.ndarray, wbits: int, out_features: int) -> np.ndarray:
    """qzeros [G, N/pf] packed along N -> int [G, N]."""
    t = np.ascontiguousarray(np.asarray(packed_zeros).T)
    return np.ascontiguousarray(unpack_rows(t, out_features, wbits).T)


def dequant_gptq(qweight, scales, scales_dtype, qzeros, g_idx, in_features,
                 out_features, out_dtype, v1=True, wbits=4):
    """Return the dequantized weight [N, K] rounded to ``out_dtype``.

    ``scales`` holds bit patterns for f16/bf16 (or float32 values for f32).
    The result holds bit patterns for f16/bf16 outputs.
    """
    w = unpack_int_weights(qweight, wbits, (out_features, in_features))
    z = unpack_zeros(qzeros, wbits, out_features)
    if v1:
        z = (z + 1) & ((1 << wbits) - 1)
    g = np.asarray(g_idx, dtype=np.int64)
    s = to_f32(scales, scales_dtype)
    s_e = s[g, :].T
    z_e = z[g, :].T.astype(np.float32)
    prod = (s_e * (w.astype(np.float32) - z_e)).astype(np.float32)
    return round_to(prod, out_dtype)


def default_g_idx(in_features: int, groupsize: int) -> np.ndarray:
    """``torch.arange(in) // gs`` (backend.py:249-252, packed_gptq_linear.py:53-56)."""
    return (np.arange(in_features, dtype=np.int64) // int(groupsize)).astype(np.int64)


def pack_rows(values: np.ndarray, wbits: int) -> np.ndarray:
    """int [R, C] -> int32 [ceil(R/pf), C] packing ``pf`` rows per word (row r at bits wbits*(r%pf))."""
    pf = 32 // wbits
    v = np.asarray(values, dtype=np.int64) & ((1 << wbits) - 1)
    rows, cols = v.shape
    prow = (rows + pf - 1) // pf
    pad = np.zeros((prow * pf, cols), dtype=np.int64)
    pad[:rows] = v
    acc = np.zeros((prow, cols), dtype=np.int64)
    for i in range(pf):
        acc |= pad[i::pf] << (i * wbits)
    return acc.astype(np.uint32).view(np.int32)


def pack_int_weights(w_int: np.ndarray, wbits: int = 4) -> np.ndarray:
    """int [N, K] -> qweight int32 [K/pf, N] (fused_int4_linear.py:76-91)."""
    return pack_rows(np.ascontiguousarray(np.asarray(w_int).T), wbits)


def pack_zeros(zeros: np.ndarray, wbits: int = 4) -> np.ndarray:
    """int [G, N] -> qzeros int32 [G, N/pf] packed along N."""
    return np.ascontiguousarray(pack_rows(np.ascontiguousarray(np.asarray(zeros).T), wbits).T)


def dequant_gptq_torch(qweight, scales, qzeros, g_idx, in_features, out_features, out_dtype, v1=True, wbits=4):
    """``dequant_gptq`` on torch CPU tensors: int32 qweight [K/pf, N], scales [G, N] (any float
    dtype), int32 qzeros [G, N/pf], g_idx [K] -> [N, K] in ``out_dtype`` (a torch dtype).
    Same fp32 product s * (q - z) and one round-to-nearest-even conversion (quant_utils.py:50-69)."""
    import torch

    pf = 32 // wbits
    mask = (1 << wbits) - 1
    shifts = torch.arange(0, 32, wbits, dtype=torch.int64)
    qw = qweight.to(torch.int64) & 0xFFFFFFFF
    q = ((qw.unsqueeze(1) >> shifts.view(1, pf, 1)) & mask).reshape(-1, qw.shape[1])[:in_features]  # [K, N]
    qz = qzeros.to(torch.int64) & 0xFFFFFFFF
    z = ((qz.unsqueeze(2) >> shifts.view(1, 1, pf)) & mask).reshape(qz.shape[0], -1)[:, :out_features]  # [G, N]
    if v1:
        z = (z + 1) & mask
    g = g_idx.to(torch.int64)
    prod = scales.to(torch.float32)[g] * (q.to(torch.float32) - z.to(torch.float32)[g])
    return prod.t().contiguous().to(out_dtype)
