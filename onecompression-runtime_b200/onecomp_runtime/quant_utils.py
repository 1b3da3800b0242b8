"""GPTQ / RTN unpack + dequant helpers, computed by the sm_100a kernels.

Same functions, arguments and results as the reference
``onecomp_runtime/quant_utils.py``:

* ``_unpack_rows`` / ``unpack_int_weights`` / ``unpack_zeros`` -- quant_utils.py:12-47
* ``dequant_gptq_to_fp``  -- quant_utils.py:50-69, bit-exact (fp32 product, one rounding)
* ``dequant_extra_u8_to_weight`` -- quant_utils.py:72-103, bit-exact (two roundings in ``dtype``)

Like the reference's helpers, these accept tensors on any device and return the
result on the device of the packed input: adapters call them on host tensors
straight from ``safe_open`` and move the result afterwards
(models/firered/loader.py:102-106, models/qwen36/loader.py:98-102). The
arithmetic always runs in the sm_100a kernels: host inputs are copied to the
current CUDA device, dequantized there, and the result is copied back. There is
no CPU fallback: without an sm_100 device every call raises ``RuntimeError``.
Error behaviour matches the reference (``ValueError`` for a ``wbits`` that does
not divide 32, ``RuntimeError`` for indivisible RTN groups).
"""
from __future__ import annotations

import torch

from . import _lib


def _dev(t: torch.Tensor) -> torch.device:
    """The CUDA device that runs the kernel for ``t``: its own, or the current one for a host tensor."""
    if t.device.type == "cuda":
        _lib.require_b200(t.device)
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError(
            f"onecomp_runtime (B200) dequantizes on CUDA sm_100 devices only; got a {t.device} tensor and no "
            "CUDA device. There is no CPU fallback.")
    dev = torch.device("cuda", torch.cuda.current_device())
    _lib.require_b200(dev)
    return dev


def _unpack_rows(packed: torch.Tensor, num_rows: int, wbits: int) -> torch.Tensor:
    """Unpack INT32-packed ``wbits`` values along dim-0 back to int values."""
    if 32 % wbits != 0:
        raise ValueError(f"wbits must divide 32, got {wbits}")
    home = packed.device
    dev = _dev(packed)
    packed = packed.to(device=dev, dtype=torch.int32).contiguous()
    rows, cols = packed.shape
    pf = 32 // wbits
    out = torch.empty((cols, rows * pf), dtype=torch.int32, device=dev)  # [N, K] then transpose
    if rows and cols:
        _lib.call("oc_b200_gptq_unpack", packed.data_ptr(), rows * pf, cols, wbits, out.data_ptr(),
                  _lib.stream_of(dev))
    return out.to(home).t()[:num_rows]


def _unpack_rows_int4(packed: torch.Tensor, num_rows: int) -> torch.Tensor:
    return _unpack_rows(packed, num_rows, 4)


def unpack_int_weights(packed: torch.Tensor, wbits: int, original_shape: tuple[int, int]) -> torch.Tensor:
    """Unpack AutoGPTQ-format packed weights (4- or 8-bit) to ``[out, in]``."""
    in_features = int(original_shape[1])
    return _unpack_rows(packed, in_features, wbits).t().contiguous()


def unpack_zeros(packed_zeros: torch.Tensor, wbits: int, out_features: int) -> torch.Tensor:
    """Unpack AutoGPTQ-format packed zero points (4- or 8-bit) to ``[G, out]``."""
    if 32 % wbits != 0:
        raise ValueError(f"wbits must divide 32, got {wbits}")
    home = packed_zeros.device
    dev = _dev(packed_zeros)
    qz = packed_zeros.to(device=dev, dtype=torch.int32).contiguous()
    G = qz.shape[0]
    pf = 32 // wbits
    n_full = qz.shape[1] * pf
    out = torch.empty((G, n_full), dtype=torch.int32, device=dev)
    if G and n_full:
        _lib.call("oc_b200_gptq_unpack_zeros", qz.data_ptr(), G, n_full, wbits, out.data_ptr(), _lib.stream_of(dev))
    return out[:, :out_features].contiguous().to(home)


def dequant_gptq_to_fp(
    qweight: torch.Tensor,
    scales: torch.Tensor,
    qzeros: torch.Tensor,
    g_idx: torch.Tensor,
    in_features: int,
    out_features: int,
    dtype: torch.dtype,
    v1: bool = True,
    wbits: int = 4,
) -> torch.Tensor:
    """Dequantize an AutoGPTQ v1/v2 packed 4- or 8-bit Linear to ``(out, in)`` ``dtype``."""
    if 32 % wbits != 0:
        raise ValueError(f"wbits must divide 32, got {wbits}")
    home = qweight.device
    dev = _dev(qweight)
    if dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"unsupported dtype {dtype}")
    if scales.dtype not in _lib.DT:
        raise TypeError(f"unsupported scales dtype {scales.dtype}")
    qweight = qweight.to(dev).contiguous()
    qzeros = qzeros.to(dev).contiguous()
    scales = scales.to(dev).contiguous()
    gi = None
    if g_idx is not None:
        gi = g_idx.to(device=dev, dtype=torch.int64).contiguous()
        if gi.numel() != in_features:
            raise ValueError(f"g_idx has {gi.numel()} entries, expected {in_features}")
    G = scales.shape[0]
    gs = 0 if gi is not None else max(1, in_features // max(G, 1))
    out = torch.empty((out_features, in_features), dtype=dtype, device=dev)
    _lib.call("oc_b200_gptq_dequant", qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(),
              _lib.DT[scales.dtype], _lib.ptr(gi), in_features, out_features, G, gs, wbits, int(bool(v1)),
              out.data_ptr(), _lib.DT[dtype], _lib.stream_of(dev))
    return out.to(home)


def dequant_extra_u8_to_weight(
    qweight_u8: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    in_features: int,
    out_features: int,
    dtype: torch.dtype,
) -> torch.Tensor:
    """Inverse of the RTN uint8-nibble packer (two 4-bit values per byte, low = even k)."""
    home = qweight_u8.device
    dev = _dev(qweight_u8)
    num_groups = scales.shape[1]
    if num_groups != 1 and in_features % num_groups != 0:
        raise RuntimeError(f"in_features={in_features} not divisible by num_groups={num_groups}")
    if dtype not in _lib.DT:
        raise TypeError(f"unsupported dtype {dtype} (the B200 RTN path computes in fp16/bf16/fp32)")
    q = qweight_u8.to(dev).contiguous()
    s = scales.to(dev)
    z = zeros.to(dev)
    if s.dtype not in _lib.DT:
        s = s.float()
    if z.dtype not in _lib.DT:
        z = z.float()
    s = s.contiguous()
    z = z.contiguous()
    out = torch.empty((out_features, in_features), dtype=dtype, device=dev)
    _lib.call("oc_b200_rtn_dequant", q.data_ptr(), q.shape[1], s.data_ptr(), _lib.DT[s.dtype], z.data_ptr(),
              _lib.DT[z.dtype], in_features, out_features, num_groups, out.data_ptr(), _lib.DT[dtype],
              _lib.stream_of(dev))
    return out.to(home)
