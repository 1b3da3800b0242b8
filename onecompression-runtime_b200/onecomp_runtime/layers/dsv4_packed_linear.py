"""Packed int4 / int2 Linear for DeepSeek-V4-style QEP weights on B200.

Same API as the reference ``layers/dsv4_packed_linear.py``:
``dequant_dsv4_packed(p, dtype, device)`` (reference :22-56) and
``Dsv4PackedLinear(packed, bias=None, buffer_device="cpu")`` (reference :59-102).

``qweight_packed`` is uint8 [out, ceil(in*wbits/8)] with ``8 // wbits`` codes
per byte (code j at bits ``j*wbits``); ``scales``/``qzeros`` are groupwise in
``[out, G]`` or ``[G, out]`` (fractional zeros allowed); the weight is
``(q - z) * s`` in fp32 rounded once -- reproduced bit for bit by
``oc_b200_dsv4_dequant``. When the buffers live on the GPU, ``forward`` runs the
fused row-packed tcgen05 GEMM (``oc_b200_rows_gemm``); buffers kept on the host
(offloaded experts) are copied to the activation's device per call, dequantized
and multiplied with ``F.linear``, as the reference does.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ._rows_base import MODE_EXACT, RowsHandle, float_param, prep_activation, rows_fusable


def _stride_of(scales: torch.Tensor, out_f: int, in_f: int, gs: int):
    """(stride_n, stride_g) of scales/zeros given as [out, G] or [G, out] (dsv4_packed_linear.py:42-51)."""
    if gs <= 0:
        return 1, 0
    num_groups = (in_f + gs - 1) // gs
    if tuple(scales.shape) == (out_f, num_groups):
        return num_groups, 1
    return 1, out_f


@torch.no_grad()
def dequant_dsv4_packed(p: dict, dtype: torch.dtype = torch.bfloat16, device=None) -> torch.Tensor:
    """Inverse of the DSV4 packer -> dense (out, in) weight on ``device``."""
    wbits = int(p["wbits"])
    gs = int(p["groupsize"])
    packed = p["qweight_packed"]
    dev = torch.device(device) if device is not None else packed.device
    _lib.require_b200(dev)
    if dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"unsupported dtype {dtype}")
    packed = packed.to(dev, non_blocking=True).contiguous()
    out_f, ncol = packed.shape
    in_f = int(p["in_features"])
    in_f = min(in_f, ncol * (8 // wbits))
    scales = p["scales"].to(dev)
    qzeros = p["qzeros"].to(dev)
    if scales.dtype not in _lib.DT:
        scales = scales.float()
    if qzeros.dtype not in _lib.DT:
        qzeros = qzeros.float()
    scales = scales.contiguous()
    qzeros = qzeros.contiguous()
    stride_n, stride_g = _stride_of(scales, out_f, in_f, gs)
    out = torch.empty((out_f, in_f), dtype=dtype, device=dev)
    _lib.call("oc_b200_dsv4_dequant", packed.data_ptr(), ncol, wbits, scales.data_ptr(), _lib.DT[scales.dtype],
              qzeros.data_ptr(), _lib.DT[qzeros.dtype], stride_n, stride_g, gs, in_f, out_f, out.data_ptr(),
              _lib.DT[dtype], _lib.stream_of(dev))
    return out


class Dsv4PackedLinear(nn.Module):
    """nn.Linear-compatible packed int4/int2 Linear for DSV4 QEP weights."""

    def __init__(self, packed: dict, bias: torch.Tensor | None = None, buffer_device="cpu") -> None:
        super().__init__()
        self.in_features = int(packed["in_features"])
        self.out_features = int(packed["qweight_packed"].shape[0])
        self.wbits = int(packed["wbits"])
        self.groupsize = int(packed["groupsize"])
        self.register_buffer("qweight_packed", packed["qweight_packed"].to(buffer_device).contiguous())
        self.register_buffer("scales", packed["scales"].to(buffer_device).contiguous())
        self.register_buffer("qzeros", packed["qzeros"].to(buffer_device).contiguous())
        if bias is not None:
            self.register_parameter("bias", nn.Parameter(bias.detach(), requires_grad=False))
        else:
            self.bias = None

    def _packed_dict(self) -> dict:
        return {"qweight_packed": self.qweight_packed, "scales": self.scales, "qzeros": self.qzeros,
                "wbits": self.wbits, "groupsize": self.groupsize, "in_features": self.in_features}

    @property
    def weight(self) -> torch.Tensor:
        """Dequantized dense (out, in) bf16 weight on the buffers' device (CUDA required)."""
        return dequant_dsv4_packed(self._packed_dict(), dtype=torch.bfloat16, device=self.qweight_packed.device)

    def _rows_handle(self):
        q = self.qweight_packed
        key = (q.data_ptr(), self.scales.data_ptr(), self.qzeros.data_ptr(), q.device)
        h = self.__dict__.get("_handle")
        if h is not None and self.__dict__.get("_handle_key") == key:
            return h
        gs = self.groupsize if self.groupsize > 0 else self.in_features
        if self.wbits not in (2, 4) or not rows_fusable(int(q.shape[1]), self.in_features, self.out_features, gs,
                                                        self.wbits):
            return None
        sn, sg = _stride_of(self.scales, self.out_features, self.in_features, self.groupsize)
        h = RowsHandle([q], [float_param(self.scales)], [float_param(self.qzeros)], self.wbits, gs,
                       self.in_features, self.out_features, MODE_EXACT, sn, sg)
        self.__dict__["_handle"] = h
        self.__dict__["_handle_key"] = key
        return h

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and self.qweight_packed.device == x.device and x.dtype in (torch.float16, torch.bfloat16):
            h = self._rows_handle()
            if h is not None:
                a = prep_activation(x, self.in_features)
                out = torch.empty((a.shape[0], self.out_features), dtype=x.dtype, device=x.device)
                if a.shape[0]:
                    bias = self.bias.to(x.dtype) if self.bias is not None else None
                    h.gemm(a, out, bias=bias)
                return out.reshape(*x.shape[:-1], self.out_features)
        w = dequant_dsv4_packed(self._packed_dict(), dtype=x.dtype, device=x.device)
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, w, bias)

    def _apply(self, fn, recurse=True):
        self.__dict__["_handle"] = None
        return super()._apply(fn, recurse=recurse)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"packed=int{self.wbits}, groupsize={self.groupsize}")
