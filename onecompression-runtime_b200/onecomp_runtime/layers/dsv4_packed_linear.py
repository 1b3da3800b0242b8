"""Packed int4 / int2 Linear for DeepSeek-V4-style QEP weights on B200.

Same API as the reference ``layers/dsv4_packed_linear.py``:
``dequant_dsv4_packed(p, dtype, device)`` (reference :22-56) and
``Dsv4PackedLinear(packed, bias=None, buffer_device="cpu")`` (reference :59-102).

``qweight_packed`` is uint8 [out, ceil(in*wbits/8)] with ``8 // wbits`` codes
per byte (code j at bits ``j*wbits``); ``scales``/``qzeros`` are groupwise in
``[out, G]`` or ``[G, out]`` (fractional zeros allowed); the weight is
``(q - z) * s`` in fp32 rounded once -- reproduced bit for bit by
``oc_b200_dsv4_dequant``. When the buffers live on the GPU, ``forward`` runs the
fused row-packed tcgen05 GEMM (``oc_b200_rows_gemm``). Buffers kept on the host
(offloaded experts, the DSV4 adapter's default) are copied per call, still
packed, into a device staging slot shared by every module of the same shape on
that stream, and the same fused GEMM runs on the slot: the reference copies the
packed bytes and dequantizes to a dense weight for ``F.linear``
(dsv4_packed_linear.py:95-98); here only the packed bytes cross and no dense
weight is materialized.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ._rows_base import MODE_EXACT, RowsHandle, float_param, group_major, prep_activation, rows_fusable


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
    home = dev
    if dev.type != "cuda":
        # host tensors and no target device: dequantize on the current CUDA device and return
        # the result on the host, as the reference does for CPU buffers (no CPU fallback)
        if not torch.cuda.is_available():
            raise RuntimeError("onecomp_runtime (B200) dequantizes on CUDA sm_100 devices only; got "
                               f"{dev} tensors and no CUDA device. There is no CPU fallback.")
        dev = torch.device("cuda", torch.cuda.current_device())
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
    return out if home == dev else out.to(home)


# Staging slots for host-resident (offloaded) layers: one set of device buffers and one kernel
# handle per (device, stream, shapes, dtypes). Every call copies its packed bytes into the slot and
# runs the GEMM on it in the same stream, so modules of one shape share the slot in stream order.
_STAGING: dict[tuple, tuple] = {}


def _staging_slot(q: torch.Tensor, s: torch.Tensor, z: torch.Tensor, dev: torch.device, wbits: int, gs: int,
                  K: int, N: int, sn: int, sg: int):
    key = (dev, _lib.stream_of(dev), tuple(q.shape), q.dtype, tuple(s.shape), s.dtype, tuple(z.shape), z.dtype,
           wbits, gs, K, N, sn, sg)
    slot = _STAGING.get(key)
    if slot is None:
        qd = torch.empty(q.shape, dtype=q.dtype, device=dev)
        sd = torch.empty(s.shape, dtype=s.dtype, device=dev)
        zd = torch.empty(z.shape, dtype=z.dtype, device=dev)
        h = RowsHandle([qd], [sd], [zd], wbits, gs, K, N, MODE_EXACT, sn, sg)
        slot = (qd, sd, zd, h)
        _STAGING[key] = slot
    return slot


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
        # group-major copies of scales / zeros (the kernel stages each block's rows by TMA)
        N, K = self.out_features, self.in_features
        s = group_major(self.scales, N, K, self.groupsize)
        z = group_major(self.qzeros, N, K, self.groupsize)
        h = RowsHandle([q], [s], [z], self.wbits, gs, K, N, MODE_EXACT, 1, N)
        self.__dict__["_handle"] = h
        self.__dict__["_handle_key"] = key
        return h

    def _fusable(self) -> bool:
        gs = self.groupsize if self.groupsize > 0 else self.in_features
        return self.wbits in (2, 4) and rows_fusable(int(self.qweight_packed.shape[1]), self.in_features,
                                                     self.out_features, gs, self.wbits)

    def _staged_handle(self, dev: torch.device):
        """Copy the host-resident packed buffers into the shared device slot; its handle."""
        gs = self.groupsize if self.groupsize > 0 else self.in_features
        s, z = float_param(self.scales), float_param(self.qzeros)
        sn, sg = _stride_of(s, self.out_features, self.in_features, self.groupsize)
        qd, sd, zd, h = _staging_slot(self.qweight_packed, s, z, dev, self.wbits, gs, self.in_features,
                                      self.out_features, sn, sg)
        qd.copy_(self.qweight_packed, non_blocking=True)
        sd.copy_(s, non_blocking=True)
        zd.copy_(z, non_blocking=True)
        return h

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and self._fusable():
            if self.qweight_packed.device == x.device:
                h = self._rows_handle()
            elif self.qweight_packed.device.type == "cpu":
                h = self._staged_handle(x.device)
            else:
                h = None
            if h is not None:
                a = prep_activation(x, self.in_features)
                out = torch.empty((a.shape[0], self.out_features), dtype=x.dtype, device=x.device)
                if a.shape[0]:
                    bias = self.bias.to(device=x.device, dtype=x.dtype) if self.bias is not None else None
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
