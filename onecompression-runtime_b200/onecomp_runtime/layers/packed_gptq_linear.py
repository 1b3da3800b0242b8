"""Packed AutoGPTQ Linear (4- or 8-bit, any groupsize, act-order, v1/v2) on B200.

Same constructor, buffers and ``forward`` contract as the reference
``layers/packed_gptq_linear.py:28-88``. Where the reference dequantizes the
whole layer with torch ops on every call and then runs ``F.linear``, 4-bit
layers here run the fused sm_100a kernels directly on the packed buffers:

* act-order ``g_idx`` is handled by a load-time K re-layout (rows sorted by
  group, ``k_perm`` gathers the activation columns), so decode reads every
  packed byte once;
* scales keep the dtype they were given (the reference's ``build_packed``
  stores them in the model dtype, backend.py:275) and the kernels multiply
  exactly the weights ``dequant_gptq_to_fp`` would produce.

8-bit layers dequantize with the B200 dequant kernel and call ``F.linear``.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..quant_utils import dequant_gptq_to_fp
from ._gptq_base import B200GPTQLinear


class PackedGPTQLinear(B200GPTQLinear):
    """nn.Linear-compatible packed GPTQ layer (4- or 8-bit, any groupsize)."""

    def __init__(self, in_features: int, out_features: int, qweight: torch.Tensor, scales: torch.Tensor,
                 qzeros: torch.Tensor, g_idx: torch.Tensor | None = None, bias: torch.Tensor | None = None,
                 groupsize: int = 128, wbits: int = 4, v1: bool = True) -> None:
        if g_idx is None:
            g_idx = (torch.arange(in_features, device=qweight.device) // groupsize).to(torch.long)
        if int(wbits) == 4:
            super().__init__(in_features, out_features, qweight, scales, qzeros, bias=bias, groupsize=groupsize,
                             g_idx=g_idx, v1=v1, wbits=4)
        else:
            torch.nn.Module.__init__(self)
            self.in_features = int(in_features)
            self.out_features = int(out_features)
            self.groupsize = int(groupsize)
            self.wbits = int(wbits)
            self.v1 = bool(v1)
            self.register_buffer("qweight", qweight.contiguous())
            self.register_buffer("scales", scales.contiguous())
            self.register_buffer("qzeros", qzeros.contiguous())
            self.register_buffer("g_idx", g_idx.to(torch.long).contiguous())
            if bias is not None:
                self.register_buffer("bias", bias.contiguous())
            else:
                self.bias = None
            self._has_bias = bias is not None
            self._relayout = False
            self._handle = None
            self._handle_key = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.wbits == 4:
            return self._forward_impl(x, "packed")
        weight = dequant_gptq_to_fp(qweight=self.qweight, scales=self.scales, qzeros=self.qzeros,
                                    g_idx=self.g_idx, in_features=self.in_features,
                                    out_features=self.out_features, dtype=x.dtype, v1=self.v1, wbits=self.wbits)
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, weight, bias)

    def _apply(self, fn, recurse=True):
        if self.wbits == 4:
            return super()._apply(fn, recurse=recurse)
        qw, qz, gi = self.qweight, self.qzeros, self.g_idx
        result = torch.nn.Module._apply(self, fn, recurse=recurse)
        if self.qweight.dtype != torch.int32:
            self.qweight = qw.to(self.qweight.device)
        if self.qzeros.dtype != torch.int32:
            self.qzeros = qz.to(self.qzeros.device)
        if self.g_idx.dtype != torch.long:
            self.g_idx = gi.to(self.g_idx.device)
        return result

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"wbits={self.wbits}, groupsize={self.groupsize}, packed=True")
