"""RTN uint8-nibble packed layers on B200.

Same API as the reference ``layers/packed_linear.py``:

* ``PackedRTNLinear(in_features, out_features, qweight_u8, scales, zeros, bias=None)``
  (reference :22-62): ``qweight_u8`` [out, ceil(in/2)] (low nibble = even k),
  ``scales``/``zeros`` [out, G]; the weight is ``(q - z) * s`` computed in the
  activation dtype with a rounding after each op (quant_utils.py:72-103).
* ``PackedEmbedding`` (reference :65-110): gathers token rows, then dequantizes.

On the GPU, ``PackedRTNLinear.forward`` runs the fused row-packed tcgen05 GEMM
(``oc_b200_rows_gemm``, RTN mode: the kernel multiplies exactly the weights
``dequant_extra_u8_to_weight`` produces) for fp16/bf16 inputs. Packed rows whose
byte stride is not a multiple of 16, or an ``in_features`` that is not a
multiple of 8 (one group per row), are copied once into a zero-padded device
layout (K rounded up to 8, rows to 16 bytes; the activations are zero-padded to
match per call). Only groups that are not a multiple of 8 columns (a group
boundary inside a 32-bit code word) and fp32 inputs dequantize with the
bit-exact ``oc_b200_rtn_dequant`` kernel and call ``F.linear`` in fp32, as the
reference does.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _lib
from ..quant_utils import dequant_extra_u8_to_weight
from ._rows_base import MODE_RTN, RowsHandle, group_major, prep_activation, rows_fusable


class PackedRTNLinear(nn.Module):
    """nn.Linear-compatible (in_features, out_features) RTN int4 packed Linear."""

    def __init__(self, in_features: int, out_features: int, qweight_u8: torch.Tensor, scales: torch.Tensor,
                 zeros: torch.Tensor, bias: torch.Tensor | None = None) -> None:
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.register_buffer("qweight_u8", qweight_u8.contiguous())
        self.register_buffer("scales", scales.contiguous())
        self.register_buffer("zeros", zeros.contiguous())
        if bias is not None:
            self.register_parameter("bias", nn.Parameter(bias.detach(), requires_grad=False))
        else:
            self.bias = None

    def _materialize(self, dtype: torch.dtype) -> torch.Tensor:
        return dequant_extra_u8_to_weight(self.qweight_u8, self.scales, self.zeros, self.in_features,
                                          self.out_features, dtype)

    def _rows_handle(self):
        """The fused-GEMM handle, or None for groups the kernel cannot take. Sets ``_k_run``, the
        K the kernel runs (``in_features`` rounded up to 8 when the layout was padded)."""
        key = (self.qweight_u8.data_ptr(), self.scales.data_ptr(), self.zeros.data_ptr(), self.scales.dtype,
               self.zeros.dtype)
        h = self.__dict__.get("_handle")
        if h is not None and self.__dict__.get("_handle_key") == key:
            return h
        K, N = self.in_features, self.out_features
        G = int(self.scales.shape[1])
        gs = K if G == 1 else K // G
        q = self.qweight_u8
        ld = int(q.shape[1])
        k_run = K
        if not rows_fusable(ld, K, N, gs, 4):
            k_run = (K + 7) // 8 * 8
            gs_run = k_run if G == 1 else gs
            ld_run = max((k_run + 1) // 2, ld)
            ld_run = (ld_run + 15) // 16 * 16
            if ld * 2 < K or not rows_fusable(ld_run, k_run, N, gs_run, 4):
                return None
            # zero-padded copy (codes past in_features meet zero activations)
            qp = torch.zeros((N, ld_run), dtype=torch.uint8, device=q.device)
            qp[:, :ld].copy_(q)
            q, gs = qp, gs_run
        # group-major copies of scales / zeros (the kernel stages each block's rows by TMA)
        s = group_major(self.scales, N, K, K if G == 1 else gs)
        z = group_major(self.zeros, N, K, K if G == 1 else gs)
        h = RowsHandle([q], [s], [z], 4, gs, k_run, N, MODE_RTN, 1, N)
        self.__dict__["_handle"] = h
        self.__dict__["_handle_key"] = key
        self.__dict__["_k_run"] = k_run
        return h

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and x.dtype in (torch.float16, torch.bfloat16):
            h = self._rows_handle()
            if h is not None:
                k_run = self.__dict__["_k_run"]
                a = prep_activation(x, self.in_features)
                if k_run != self.in_features:
                    a = F.pad(a, (0, k_run - self.in_features))
                out = torch.empty((a.shape[0], self.out_features), dtype=x.dtype, device=x.device)
                if a.shape[0]:
                    bias = self.bias.to(x.dtype) if self.bias is not None else None
                    h.gemm(a, out, bias=bias)
                return out.reshape(*x.shape[:-1], self.out_features)
        w = self._materialize(x.dtype)
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, w, bias)

    def _apply(self, fn, recurse=True):
        self.__dict__["_handle"] = None
        return super()._apply(fn, recurse=recurse)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, packed=int4")


class PackedEmbedding(nn.Module):
    """nn.Embedding-compatible RTN int4 packed table (rows gathered, then dequantized)."""

    def __init__(self, num_embeddings: int, embedding_dim: int, qweight_u8: torch.Tensor, scales: torch.Tensor,
                 zeros: torch.Tensor, padding_idx: int | None = None) -> None:
        super().__init__()
        self.num_embeddings = int(num_embeddings)
        self.embedding_dim = int(embedding_dim)
        self.padding_idx = padding_idx
        self.register_buffer("qweight_u8", qweight_u8.contiguous())
        self.register_buffer("scales", scales.contiguous())
        self.register_buffer("zeros", zeros.contiguous())

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Gather + dequantize the requested rows in one kernel (``oc_b200_rtn_embedding``);
        same output as the reference's gathers + ``dequant_extra_u8_to_weight``
        (packed_linear.py:92-104), in the scales' dtype (fp16 for integer scales; fp16,
        bf16 and fp32 tables are supported).
        Negative ids count from the end of the table; ids outside the table give zero rows
        and set the device error word (``_lib.read_device_error``)."""
        dev = self.qweight_u8.device
        _lib.require_b200(dev)
        flat = input_ids.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
        dtype = self.scales.dtype if self.scales.dtype.is_floating_point else torch.float16
        if dtype not in _lib.DT:
            raise TypeError(f"unsupported scales dtype {dtype} (fp16/bf16/fp32 or integer)")
        out = torch.empty((flat.shape[0], self.embedding_dim), dtype=dtype, device=dev)
        s = self.scales if self.scales.dtype in _lib.DT else self.scales.float()
        z = self.zeros if self.zeros.dtype in _lib.DT else self.zeros.float()
        s, z = s.contiguous(), z.contiguous()
        if flat.shape[0]:
            _lib.call("oc_b200_rtn_embedding", flat.data_ptr(), flat.shape[0], self.num_embeddings,
                      self.qweight_u8.data_ptr(), self.qweight_u8.shape[1], s.data_ptr(), _lib.DT[s.dtype],
                      z.data_ptr(), _lib.DT[z.dtype], self.embedding_dim, int(s.shape[1]), out.data_ptr(),
                      _lib.DT[dtype], _lib.stream_of(dev))
        return out.reshape(*input_ids.shape, self.embedding_dim)

    def extra_repr(self) -> str:
        return f"num_embeddings={self.num_embeddings}, embedding_dim={self.embedding_dim}, packed=int4"
