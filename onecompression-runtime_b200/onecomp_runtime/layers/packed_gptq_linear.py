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

8-bit layers with uniform groups (``g_idx == k // groupsize``, groupsize 32 or a multiple
of 64) run the 8-bit decode GEMV for M <= 16 tokens and the tcgen05 GEMM up to
``_KERNEL8_MAX_M`` tokens (measured on B200 at 3072 -> 9216: 2.1x the dequant + ``F.linear``
path at M = 64, 1.8x at 512, 0.9x at 4608). Act-order 8-bit layers whose groups each hold
``groupsize`` rows (g_idx a permutation of ``k // groupsize``, what GPTQ's act-order writes) run
the same kernels after a K re-layout: rows sorted by group on the GPU
(``oc_b200_gptq_repack_k_ex``) and the activation columns gathered in that order. Larger M,
other group layouts and fp32 inputs dequantize with the B200 dequant kernel and call
``F.linear``, as the reference does for every call.
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from .. import _lib
from ..quant_utils import dequant_gptq_to_fp
from ._gptq_base import B200GPTQLinear

_KERNEL8_MAX_M = 2048



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
            K, N, gs = self.in_features, self.out_features, self.groupsize
            shapes_ok = (self.wbits == 8 and K >= 64 and K % 8 == 0 and N >= 128 and N % 32 == 0
                         and (gs == 32 or (gs > 0 and gs % 64 == 0))
                         and tuple(self.qweight.shape) == (K // 4, N)
                         and int(self.scales.shape[0]) == (K + gs - 1) // gs
                         and tuple(self.g_idx.shape) == (K,))
            self._kperm8 = None   # group-sorted row order of an act-order layer (host int32)
            self._h8_bufs = None  # the device copies the handle reads: (k_perm, repacked qweight)
            uniform = False
            if shapes_ok:
                trivial = torch.arange(K, device=self.g_idx.device, dtype=torch.long) // gs
                uniform = bool(torch.equal(self.g_idx, trivial))
                if not uniform:
                    order = torch.argsort(self.g_idx, stable=True)
                    if bool(torch.equal(self.g_idx[order], trivial)):   # every group holds gs rows
                        self._kperm8 = order.to(torch.int32).cpu()
                        uniform = True
            self._kernel8_ok = shapes_ok and uniform

    # ------------------------------------------------------------------ 8-bit kernels
    def _get_handle8(self):
        key = (self.qweight.data_ptr(), self.qzeros.data_ptr(), self.scales.data_ptr(), self.scales.dtype,
               self.qweight.device)
        if self._handle is not None and self._handle_key == key:
            return self._handle
        self._release_handle()
        dev = self.qweight.device
        _lib.require_b200(dev)
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            qw, kp = self.qweight, None
            if self._kperm8 is not None:   # act-order: rows sorted by group, activations gathered
                kp = self._kperm8.to(dev)
                qw = torch.empty_like(self.qweight)
                _lib.call("oc_b200_gptq_repack_k_ex", self.qweight.data_ptr(), kp.data_ptr(), self.in_features,
                          self.out_features, 8, qw.data_ptr(), _lib.stream_of(dev))
                self._h8_bufs = (kp, qw)
            _lib.call("oc_b200_gptq_layer_create_ex", qw.data_ptr(), self.qzeros.data_ptr(),
                      self.scales.data_ptr(), _lib.DT[self.scales.dtype], None if kp is None else kp.data_ptr(),
                      None, self.in_features, self.in_features, self.out_features, int(self.scales.shape[0]),
                      self.groupsize, 8, int(self.v1), ctypes.byref(h))
        self._handle = h
        self._handle_key = key
        return h

    def _use_kernel8(self, x: torch.Tensor, M: int) -> bool:
        return (self._kernel8_ok and 0 < M <= _KERNEL8_MAX_M and x.is_cuda and x.dtype in (torch.float16, torch.bfloat16)
                and self.scales.dtype in (torch.float16, torch.bfloat16) and self.qweight.device == x.device
                and all(t.data_ptr() % 16 == 0 for t in (self.qweight, self.qzeros, self.scales)))

    def _forward_kernel8(self, x: torch.Tensor, M: int) -> torch.Tensor:
        lead = x.shape[:-1]
        a_2d = x.reshape(M, self.in_features)
        if a_2d.stride(1) != 1 or a_2d.stride(0) % 8 != 0 or a_2d.data_ptr() % 16 != 0:
            a_2d = a_2d.contiguous()
            if a_2d.data_ptr() % 16 != 0:
                a_2d = a_2d.clone()
        out = torch.empty((M, self.out_features), dtype=x.dtype, device=x.device)
        h = self._get_handle8()
        lib = _lib.lib()
        ws = _lib.workspace(x.device, lib.oc_b200_gptq_gemm_workspace(h, M))
        bias = self.bias
        _lib.check(lib.oc_b200_gptq_gemm(h, a_2d.data_ptr(), _lib.DT[x.dtype], M, a_2d.stride(0),
                                         None if bias is None else bias.data_ptr(),
                                         _lib.DT[bias.dtype] if bias is not None else 0, out.data_ptr(),
                                         out.stride(0), ws.data_ptr(), ws.numel(), _lib.stream_of(x.device)),
                   "oc_b200_gptq_gemm (8-bit)")
        return out.reshape(*lead, self.out_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.wbits == 4:
            return self._forward_impl(x, "packed")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected last dim {self.in_features}, got {tuple(x.shape)}")
        M = x.numel() // self.in_features
        if self._use_kernel8(x, M):
            return self._forward_kernel8(x, M)
        weight = dequant_gptq_to_fp(qweight=self.qweight, scales=self.scales, qzeros=self.qzeros,
                                    g_idx=self.g_idx, in_features=self.in_features,
                                    out_features=self.out_features, dtype=x.dtype, v1=self.v1, wbits=self.wbits)
        bias = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, weight, bias)

    def _apply(self, fn, recurse=True):
        if self.wbits == 4:
            return super()._apply(fn, recurse=recurse)
        self._release_handle()
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
