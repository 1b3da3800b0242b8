"""Handle management for row-packed (RTN / DSV4) weights on the sm_100a tcgen05 kernel.

A ``RowsHandle`` describes E row-packed matrices of one shape [N, K] (E = 1 for
a dense layer, E = experts for the MoE grouped GEMM). The TMA descriptors and
pointer tables live in a small device buffer owned by the handle; the weight
tensors stay owned by the module.
"""
from __future__ import annotations

import ctypes

import torch

from .. import _lib

MODE_EXACT = 0   # DSV4: (q - z) * s in fp32, one rounding
MODE_RTN = 1     # RTN: two roundings in the activation dtype


def rows_fusable(ld_bytes: int, K: int, N: int, groupsize: int, wbits: int) -> bool:
    """Shapes the fused row-packed kernel takes (16-byte row stride, word-aligned groups)."""
    span = 32 // wbits
    return (ld_bytes % 16 == 0 and ld_bytes * (8 // wbits) >= K and K % 8 == 0 and N > 0
            and (groupsize % span == 0 or groupsize >= K))


class RowsHandle:
    def __init__(self, packed: list[torch.Tensor], scales: list[torch.Tensor], zeros: list[torch.Tensor],
                 wbits: int, groupsize: int, K: int, N: int, mode: int, stride_n: int, stride_g: int):
        dev = packed[0].device
        _lib.require_b200(dev)
        E = len(packed)
        lib = _lib.lib()
        self.h = None
        self.keep = (packed, scales, zeros)
        self.table = torch.empty(lib.oc_b200_rows_table_bytes(E), dtype=torch.uint8, device=dev)
        arr = ctypes.c_void_p * E
        pk = arr(*[t.data_ptr() for t in packed])
        sp = arr(*[t.data_ptr() for t in scales])
        zp = arr(*[t.data_ptr() for t in zeros])
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _lib.call("oc_b200_rows_layer_create", E, pk, packed[0].stride(0), wbits, sp, _lib.DT[scales[0].dtype],
                      zp, _lib.DT[zeros[0].dtype], stride_n, stride_g, groupsize, K, N, mode, self.table.data_ptr(),
                      _lib.stream_of(dev), ctypes.byref(h))
        self.h = h
        self.K, self.N, self.E = K, N, E
        self.device = dev

    def gemm(self, a: torch.Tensor, out: torch.Tensor, offsets: torch.Tensor | None = None,
             bias: torch.Tensor | None = None) -> None:
        _lib.call("oc_b200_rows_gemm", self.h, a.data_ptr(), _lib.DT[a.dtype], a.shape[0], a.stride(0),
                  None if offsets is None else offsets.data_ptr(),
                  None if bias is None else bias.data_ptr(), _lib.DT[bias.dtype] if bias is not None else 0,
                  out.data_ptr(), out.stride(0), _lib.stream_of(a.device))

    def gemm_swiglu(self, a: torch.Tensor, out: torch.Tensor, offsets: torch.Tensor | None = None) -> None:
        """``out = silu(a @ gate.T) * (a @ up.T)`` for a handle built on [N, 2K] gate|up matrices
        (``oc_b200_rows_gemm_swiglu``); ``a`` has K = self.K / 2 columns."""
        _lib.call("oc_b200_rows_gemm_swiglu", self.h, a.data_ptr(), _lib.DT[a.dtype], a.shape[0], a.stride(0),
                  None if offsets is None else offsets.data_ptr(), out.data_ptr(), out.stride(0),
                  _lib.stream_of(a.device))

    def close(self):
        if self.h is not None:
            try:
                _lib.lib().oc_b200_layer_destroy(self.h)
            except Exception:
                pass
            self.h = None

    def __del__(self):
        self.close()


def group_major(t: torch.Tensor, N: int, K: int, gs: int) -> torch.Tensor:
    """Scales or zeros as a contiguous [G, N] float tensor (the layout the kernel stages by TMA with
    each weight block): given [N, G] (``scales.shape == (out, groups)``, transposed as
    dsv4_packed_linear.py:50-51 does) or [G, N]; one group per row (``gs <= 0`` or ``gs >= K``) gives
    [1, N]."""
    t = float_param(t)
    G = 1 if (gs <= 0 or gs >= K) else (K + gs - 1) // gs
    if G == 1:
        return t.reshape(1, N).contiguous()
    if tuple(t.shape) == (N, G):
        return t.t().contiguous()
    return t.reshape(G, N).contiguous()


def float_param(t: torch.Tensor) -> torch.Tensor:
    """Scales/zeros as a float dtype the kernels read (int zero points become fp32, exactly)."""
    if t.dtype in (torch.float16, torch.bfloat16, torch.float32):
        return t.contiguous()
    return t.float().contiguous()


def prep_activation(x: torch.Tensor, K: int) -> torch.Tensor:
    a = x.reshape(-1, K)
    if a.stride(1) != 1 or a.data_ptr() % 16 or a.stride(0) % 8 or a.stride(0) < K:
        a = a.contiguous()
        if a.data_ptr() % 16:
            a = a.clone()
    return a
