"""Shared machinery of the B200 GPTQ int4 linear modules.

``B200GPTQLinear`` keeps the reference modules' buffers (``qweight`` int32
[K/8, N], ``scales`` [G, N], ``qzeros`` int32 [G, N/8], optional ``g_idx`` and
``bias``) verbatim and derives, once at load time, the kernel-side K order:

* natural order (no re-layout) when groups are contiguous runs of ``gs``
  rows with ``gs % 8 == 0`` -- the common case;
* otherwise (act-order ``g_idx``, irregular ``g_idx``, or a groupsize that is
  not a multiple of 8, e.g. 26) rows are sorted by group and every group is
  padded to a multiple of 8 rows with zero codes; ``k_perm`` maps each kernel
  row to its activation column (-1 = padding) and ``word_group`` gives the
  group of each 8-row word. This replaces both the padded-group re-layout
  (fused_int4_linear.py:94-124) and the per-call ``scales[g_idx]`` gathers
  (quant_utils.py:66-67).

``forward`` calls ``oc_b200_gptq_gemm`` on the current stream (split-K GEMV for
M <= 16, tcgen05 kernel above) and never synchronises.
"""
from __future__ import annotations

import atexit
import ctypes
import os
import time

import torch

from .. import _lib

_PROFILE_SHAPES = os.environ.get("ONECOMP_PROFILE_SHAPES") == "1"
_PROFILE_PADDED_GROUPS = os.environ.get("ONECOMP_PROFILE_PADDED_GROUPS") == "1"
_SHAPE_STATS: dict[tuple[str, int, int, int], int] = {}
_PADDED_GROUPS_STATS: dict[str, float] = {"calls": 0.0, "seconds": 0.0}


def _print_shape_stats() -> None:
    # same output format as fused_int4_linear.py:58-70
    if not _PROFILE_SHAPES or not _SHAPE_STATS:
        return
    print("[onecomp-profile] fused shape calls:", flush=True)
    for (kind, m, k, n), count in sorted(_SHAPE_STATS.items(), key=lambda item: item[1], reverse=True)[:40]:
        print(f"[onecomp-profile] {kind:14s} M={m:<5d} K={k:<5d} N={n:<5d} calls={count}", flush=True)


def _print_padded_groups_stats() -> None:
    # same output format as fused_int4_linear.py:42-52
    if not _PROFILE_PADDED_GROUPS:
        return
    calls = int(_PADDED_GROUPS_STATS["calls"])
    seconds = _PADDED_GROUPS_STATS["seconds"]
    if calls:
        print(f"[onecomp-profile] FusedInt4LinearPaddedGroups calls={calls} "
              f"total={seconds:.6f}s avg={seconds / calls * 1000:.3f}ms", flush=True)


atexit.register(_print_padded_groups_stats)
atexit.register(_print_shape_stats)


def plan_k_layout(in_features: int, groupsize: int, num_groups: int, g_idx: torch.Tensor | None):
    """Return ``(k_packed, k_perm, word_group, gs_eff)`` for the kernels.

    ``k_perm``/``word_group`` are CPU int32 tensors or None. ``gs_eff`` is the
    uniform kernel groupsize (0 when ``word_group`` is needed).
    """
    K = int(in_features)
    gs = int(groupsize)
    if g_idx is None:
        gi = torch.arange(K, dtype=torch.int64) // max(gs, 1)
    else:
        gi = g_idx.detach().to("cpu", torch.int64).reshape(-1)
        if gi.numel() != K:
            raise ValueError(f"g_idx has {gi.numel()} entries, expected in_features={K}")
    if gi.numel() and (int(gi.min()) < 0 or int(gi.max()) >= num_groups):
        raise ValueError(f"g_idx values must lie in [0, {num_groups})")
    natural = gs > 0 and gs % 8 == 0 and K % 8 == 0 and torch.equal(gi, torch.arange(K) // gs)
    if natural:
        return K, None, None, gs
    order = torch.argsort(gi, stable=True)
    counts = torch.bincount(gi, minlength=num_groups)
    padded = (counts + 7) // 8 * 8
    kp = int(padded.sum())
    kperm = torch.full((kp,), -1, dtype=torch.int32)
    word_group = torch.repeat_interleave(torch.arange(num_groups, dtype=torch.int32), padded // 8)
    src = 0
    dst = 0
    for g in range(num_groups):
        c = int(counts[g])
        kperm[dst:dst + c] = order[src:src + c].to(torch.int32)
        src += c
        dst += int(padded[g])
    nonempty = padded[counts > 0]
    if nonempty.numel() and bool((nonempty == nonempty[0]).all()) and bool((counts > 0).all()):
        return kp, kperm, None, int(nonempty[0])
    return kp, kperm, word_group, 0


class B200GPTQLinear(torch.nn.Module):
    """Common base: AutoGPTQ int4 layer run by the sm_100a kernels."""

    _kind = "b200"

    def __init__(self, in_features: int, out_features: int, qweight: torch.Tensor, scales: torch.Tensor,
                 qzeros: torch.Tensor, bias: torch.Tensor | None = None, groupsize: int = 32,
                 g_idx: torch.Tensor | None = None, v1: bool = True, wbits: int = 4):
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.groupsize = int(groupsize)
        self.wbits = int(wbits)
        self.v1 = bool(v1)
        if self.out_features % 8 != 0:
            raise ValueError(f"out_features={out_features} must be a multiple of 8 (qzeros packing)")
        self.register_buffer("qweight", qweight.contiguous())
        self.register_buffer("scales", scales.contiguous())
        self.register_buffer("qzeros", qzeros.contiguous())
        if g_idx is not None:
            self.register_buffer("g_idx", g_idx.to(torch.long).contiguous())
        else:
            self.g_idx = None
        if bias is not None:
            self.register_buffer("bias", bias.contiguous())
            self._has_bias = True
        else:
            self.bias = None
            self._has_bias = False
        G = int(self.scales.shape[0])
        kp, kperm, wgrp, gs_eff = plan_k_layout(self.in_features, self.groupsize, G, g_idx)
        self._k_packed = kp
        self._gs_eff = gs_eff
        self._relayout = kperm is not None
        if self._relayout:
            self.register_buffer("_k_perm", kperm, persistent=False)
            self.register_buffer("_word_group", wgrp, persistent=False)
            self.register_buffer("_qweight_k", torch.empty(0, dtype=torch.int32), persistent=False)
        self._layout_key = None
        self._handle = None
        self._handle_key = None

    # ------------------------------------------------------------------ kernel state
    def _ensure_layout(self) -> torch.Tensor:
        """The qweight tensor in kernel K order (repacked on the device once)."""
        if not self._relayout:
            return self.qweight
        key = (self.qweight.data_ptr(), self.qweight.device)
        if self._layout_key != key or self._qweight_k.numel() == 0:
            dev = self.qweight.device
            kperm = self._k_perm.to(dev)
            self._k_perm = kperm
            if self._word_group is not None:
                self._word_group = self._word_group.to(dev)
            out = torch.empty((self._k_packed // 8, self.out_features), dtype=torch.int32, device=dev)
            _lib.call("oc_b200_gptq_repack_k", self.qweight.data_ptr(), kperm.data_ptr(), self._k_packed,
                      self.out_features, out.data_ptr(), _lib.stream_of(dev))
            self._qweight_k = out
            self._layout_key = key
        return self._qweight_k

    def _get_handle(self):
        qw = self._ensure_layout()
        key = (qw.data_ptr(), self.qzeros.data_ptr(), self.scales.data_ptr(), self.scales.dtype,
               self.qweight.device)
        if self._handle is not None and self._handle_key == key:
            return self._handle
        self._release_handle()
        _lib.require_b200(self.qweight.device)
        if self.wbits != 4:
            raise NotImplementedError("the B200 GEMM kernels take 4-bit weights")
        if self.scales.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"scales must be fp16 or bf16, got {self.scales.dtype}")
        h = ctypes.c_void_p()
        kperm = self._k_perm if self._relayout else None
        wgrp = self._word_group if self._relayout else None
        with torch.cuda.device(self.qweight.device):
            _lib.call("oc_b200_gptq_layer_create", qw.data_ptr(), self.qzeros.data_ptr(), self.scales.data_ptr(),
                      _lib.DT[self.scales.dtype], _lib.ptr(kperm), _lib.ptr(wgrp), self.in_features,
                      self._k_packed, self.out_features, int(self.scales.shape[0]), self._gs_eff,
                      int(self.v1), ctypes.byref(h))
        self._handle = h
        self._handle_key = key
        return h

    def _release_handle(self):
        h = self.__dict__.get("_handle")
        if h is not None:
            try:
                _lib.lib().oc_b200_layer_destroy(h)
            except Exception:
                pass
        self.__dict__["_handle"] = None
        self.__dict__["_handle_key"] = None

    def __del__(self):
        self._release_handle()

    def _gemm_2d(self, a_2d: torch.Tensor, out: torch.Tensor, residual: torch.Tensor | None = None,
                 act: int = 0) -> None:
        h = self._get_handle()
        M = a_2d.shape[0]
        dev = a_2d.device
        lib = _lib.lib()
        need = lib.oc_b200_gptq_gemm_workspace(h, M)
        ws = _lib.workspace(dev, need)
        bias = self.bias
        rc = lib.oc_b200_gptq_gemm_ex(h, a_2d.data_ptr(), _lib.DT[a_2d.dtype], M, a_2d.stride(0),
                                      None if bias is None else bias.data_ptr(),
                                      _lib.DT[bias.dtype] if bias is not None else 0,
                                      None if residual is None else residual.data_ptr(),
                                      0 if residual is None else residual.stride(0), act,
                                      out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(), _lib.stream_of(dev))
        _lib.check(rc, "oc_b200_gptq_gemm_ex")

    _ACTS = {None: 0, "none": 0, "gelu_tanh": 1}

    def forward_fused(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                      activation: str | None = None) -> torch.Tensor:
        """``act(x @ W.T + bias) + residual`` with the activation and residual add in the
        GEMM epilogue (one rounding). ``activation``: None or ``"gelu_tanh"``; ``residual``:
        same shape and dtype as the output."""
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"forward_fused takes fp16/bf16 inputs, got {x.dtype}")
        act = self._ACTS[activation]
        lead = x.shape[:-1]
        a_2d = x.reshape(-1, self.in_features)
        if (a_2d.stride(1) != 1 or a_2d.data_ptr() % 16 != 0 or a_2d.stride(0) % 8 != 0
                or a_2d.stride(0) < self.in_features):
            a_2d = a_2d.contiguous()
        M = a_2d.shape[0]
        r2 = None
        if residual is not None:
            r2 = residual.reshape(M, self.out_features)
            if r2.dtype != x.dtype or r2.stride(1) != 1:
                raise ValueError("residual must match the output's dtype with unit column stride")
        out = torch.empty((M, self.out_features), dtype=x.dtype, device=x.device)
        if M:
            self._gemm_2d(a_2d, out, r2, act)
        return out.reshape(*lead, self.out_features)

    def _forward_impl(self, x: torch.Tensor, kind: str) -> torch.Tensor:
        if x.dtype == torch.float32:
            # the reference runs fp32 inputs through the fp16 kernel and upcasts the
            # result (fused_int4_linear.py:415-419, 535-536)
            return self._forward_impl(x.to(torch.float16), kind).to(torch.float32)
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise TypeError(f"unsupported input dtype {x.dtype}")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected last dim {self.in_features}, got {tuple(x.shape)}")
        lead = x.shape[:-1]
        a_2d = x.reshape(-1, self.in_features)
        # rows may be strided (e.g. a column slice of a wider output): the kernels
        # take lda; they need unit column stride and 16-byte aligned rows.
        if (a_2d.stride(1) != 1 or a_2d.data_ptr() % 16 != 0 or a_2d.stride(0) % 8 != 0
                or a_2d.stride(0) < self.in_features):
            a_2d = a_2d.contiguous()
            if a_2d.data_ptr() % 16 != 0:
                a_2d = a_2d.clone()
        M = a_2d.shape[0]
        if _PROFILE_SHAPES:
            key = (kind, int(M), self.in_features, self.out_features)
            _SHAPE_STATS[key] = _SHAPE_STATS.get(key, 0) + 1
        out = torch.empty((M, self.out_features), dtype=x.dtype, device=x.device)
        if M:
            self._gemm_2d(a_2d, out)
        return out.reshape(*lead, self.out_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._forward_impl(x, "fused")

    @torch.no_grad()
    def warmup(self, m_values=(32, 128, 256, 1024, 2250)) -> None:
        """Kernels are compiled ahead of time; this builds the layer handle and
        sizes the shared workspace for the given token counts."""
        device = self.qweight.device
        dtype = self.scales.dtype if self.scales.dtype in (torch.float16, torch.bfloat16) else torch.float16
        for m in m_values:
            if m <= 0:
                continue
            x = torch.zeros((int(m), self.in_features), dtype=dtype, device=device)
            _ = self.forward(x)
        if device.type == "cuda":
            torch.cuda.synchronize(device)

    def _apply(self, fn, recurse=True):
        # keep packed integer buffers int32 and scales 16-bit across .to(dtype)
        # (fused_int4_linear.py:1230-1246)
        qweight_before = self.qweight
        qzeros_before = self.qzeros
        g_before = self.g_idx
        result = super()._apply(fn, recurse=recurse)
        if self.qweight.dtype != torch.int32:
            self.qweight = qweight_before.to(self.qweight.device)
        if self.qzeros.dtype != torch.int32:
            self.qzeros = qzeros_before.to(self.qzeros.device)
        if g_before is not None and self.g_idx.dtype != torch.long:
            self.g_idx = g_before.to(self.g_idx.device)
        if self._relayout:
            if self._k_perm.dtype != torch.int32:
                self._k_perm = self._k_perm.to(torch.int32)
            if self._word_group is not None and self._word_group.dtype != torch.int32:
                self._word_group = self._word_group.to(torch.int32)
            if self._qweight_k.dtype != torch.int32:
                self._qweight_k = self._qweight_k.to(torch.int32)
            self._layout_key = None
        if self.scales.dtype not in (torch.float16, torch.bfloat16):
            self.scales = self.scales.to(torch.float16)
        self._release_handle()
        return result

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"groupsize={self.groupsize}, v1={self.v1}, backend=b200")
