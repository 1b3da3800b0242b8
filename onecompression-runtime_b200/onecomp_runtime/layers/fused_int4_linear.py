"""Fused int4 dequant + GEMM for AutoGPTQ packed weights on B200 (sm_100a).

Same public API as the reference ``onecomp_runtime/layers/fused_int4_linear.py``:

* ``FusedInt4Linear(in_features, out_features, qweight, scales, qzeros, bias=None, groupsize=32)``
  (reference :958-1246) with ``forward``, ``warmup``, ``from_gptq_linear``,
  ``_apply`` and the ``in_features/out_features/groupsize/bias`` attributes;
* ``FusedInt4LinearAnyGroup`` (reference :639-758) and
  ``FusedInt4LinearPaddedGroups`` (reference :761-955, exposes ``padded_in_features``);
* ``fused_int4_gemm(a, qweight, scales, qzeros, bias=None, groupsize=32)`` (reference :388-537);
* ``_pack_int4_weights`` / ``_repack_groups_to_32`` helpers (reference :76-124).

The Triton kernels are replaced by the sm_100a kernels of ``liboc_b200.so``:
a tcgen05/TMEM GEMM for large M and a split-K tensor-core GEMV for M <= 16.
Dequantization is exact: every weight the kernels multiply equals
``quant_utils.dequant_gptq_to_fp`` bit for bit (fp32 product, one rounding),
where the reference Triton kernel rounds to fp16 first (:244).

Extra keyword arguments (defaults reproduce the reference): ``v1`` selects the
AutoGPTQ-v1 zero restore (the reference kernel always applies it, :221);
``g_idx`` is accepted by the generic classes.
"""
from __future__ import annotations

import time
from collections import OrderedDict

import torch

from .. import _lib
from ..quant_utils import unpack_int_weights
from ._gptq_base import B200GPTQLinear, _PADDED_GROUPS_STATS, _PROFILE_PADDED_GROUPS


def _pack_int4_weights(weight_int: torch.Tensor) -> torch.Tensor:
    """Pack integer weights from [out, in] to GPTQ qweight [in//8, out]."""
    if weight_int.dtype != torch.int32:
        weight_int = weight_int.to(torch.int32)
    out_features, in_features = weight_int.shape
    if in_features % 8 != 0:
        raise ValueError(f"in_features must be divisible by 8, got {in_features}")
    _lib.require_b200(weight_int.device)
    w = weight_int.contiguous()
    packed = torch.empty((in_features // 8, out_features), dtype=torch.int32, device=w.device)
    _lib.call("oc_b200_gptq_pack", w.data_ptr(), out_features, in_features, 4, packed.data_ptr(),
              _lib.stream_of(w.device))
    return packed


def _repack_groups_to_32(qweight: torch.Tensor, *, in_features: int, out_features: int,
                         groupsize: int) -> tuple[torch.Tensor, int]:
    """Re-layout odd-size GPTQ groups as 32-wide groups without re-quantizing."""
    if groupsize <= 0 or groupsize > 32:
        raise ValueError(f"groupsize must be in 1..32, got {groupsize}")
    if in_features % groupsize != 0:
        raise ValueError(f"in_features={in_features} must be divisible by groupsize={groupsize}")
    num_groups = in_features // groupsize
    padded_in_features = num_groups * 32
    weight_int = unpack_int_weights(qweight, 4, (out_features, in_features))
    padded = torch.zeros((out_features, padded_in_features), dtype=torch.int32, device=weight_int.device)
    padded.view(out_features, num_groups, 32)[:, :, :groupsize].copy_(
        weight_int.view(out_features, num_groups, groupsize))
    return _pack_int4_weights(padded), padded_in_features


class FusedInt4Linear(B200GPTQLinear):
    """Drop-in for a 4-bit / groupsize=32 GPTQ Linear; holds packed buffers verbatim."""

    def __init__(self, in_features: int, out_features: int, qweight: torch.Tensor, scales: torch.Tensor,
                 qzeros: torch.Tensor, bias: torch.Tensor | None = None, groupsize: int = 32, *,
                 v1: bool = True):
        assert groupsize == 32, "FusedInt4Linear supports groupsize=32 only"
        super().__init__(in_features, out_features, qweight, scales, qzeros, bias=bias, groupsize=32, v1=v1)
        # the reference pads K to a multiple of 256 for its Triton tiles; the
        # B200 kernels take any K (TMA zero-fills the tail), so no padding.
        self._k_padded = self.in_features
        self._empty_bias = None
        self._cfg_cache: dict[int, tuple] = {}

    @classmethod
    def from_gptq_linear(cls, layer) -> "FusedInt4Linear":
        """Build from a GPTQLinear (4-bit, groupsize=32), reusing its packed buffers."""
        assert layer.wbits == 4, f"FusedInt4Linear requires wbits=4, got {layer.wbits}"
        assert layer.groupsize == 32, f"FusedInt4Linear requires groupsize=32, got {layer.groupsize}"
        return cls(in_features=layer.in_features, out_features=layer.out_features, qweight=layer.qweight,
                   scales=layer.scales.to(torch.float16), qzeros=layer.qzeros,
                   bias=layer.bias if layer.bias is not None else None, groupsize=32)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._forward_impl(x, "fused")


class FusedInt4LinearAnyGroup(B200GPTQLinear):
    """Fused int4 GEMM for GPTQ layers with any groupsize (and optional g_idx)."""

    def __init__(self, in_features: int, out_features: int, qweight: torch.Tensor, scales: torch.Tensor,
                 qzeros: torch.Tensor, bias: torch.Tensor | None = None, groupsize: int = 32, *,
                 v1: bool = True, g_idx: torch.Tensor | None = None):
        super().__init__(in_features, out_features, qweight, scales, qzeros, bias=bias, groupsize=groupsize,
                         g_idx=g_idx, v1=v1)
        self._empty_bias = None
        self._cfg_cache: dict[int, tuple] = {}

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._forward_impl(x, "any_group")


class FusedInt4LinearPaddedGroups(B200GPTQLinear):
    """Odd groupsizes (< 32): groups are padded with zero codes at load time.

    The reference re-packs the weights into 32-wide groups and maps padded K
    rows back to the compact activations in its kernel (:761-955). Here the
    same padding is part of the kernel K order (``k_perm``); ``qweight`` keeps
    the checkpoint layout and ``padded_in_features`` reports the padded K.
    """

    def __init__(self, in_features: int, out_features: int, qweight: torch.Tensor, scales: torch.Tensor,
                 qzeros: torch.Tensor, bias: torch.Tensor | None = None, groupsize: int = 32, *,
                 v1: bool = True):
        if groupsize == 32:
            raise ValueError("FusedInt4LinearPaddedGroups is only for odd groupsizes")
        if groupsize <= 0 or groupsize > 32:
            raise ValueError(f"groupsize must be in 1..32, got {groupsize}")
        if in_features % groupsize != 0:
            raise ValueError(f"in_features={in_features} must be divisible by groupsize={groupsize}")
        super().__init__(in_features, out_features, qweight, scales, qzeros, bias=bias, groupsize=groupsize, v1=v1)
        self.num_groups = self.in_features // self.groupsize
        self.padded_in_features = int(self._k_packed)
        self._empty_bias = None
        self._cfg_cache: dict[int, tuple] = {}

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _PROFILE_PADDED_GROUPS and x.is_cuda:
            torch.cuda.synchronize(x.device)
            t0 = time.perf_counter()
            out = self._forward_impl(x, "padded")
            torch.cuda.synchronize(x.device)
            _PADDED_GROUPS_STATS["calls"] += 1.0
            _PADDED_GROUPS_STATS["seconds"] += time.perf_counter() - t0
            return out
        return self._forward_impl(x, "padded")


def fused_int4_gemm(a: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor,
                    bias: torch.Tensor | None = None, groupsize: int = 32) -> torch.Tensor:
    """Compute ``c = a @ dequantize(qweight) + bias`` (AutoGPTQ v1, groupsize 32).

    Args and checks follow the reference (fused_int4_linear.py:388-440); the
    output has ``a``'s dtype and leading shape (fp32 inputs run through fp16).
    """
    assert groupsize == 32, "fused_int4_gemm currently supports groupsize=32 only"
    assert qweight.dtype == torch.int32
    assert qzeros.dtype == torch.int32
    assert a.dtype in (torch.float16, torch.bfloat16, torch.float32), f"unsupported a.dtype={a.dtype}"
    K = a.shape[-1]
    N = scales.shape[1]
    assert qweight.shape == (K // 8, N), (
        f"qweight shape mismatch: expected ({K//8}, {N}), got {tuple(qweight.shape)}")
    assert scales.shape == (K // groupsize, N), (
        f"scales shape mismatch: expected ({K//groupsize}, {N}), got {tuple(scales.shape)}")
    assert qzeros.shape == (K // groupsize, N // 8), (
        f"qzeros shape mismatch: expected ({K//groupsize}, {N//8}), got {tuple(qzeros.shape)}")
    assert N % 8 == 0, f"N must be a multiple of 8 (qzeros packing), got N={N}"
    assert K % 32 == 0, f"K must be a multiple of 32 (groupsize), got K={K}"
    compute = torch.float16 if a.dtype == torch.float32 else a.dtype
    return _functional_layer(qweight, scales, qzeros, bias, compute)(a)


# Layers built by fused_int4_gemm, reused across calls on the same weight tensors: the handle
# (K layout, TMA descriptors) is host work done once instead of per call. An entry holds its
# weight tensors (so their memory cannot be reused while it exists) and matches on their data
# pointers, shapes, dtypes and torch's in-place version counters, so an edited weight rebuilds
# it. At most _FUNCTIONAL_MAX entries are kept (least recently used dropped first).
_FUNCTIONAL: "OrderedDict[tuple, FusedInt4Linear]" = OrderedDict()
_FUNCTIONAL_MAX = 64


def _functional_layer(qweight, scales, qzeros, bias, compute) -> FusedInt4Linear:
    srcs = (qweight, scales, qzeros) + ((bias,) if bias is not None else ())
    key = (tuple((t.data_ptr(), tuple(t.shape), t.stride(), t.dtype, t.device, t._version) for t in srcs), compute)
    layer = _FUNCTIONAL.get(key)
    if layer is not None:
        _FUNCTIONAL.move_to_end(key)
        return layer
    K, N = qweight.shape[0] * 8, scales.shape[1]
    s = scales if scales.dtype == compute else scales.to(compute)   # the reference casts scales (:421-422)
    b = None if bias is None else (bias if bias.dtype == compute else bias.to(compute))  # ... and bias (:445-447)
    layer = FusedInt4Linear(K, N, qweight, s, qzeros, bias=b, groupsize=32)
    layer._functional_srcs = srcs   # pins the caller's tensors for the key's lifetime
    _FUNCTIONAL[key] = layer
    while len(_FUNCTIONAL) > _FUNCTIONAL_MAX:
        _, old = _FUNCTIONAL.popitem(last=False)
        old._release_handle()
    return layer
