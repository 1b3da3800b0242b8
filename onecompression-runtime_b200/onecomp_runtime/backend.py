"""Backend selection + per-layer int4 module construction (B200 build).

Same functions and decision ladder as the reference ``onecomp_runtime/backend.py``
(:51-321), with one new backend name:

    - ``b200``   -- the sm_100a kernels of this package (fused int4 GEMM for
      large M, split-K GEMV for M <= 16, act-order/any-groupsize via a load-time
      K re-layout). ``auto`` resolves to it.
    - ``fused``  -- same modules as ``b200`` (the Triton kernel of the
      reference is replaced by the B200 kernels).
    - ``packed`` -- ``PackedGPTQLinear`` on the B200 kernels.
    - ``eager``  -- dequantize once (B200 dequant kernel) into ``nn.Linear``.

The GemLite backends (``gemlite``, ``a8w4*``, ``mxfp4*``, ``nvfp4_ffn``) are not
part of this build and raise, as the reference does when GemLite is missing.
``build_quant_layer`` keeps the reference's ``kind`` strings
(``fused`` / ``packed`` / ``eager``) so the loaders' counters work unchanged.

Differences from the reference, both corrections: the fused path honours
``checkpoint_format == "gptq_v2"`` (the reference Triton kernel always applies
the v1 zero restore, fused_int4_linear.py:221), and dequantization is exact
(one rounding) in every module.
"""
from __future__ import annotations

from typing import Any

import torch

from . import _lib
from .layers.fused_int4_linear import FusedInt4Linear, FusedInt4LinearAnyGroup, FusedInt4LinearPaddedGroups
from .layers import gemlite_available
from .layers.packed_gptq_linear import PackedGPTQLinear
from .quant_utils import dequant_gptq_to_fp

_DTYPES = {
    "float16": torch.float16,
    "fp16": torch.float16,
    "bfloat16": torch.bfloat16,
    "bf16": torch.bfloat16,
    "float32": torch.float32,
    "fp32": torch.float32,
}

_GEMLITE_BACKENDS = ("gemlite", "a8w4", "a8w4_ffn_up", "mxfp4_ffn", "mxfp4_ffn_up", "nvfp4_ffn")
BACKENDS = ("b200", "fused", "packed", "eager")


def resolve_dtype(dtype: str | torch.dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    try:
        return _DTYPES[str(dtype).lower()]
    except KeyError:
        raise ValueError(f"unsupported dtype: {dtype!r}")


def can_use_fused(entry: dict[str, Any]) -> bool:
    """True if a layer meets the reference's fused/gemlite kernel constraints (backend.py:60-68)."""
    return (
        not bool(entry.get("actorder", False))
        and int(entry["wbits"]) == 4
        and int(entry["groupsize"]) == 32
        and int(entry["in_features"]) % 32 == 0
        and int(entry["out_features"]) % 8 == 0
    )


def can_use_fused_any_group(entry: dict[str, Any]) -> bool:
    """True if the generic fused kernel can run this GPTQ int4 layer (backend.py:71-78)."""
    return (
        not bool(entry.get("actorder", False))
        and int(entry["wbits"]) == 4
        and int(entry["in_features"]) % 8 == 0
        and int(entry["out_features"]) % 8 == 0
    )


def can_use_fused_padded_groups(entry: dict[str, Any]) -> bool:
    """True if odd groups can be re-laid out onto the groupsize-32 kernel (backend.py:81-92)."""
    gs = int(entry["groupsize"])
    in_features = int(entry["in_features"])
    return (
        not bool(entry.get("actorder", False))
        and int(entry["wbits"]) == 4
        and gs != 32
        and 0 < gs < 32
        and in_features % gs == 0
        and int(entry["out_features"]) % 8 == 0
    )


def is_ffn_layer(entry: dict[str, Any]) -> bool:
    return ".ffn." in str(entry.get("name", ""))


def is_ffn_up_layer(entry: dict[str, Any]) -> bool:
    return ".ffn.net.0.proj" in str(entry.get("name", ""))


def resolve_backend(backend: str | None, use_fused: bool = True) -> str:
    """Pick the int4 GEMM backend. ``use_fused=False`` (legacy) forces eager; ``auto`` -> ``b200``."""
    if not use_fused:
        return "eager"
    b = (backend or "auto").lower()
    if b == "auto":
        return "b200"
    if b in _GEMLITE_BACKENDS:
        if not gemlite_available():
            raise RuntimeError(
                f"backend={b!r} requested but the 'gemlite' package is not importable; "
                "use backend='b200'")
        raise RuntimeError(f"backend={b!r}: the GemLite wrappers are not part of the B200 build; use backend='b200'")
    if b not in BACKENDS:
        raise ValueError(f"unknown backend: {backend!r}")
    return b


def _v1(entry: dict) -> bool:
    return entry.get("checkpoint_format", "gptq") != "gptq_v2"


def build_fused(entry: dict, st: dict, device: torch.device) -> FusedInt4Linear:
    return FusedInt4Linear(
        in_features=int(entry["in_features"]),
        out_features=int(entry["out_features"]),
        qweight=st["qweight"].to(device),
        scales=st["scales"].to(device=device, dtype=torch.float16),
        qzeros=st["qzeros"].to(device),
        bias=(st["bias"].to(device) if "bias" in st else None),
        groupsize=32,
        v1=_v1(entry),
    )


def build_fused_any_group(entry: dict, st: dict, device: torch.device) -> FusedInt4LinearAnyGroup:
    return FusedInt4LinearAnyGroup(
        in_features=int(entry["in_features"]),
        out_features=int(entry["out_features"]),
        qweight=st["qweight"].to(device),
        scales=st["scales"].to(device=device, dtype=torch.float16),
        qzeros=st["qzeros"].to(device),
        bias=(st["bias"].to(device) if "bias" in st else None),
        groupsize=int(entry["groupsize"]),
        v1=_v1(entry),
    )


def build_fused_padded_groups(entry: dict, st: dict, device: torch.device) -> FusedInt4LinearPaddedGroups:
    return FusedInt4LinearPaddedGroups(
        in_features=int(entry["in_features"]),
        out_features=int(entry["out_features"]),
        qweight=st["qweight"].to(device),
        scales=st["scales"].to(device=device, dtype=torch.float16),
        qzeros=st["qzeros"].to(device),
        bias=(st["bias"].to(device) if "bias" in st else None),
        groupsize=int(entry["groupsize"]),
        v1=_v1(entry),
    )


def build_eager(entry: dict, st: dict, dtype: torch.dtype, device: torch.device) -> torch.nn.Linear:
    in_f, out_f = int(entry["in_features"]), int(entry["out_features"])
    device = torch.device(device)
    g_idx = st.get("g_idx")
    if g_idx is None:
        gs = int(entry["groupsize"])
        g_idx = (torch.arange(in_f) // gs).to(torch.long)
    weight = dequant_gptq_to_fp(
        qweight=st["qweight"].to(device), scales=st["scales"].to(device), qzeros=st["qzeros"].to(device),
        g_idx=g_idx.to(device), in_features=in_f, out_features=out_f, dtype=dtype, v1=_v1(entry),
        wbits=int(entry.get("wbits", 4)),
    )
    has_bias = "bias" in st
    lin = torch.nn.Linear(in_f, out_f, bias=has_bias, device=device, dtype=dtype)
    with torch.no_grad():
        lin.weight.copy_(weight)
        if has_bias:
            lin.bias.copy_(st["bias"].to(dtype=dtype, device=device))
    return lin


def build_packed(entry: dict, st: dict, dtype: torch.dtype, device: torch.device) -> PackedGPTQLinear:
    in_f, out_f = int(entry["in_features"]), int(entry["out_features"])
    g_idx = st.get("g_idx")
    return PackedGPTQLinear(
        in_features=in_f,
        out_features=out_f,
        qweight=st["qweight"].to(device),
        scales=st["scales"].to(device=device, dtype=dtype),
        qzeros=st["qzeros"].to(device),
        g_idx=g_idx.to(device) if g_idx is not None else None,
        bias=(st["bias"].to(device) if "bias" in st else None),
        groupsize=int(entry["groupsize"]),
        wbits=int(entry["wbits"]),
        v1=_v1(entry),
    )


def build_quant_layer(entry: dict, st: dict, backend: str, dtype: torch.dtype, device: torch.device):
    """Dispatch a single quant-layer build, returning ``(module, kind)``.

    ``kind`` is ``"fused"``, ``"packed"`` or ``"eager"`` (reference backend.py:285-321).
    """
    device = torch.device(device)
    if backend in _GEMLITE_BACKENDS:
        resolve_backend(backend)  # raises
    _lib.require_b200(device)
    if backend in ("b200", "fused") and can_use_fused(entry):
        return build_fused(entry, st, device), "fused"
    if backend in ("b200", "fused") and can_use_fused_padded_groups(entry):
        return build_fused_padded_groups(entry, st, device), "fused"
    if backend in ("b200", "fused") and can_use_fused_any_group(entry):
        return build_fused_any_group(entry, st, device), "fused"
    if backend in ("b200", "fused", "packed"):
        return build_packed(entry, st, dtype, device), "packed"
    return build_eager(entry, st, dtype, device), "eager"
