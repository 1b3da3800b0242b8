"""onecomp-runtime, B200 build -- the int4 linear hot path of OneCompression
checkpoints on NVIDIA B200 (sm_100a), behind the reference package's API.

    from onecomp_runtime.diffusion import load_int4_model
    from onecomp_runtime.layers import FusedInt4Linear, PackedGPTQLinear

Same import name, module layout and public symbols as the reference
``onecomp_runtime`` (kizuna-intelligence/onecompression-runtime); the compute
runs in the hand-written sm_100a kernels of ``liboc_b200.so`` (C ABI in
``include/oc_b200.h``). There is no CPU or Triton fallback.
"""
from __future__ import annotations

from . import backend, quant_utils
from .diffusion import load_int4_model
from .layers import (
    Dsv4PackedLinear,
    FusedInt4Linear,
    FusedInt4LinearAnyGroup,
    FusedInt4LinearPaddedGroups,
    GemLiteInt4Linear,
    PackedEmbedding,
    PackedGPTQLinear,
    PackedInt4Conv1d,
    PackedInt4ConvTranspose1d,
    PackedRTNLinear,
    dequant_dsv4_packed,
    fused_int4_gemm,
    gemlite_available,
    replace_conv_with_packed,
)

__version__ = "0.1.0+b200"

__all__ = [
    "load_int4_model",
    "FusedInt4Linear",
    "FusedInt4LinearAnyGroup",
    "FusedInt4LinearPaddedGroups",
    "fused_int4_gemm",
    "gemlite_available",
    "GemLiteInt4Linear",
    "PackedGPTQLinear",
    "PackedInt4Conv1d",
    "PackedInt4ConvTranspose1d",
    "replace_conv_with_packed",
    "PackedRTNLinear",
    "PackedEmbedding",
    "Dsv4PackedLinear",
    "dequant_dsv4_packed",
    "backend",
    "quant_utils",
]
