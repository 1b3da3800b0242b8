"""Int4 inference layers on B200 (sm_100a), same names as the reference
``onecomp_runtime/layers/__init__.py:20-57``:

- :class:`FusedInt4Linear` / :func:`fused_int4_gemm` -- AutoGPTQ int4, groupsize 32;
- :class:`FusedInt4LinearAnyGroup` / :class:`FusedInt4LinearPaddedGroups` -- other groupsizes;
- :class:`PackedGPTQLinear` -- 4/8-bit, any groupsize, act-order, v1/v2;
- :class:`PackedRTNLinear` / :class:`PackedEmbedding` -- RTN uint8-nibble layers;
- :class:`Dsv4PackedLinear` / :func:`dequant_dsv4_packed` -- int4/int2 byte-packed layers;
- :class:`PackedInt4Conv1d` / :class:`PackedInt4ConvTranspose1d` and the conv codec helpers.

GemLite is not part of this build: ``GemLiteInt4Linear`` imports but raises on construction
and ``gemlite_available()`` reports whether GemLite is importable.
"""
from __future__ import annotations

from .dsv4_packed_linear import Dsv4PackedLinear, dequant_dsv4_packed
from .fused_int4_linear import (
    FusedInt4Linear,
    FusedInt4LinearAnyGroup,
    FusedInt4LinearPaddedGroups,
    fused_int4_gemm,
)
from .gemlite_int4_linear import GemLiteInt4Linear, gemlite_available
from .packed_conv import (
    PackedInt4Conv1d,
    PackedInt4ConvTranspose1d,
    quantize_conv_module,
    quantize_conv_weight,
    replace_conv_with_packed,
)
from .packed_gptq_linear import PackedGPTQLinear
from .packed_linear import PackedEmbedding, PackedRTNLinear


__all__ = [
    "FusedInt4Linear",
    "FusedInt4LinearAnyGroup",
    "FusedInt4LinearPaddedGroups",
    "fused_int4_gemm",
    "gemlite_available",
    "GemLiteInt4Linear",
    "PackedInt4Conv1d",
    "PackedInt4ConvTranspose1d",
    "quantize_conv_module",
    "quantize_conv_weight",
    "replace_conv_with_packed",
    "PackedGPTQLinear",
    "PackedRTNLinear",
    "PackedEmbedding",
    "Dsv4PackedLinear",
    "dequant_dsv4_packed",
]
