"""Int4 inference layers on B200 (sm_100a), same names as the reference
``onecomp_runtime/layers/__init__.py:20-57``:

- :class:`FusedInt4Linear` / :func:`fused_int4_gemm` -- AutoGPTQ int4, groupsize 32;
- :class:`FusedInt4LinearAnyGroup` / :class:`FusedInt4LinearPaddedGroups` -- other groupsizes;
- :class:`PackedGPTQLinear` -- 4/8-bit, any groupsize, act-order, v1/v2;
- :class:`PackedRTNLinear` / :class:`PackedEmbedding` -- RTN uint8-nibble layers;
- :class:`Dsv4PackedLinear` / :func:`dequant_dsv4_packed` -- int4/int2 byte-packed layers.

The GemLite wrappers and the int4 conv codecs of the reference are not part of
this build (``gemlite_available()`` reports whether GemLite is importable).
"""
from __future__ import annotations

from .dsv4_packed_linear import Dsv4PackedLinear, dequant_dsv4_packed
from .fused_int4_linear import (
    FusedInt4Linear,
    FusedInt4LinearAnyGroup,
    FusedInt4LinearPaddedGroups,
    fused_int4_gemm,
)
from .packed_gptq_linear import PackedGPTQLinear
from .packed_linear import PackedEmbedding, PackedRTNLinear


def gemlite_available() -> bool:
    try:
        import gemlite  # noqa: F401
    except Exception:
        return False
    return True


__all__ = [
    "FusedInt4Linear",
    "FusedInt4LinearAnyGroup",
    "FusedInt4LinearPaddedGroups",
    "fused_int4_gemm",
    "gemlite_available",
    "PackedGPTQLinear",
    "PackedRTNLinear",
    "PackedEmbedding",
    "Dsv4PackedLinear",
    "dequant_dsv4_packed",
]
