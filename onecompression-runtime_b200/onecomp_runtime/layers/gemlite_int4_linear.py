"""Import-compatible stand-in for the reference's GemLite wrapper.

GemLite (a Triton library) is not part of the B200 build. As with the reference when the
``gemlite`` package is missing (gemlite_int4_linear.py:36-50 imports it in ``__init__``),
the name imports and constructing it raises ``ImportError``; ``backend.resolve_backend``
rejects the GemLite backends the same way.
"""
from __future__ import annotations

from torch import nn


def gemlite_available() -> bool:
    try:
        import gemlite  # noqa: F401
    except Exception:
        return False
    return True


class GemLiteInt4Linear(nn.Module):
    def __init__(self, *args, **kwargs) -> None:
        raise ImportError("GemLiteInt4Linear needs the gemlite package, which is not part of the B200 build; "
                          "use FusedInt4Linear (backend='b200')")
