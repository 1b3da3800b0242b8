"""Model adapters: the reference's ``onecomp_runtime.models`` subpackages, run unchanged.

The adapters (Cosmos-Predict2.5 / Transfer2.5, Wan-VACE, FireRed, Qwen3.6, DeepSeek-V4) are
model-assembly code around the quantized layers and are not part of this build. Point
``ONECOMP_ADAPTERS_DIR`` at a reference checkout (its root, its ``onecomp_runtime`` directory or
its ``onecomp_runtime/models`` directory; several paths separated by ``os.pathsep``) and its
adapters import as ``onecomp_runtime.models.<name>``. Their relative imports (``...layers``,
``...backend``, ``...quant_utils``, ``...diffusion``) then resolve to this package, so every
quantized layer they build (``FusedInt4Linear``, ``PackedGPTQLinear``, ``Dsv4PackedLinear``, the
``build_quant_layer`` ladder) runs on the sm_100a kernels: FireRed's ``"fused"`` and Qwen3.6's
``"packed"`` backends reach B200 without an edit to the adapter.
"""
from __future__ import annotations

import os
from pathlib import Path


def adapter_dirs(spec: str | None = None) -> list[str]:
    """Directories holding adapter subpackages named by ``spec`` (default: the
    ``ONECOMP_ADAPTERS_DIR`` environment variable)."""
    spec = os.environ.get("ONECOMP_ADAPTERS_DIR", "") if spec is None else spec
    found: list[str] = []
    for entry in spec.split(os.pathsep):
        if not entry:
            continue
        root = Path(entry).expanduser()
        for cand in (root / "onecomp_runtime" / "models", root / "models", root):
            if cand.is_dir() and any((d / "__init__.py").is_file() for d in cand.iterdir() if d.is_dir()):
                found.append(str(cand.resolve()))
                break
    return found


__path__.extend(d for d in adapter_dirs() if d not in __path__)  # noqa: F821 (package __path__)
