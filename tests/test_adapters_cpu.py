"""Adapter reachability: a reference-style model adapter, placed outside the package and named
by ONECOMP_ADAPTERS_DIR, imports as onecomp_runtime.models.<name> and its relative imports bind
to this build's layers and dispatch (no GPU needed: import and class identity only)."""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

PKG = Path(__file__).resolve().parents[1] / "onecompression-runtime_b200"

ADAPTER = textwrap.dedent('''
    from ...backend import build_quant_layer, resolve_backend
    from ...layers.fused_int4_linear import FusedInt4Linear, FusedInt4LinearAnyGroup
    from ...layers.gemlite_int4_linear import GemLiteInt4Linear, gemlite_available
    from ...layers.packed_gptq_linear import PackedGPTQLinear
    from ...quant_utils import dequant_gptq_to_fp


    def pick(backend):
        return resolve_backend(backend), PackedGPTQLinear, FusedInt4Linear
''')

PROBE = textwrap.dedent('''
    import onecomp_runtime, onecomp_runtime.layers as L
    from onecomp_runtime.models.fake_adapter.loader import pick
    backend, packed, fused = pick("auto")
    assert packed is L.PackedGPTQLinear and fused is L.FusedInt4Linear, (packed, fused)
    assert backend == "b200", backend
    import onecomp_runtime.models as m
    print("OK", m.__name__, packed.__module__)
''')


def _tree(tmp_path: Path, layout: str) -> Path:
    base = {"root": tmp_path / "onecomp_runtime" / "models", "models": tmp_path}[layout]
    pkg = base / "fake_adapter"
    pkg.mkdir(parents=True)
    (pkg / "__init__.py").write_text("")
    (pkg / "loader.py").write_text(ADAPTER)
    return tmp_path if layout == "root" else base


def _run(adapters_dir: Path) -> subprocess.CompletedProcess:
    env = dict(os.environ, ONECOMP_ADAPTERS_DIR=str(adapters_dir),
               PYTHONPATH=str(PKG) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    return subprocess.run([sys.executable, "-c", PROBE], env=env, capture_output=True, text=True, timeout=300)


def test_adapter_from_checkout_root(tmp_path):
    r = _run(_tree(tmp_path, "root"))
    assert r.returncode == 0 and "OK onecomp_runtime.models onecomp_runtime.layers" in r.stdout, r.stderr[-2000:]


def test_adapter_from_models_dir(tmp_path):
    r = _run(_tree(tmp_path, "models"))
    assert r.returncode == 0, r.stderr[-2000:]


def test_no_adapters_without_env(tmp_path):
    sys.path.insert(0, str(PKG))
    from onecomp_runtime.models import adapter_dirs
    assert adapter_dirs("") == []
    assert adapter_dirs(str(tmp_path / "missing")) == []
