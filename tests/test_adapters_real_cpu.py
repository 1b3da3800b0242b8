"""The reference's own model adapters, imported unchanged through ONECOMP_ADAPTERS_DIR.

FireRed (models/firered/loader.py:83-135), Qwen3.6 (models/qwen36/loader.py:93-158),
DeepSeek-V4 (models/dsv4/loader.py:109-119) and the Cosmos adapters are loaded from a
reference checkout; their relative imports must bind to this build, their backend whitelists
must resolve to the B200 modules, and their eager builders must reach this build's dequant
with the host tensors they pass (straight from safe_open). No GPU here: the dequant call is
expected to reach the B200 boundary and refuse to compute on the CPU.

Skipped when no reference checkout is present (the GPU box has none).
"""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

PKG = Path(__file__).resolve().parents[1] / "onecompression-runtime_b200"
REF = Path(os.environ.get("ONECOMP_REFERENCE_DIR", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REF / "onecomp_runtime" / "models" / "firered").is_dir(),
                                reason="no reference checkout with model adapters")

PROBE = textwrap.dedent('''
    import torch
    import onecomp_runtime as R
    import onecomp_runtime.layers as L
    from onecomp_runtime import quant_utils
    from onecomp_runtime.testing import gptq_layer
    import onecomp_runtime.models.firered.loader as FR
    import onecomp_runtime.models.qwen36.loader as QW
    import onecomp_runtime.models.dsv4.loader as DS
    import onecomp_runtime.models.cosmos_predict25.loader as CP

    # the adapters' names bind to this build
    assert FR.__file__.startswith(REF), FR.__file__
    assert FR.FusedInt4Linear is L.FusedInt4Linear
    assert FR.dequant_gptq_to_fp is quant_utils.dequant_gptq_to_fp
    assert QW.PackedGPTQLinear is L.PackedGPTQLinear
    assert QW.dequant_gptq_to_fp is quant_utils.dequant_gptq_to_fp
    assert DS.Dsv4PackedLinear is L.Dsv4PackedLinear
    # FireRed's whitelist: "auto" / "fused" reach the fused module (gemlite is absent)
    assert FR._resolve_backend("auto", True) == "fused"
    assert FR._resolve_backend("fused", True) == "fused"

    # FireRed's fused builder on host tensors: a B200 module with the checkpoint buffers verbatim
    t = gptq_layer(256, 128, 32, seed=3, bias=True)
    st = {"qweight": t["qweight"], "scales": t["scales"], "qzeros": t["qzeros"], "bias": t["bias"]}
    entry = {"in_features": 256, "out_features": 128, "groupsize": 32}
    m = FR._build_fused(entry, st, torch.device("cpu"))
    assert isinstance(m, L.FusedInt4Linear) and torch.equal(m.qweight, st["qweight"])

    # the eager builders pass host tensors to dequant_gptq_to_fp: on a box without an sm_100 GPU
    # that reaches this build's boundary and raises (no CPU fallback)
    for build in (lambda: FR._build_eager(entry, st, torch.bfloat16, torch.device("cpu")),
                  lambda: QW._build_eager(st, 256, 128, 4, 32, torch.bfloat16, torch.device("cpu"), True)):
        try:
            build()
        except RuntimeError as e:
            assert "no CPU fallback" in str(e) or "sm_100" in str(e), e
        else:
            assert torch.cuda.is_available(), "computed on the CPU"
    print("ADAPTERS OK")
''')


def test_reference_adapters_bind_to_this_build():
    env = dict(os.environ, ONECOMP_ADAPTERS_DIR=str(REF), PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=str(PKG) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    code = f"REF = {str(REF)!r}\n" + PROBE
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ADAPTERS OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
