"""The C-ABI library loads and exports every entry point of include/oc_b200.h (no GPU needed)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "oc_b200.h"


def header_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(oc_b200_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from onecomp_runtime import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    fns = header_functions()
    assert "oc_b200_gptq_gemm" in fns and "oc_b200_gptq_dequant" in fns
    assert len(fns) >= 15


def test_library_exports_every_header_symbol(lib):
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_python_binding_covers_header():
    from onecomp_runtime import _lib
    assert sorted(_lib.exported_symbols()) == header_functions()


def test_abi_version_and_options(lib):
    from onecomp_runtime import _lib
    assert lib.oc_b200_abi_version() == 1
    assert lib.oc_b200_set_option(_lib.OPT_GEMM_PATH, 7) != 0
    assert "OC_OPT_GEMM_PATH" in _lib.last_error()
    assert lib.oc_b200_set_option(999, 0) != 0
    assert lib.oc_b200_set_option(_lib.OPT_GEMM_PATH, 0) == 0
    assert lib.oc_b200_set_option(_lib.OPT_TC_TILE, 100) != 0


def test_null_arguments_rejected_before_any_launch(lib):
    from onecomp_runtime import _lib
    rc = lib.oc_b200_gptq_dequant(None, None, None, 0, None, 8, 8, 1, 8, 4, 1, None, 1, None)
    assert rc == 1
    assert "NULL" in _lib.last_error()
    out = ctypes.c_void_p()
    rc = lib.oc_b200_gptq_layer_create(None, None, None, 0, None, None, 64, 64, 64, 2, 32, 1, ctypes.byref(out))
    assert rc == 1
    assert lib.oc_b200_gptq_gemm(None, None, 1, 1, 64, None, 0, None, 64, None, 0, None) == 1
    assert lib.oc_b200_gptq_gemm_workspace(None, 4) == 1024
