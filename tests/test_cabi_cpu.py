"""The C-ABI library loads and exports every entry point of include/oc_b200.h (no GPU needed)."""
from __future__ import annotations

import ctypes
import re

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
    assert lib.oc_b200_gptq_gemm_workspace(None, 4) == 8192   # the ticket area alone


def test_layer_create_ex_validation(lib):
    """wbits and 8-bit layout checks happen on the host, before any device work (the pointers
    below are never dereferenced)."""
    from onecomp_runtime import _lib
    out = ctypes.c_void_p()
    qw, qz, sc = ctypes.c_void_p(0x10000), ctypes.c_void_p(0x20000), ctypes.c_void_p(0x30000)
    assert lib.oc_b200_gptq_layer_create_ex(qw, qz, sc, 0, None, None, 256, 256, 128, 8, 32, 3, 1,
                                            ctypes.byref(out)) != 0
    assert "wbits" in _lib.last_error()
    kp = ctypes.c_void_p(0x40000)
    assert lib.oc_b200_gptq_layer_create_ex(qw, qz, sc, 0, kp, None, 256, 264, 128, 8, 32, 8, 1,
                                            ctypes.byref(out)) != 0   # padding rows in the K order
    assert "K permutation" in _lib.last_error()
    assert lib.oc_b200_gptq_layer_create_ex(qw, qz, sc, 0, None, None, 256, 256, 128, 6, 48, 8, 1,
                                            ctypes.byref(out)) != 0
    assert "groupsize" in _lib.last_error()
    assert lib.oc_b200_gptq_layer_create_ex(qw, qz, sc, 0, None, None, 256, 256, 64, 8, 32, 8, 1,
                                            ctypes.byref(out)) != 0
    assert "N=64" in _lib.last_error()
    assert lib.oc_b200_gptq_layer_create_ex(qw, qz, sc, 0, None, None, 256, 256, 128, 7, 32, 8, 1,
                                            ctypes.byref(out)) != 0
    assert "G=7" in _lib.last_error()
    assert not out.value


def test_embedding_and_rtn_validation(lib):
    from onecomp_runtime import _lib
    p = ctypes.c_void_p(0x10000)
    # no ids: nothing to do, no device work
    assert lib.oc_b200_rtn_embedding(None, 0, 10, p, 32, p, 0, p, 0, 64, 1, p, 0, None) == 0
    assert lib.oc_b200_rtn_embedding(None, -1, 10, p, 32, p, 0, p, 0, 64, 1, p, 0, None) != 0
    assert lib.oc_b200_rtn_embedding(None, 4, 10, p, 32, p, 0, p, 0, 64, 1, p, 0, None) != 0
    assert "NULL" in _lib.last_error()
    assert lib.oc_b200_rtn_embedding(p, 4, 10, p, 32, p, 0, p, 0, 64, 3, p, 0, None) != 0
    assert "num_groups" in _lib.last_error()
    assert lib.oc_b200_rtn_embedding(p, 4, 10, p, 32, p, 0, p, 0, 64, 1, p, 9, None) != 0
    assert "dtype" in _lib.last_error()
    assert lib.oc_b200_rtn_dequant(p, 32, p, 0, p, 0, 64, 8, 1, p, 9, None) != 0
    assert "dtype" in _lib.last_error()


def test_gemv_noalloc_validation(lib):
    from onecomp_runtime import _lib
    assert lib.oc_b200_gptq_gemv_noalloc(None, None, 1, 1, 64, None, 0, None, 64, None) != 0
    assert "NULL" in _lib.last_error()


def test_moe_entry_points_validation(lib):
    """Routing / gather / SwiGLU / combine reject bad arguments before any launch, and an
    empty batch (with valid pointers) returns at once without device work."""
    from onecomp_runtime import _lib
    p = ctypes.c_void_p(0x10000)
    # route: logits [T, E] -> ids, weights [T, k]
    assert lib.oc_b200_moe_route(None, 1, 4, 8, 2, 1, p, p, None) != 0
    assert "NULL" in _lib.last_error()
    for T, E, k in ((-1, 8, 2), (4, 0, 1), (4, 2048, 2), (4, 8, 0), (4, 8, 17), (4, 4, 5)):
        assert lib.oc_b200_moe_route(p, 1, T, E, k, 1, p, p, None) != 0, (T, E, k)
    assert lib.oc_b200_moe_route(p, 7, 4, 8, 2, 1, p, p, None) != 0
    assert "dtype" in _lib.last_error()
    assert lib.oc_b200_moe_route(p, 1, 0, 8, 2, 1, p, p, None) == 0
    # permute: bad sizes
    assert lib.oc_b200_moe_permute(None, 4, 2, 8, p, p, p, p, None) != 0
    assert lib.oc_b200_moe_permute(p, 4, 2, 4096, p, p, p, p, None) != 0
    assert lib.oc_b200_moe_permute(p, -1, 2, 8, p, p, p, p, None) != 0
    # gather: 16-bit rows of H % 8 == 0, 16-byte aligned
    assert lib.oc_b200_gather_rows(p, 64, p, 4, 60, p, 64, None) != 0
    assert lib.oc_b200_gather_rows(ctypes.c_void_p(0x10002), 64, p, 4, 64, p, 64, None) != 0
    assert lib.oc_b200_gather_rows(p, 64, p, 0, 64, p, 64, None) == 0
    # silu * mul and combine: 16-bit only
    assert lib.oc_b200_silu_mul(p, p, 64, 4, 32, p, 32, 2, None) != 0
    assert lib.oc_b200_silu_mul(p, p, 64, 0, 32, p, 32, 1, None) == 0
    assert lib.oc_b200_moe_combine(p, 64, p, p, 4, 0, 64, None, 0, p, 64, 1, None) != 0
    assert lib.oc_b200_moe_combine(p, 64, p, p, 4, 2, 64, None, 0, p, 64, 2, None) != 0
    assert lib.oc_b200_moe_combine(None, 64, p, p, 4, 2, 64, None, 0, p, 64, 1, None) != 0
    assert lib.oc_b200_moe_combine(p, 64, p, p, 0, 2, 64, None, 0, p, 64, 1, None) == 0


def test_rows_layer_validation(lib):
    """The row-packed layer rejects unsupported layouts before it touches the device (the
    pointer arrays are not read on these paths)."""
    from onecomp_runtime import _lib
    p = ctypes.c_void_p(0x10000)
    out = ctypes.c_void_p()

    def create(E=2, wbits=2, ld=128, mode=0, K=512, N=256, gs=64, sdt=0, zdt=0, table=p, packed=p):
        return lib.oc_b200_rows_layer_create(E, packed, ld, wbits, p, sdt, p, zdt, 1, 256, gs, K, N, mode, table,
                                             None, ctypes.byref(out))

    assert lib.oc_b200_rows_layer_create(2, p, 128, 2, p, 0, p, 0, 1, 256, 64, 512, 256, 0, p, None, None) != 0
    cases = {
        "E=": dict(E=0), "E=2000": dict(E=2000), "NULL": dict(packed=None), "wbits": dict(wbits=3),
        "mode=": dict(mode=2), "RTN layers are 4-bit": dict(mode=1), "K=": dict(K=12),
        "row stride": dict(ld=64), "groupsize": dict(gs=24), "dtype": dict(sdt=7),
        "256-byte aligned": dict(table=ctypes.c_void_p(0x10010)),
    }
    for msg, kw in cases.items():
        assert create(**kw) != 0, kw
        assert msg.split("=")[0] in _lib.last_error(), (kw, _lib.last_error())
        assert not out.value
    assert lib.oc_b200_rows_gemm(None, p, 1, 4, 512, None, None, 0, p, 256, None) != 0
    assert lib.oc_b200_rows_table_bytes(0) == 0
    assert lib.oc_b200_rows_table_bytes(3) > 0 and lib.oc_b200_rows_table_bytes(3) % 256 == 0


def test_fused_entry_points_reject_bad_arguments_before_any_launch(lib):
    """The fused SwiGLU grouped GEMM and the all-reduce + RMS norm check their arguments on the host."""
    from onecomp_runtime import _lib
    assert lib.oc_b200_rows_gemm_swiglu(None, None, 1, 4, 64, None, None, 64, None) == 1
    assert "not a row-packed layer" in _lib.last_error()
    buf = ctypes.create_string_buffer(64)
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.oc_b200_gptq_repack_k_ex(p, p, 64, 128, 3, p, None) == 2          # wbits 4 or 8
    assert lib.oc_b200_gptq_repack_k_ex(None, p, 64, 128, 8, p, None) == 1       # NULL weights
    assert lib.oc_b200_gptq_repack_k_ex(p, p, 66, 128, 8, p, None) == 1          # k_packed % 4
    args = (p, 4, 4096, None, 1e-6, p, 0, 2, 1, 8, None)
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(None, *args[1:]) == 1          # no buffer
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(p, 4, 4100, *args[3:]) == 1     # cols not a multiple of 8
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(p, 4, 8192, *args[3:]) == 1     # wider than a warp's row
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(p, 4, 4096, None, -1.0, *args[5:]) == 1   # eps
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(*args[:6], 2, 2, *args[8:]) == 1   # rank outside the job
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(*args[:9], 65, None) == 1          # blocks
    assert lib.oc_b200_nvls_allreduce_rmsnorm_bf16(p, 0, 4096, *args[3:]) == 0        # no rows: nothing to do
