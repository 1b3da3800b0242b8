"""ctypes binding of the sm_100a C ABI (``include/oc_b200.h``, ``liboc_b200.so``).

The shared library is built in-tree by ``onecompression-runtime_b200/build.py``.
There is no CPU fallback: if the library is missing or the device is not an
sm_100 GPU, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).with_name("liboc_b200.so")

OC_OK = 0
DT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

OPT_GEMM_PATH = 1
OPT_TC_TILE = 2
OPT_GEMV_CTAS = 3
OPT_GEMV_IMPL = 4
OPT_TC_PAIR = 5
OPT_WAIT_US = 6
OPT_TEST_STALL = 7
OPT_TC_MAX_CTAS = 8
OPT_GEMV_PREP = 9
ACT_NONE = 0
ACT_GELU_TANH = 1

_lock = threading.Lock()
_lib = None

_c = ctypes
_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t

_SIGNATURES = {
    "oc_b200_abi_version": ([], _i),
    "oc_b200_last_error": ([], ctypes.c_char_p),
    "oc_b200_device_check": ([_i], _i),
    "oc_b200_set_option": ([_i, _i], _i),
    "oc_b200_get_option": ([_i, ctypes.POINTER(_i)], _i),
    "oc_b200_read_device_error": ([ctypes.POINTER(_i), _p], _i),
    "oc_b200_gptq_unpack": ([_p, _i, _i, _i, _p, _p], _i),
    "oc_b200_gptq_unpack_zeros": ([_p, _i, _i, _i, _p, _p], _i),
    "oc_b200_gptq_pack": ([_p, _i, _i, _i, _p, _p], _i),
    "oc_b200_gptq_dequant": ([_p, _p, _p, _i, _p, _i, _i, _i, _i, _i, _i, _p, _i, _p], _i),
    "oc_b200_rtn_dequant": ([_p, _i64, _p, _i, _p, _i, _i, _i, _i, _p, _i, _p], _i),
    "oc_b200_rtn_embedding": ([_p, _i64, _i64, _p, _i64, _p, _i, _p, _i, _i, _i, _p, _i, _p], _i),
    "oc_b200_dsv4_dequant": ([_p, _i64, _i, _p, _i, _p, _i, _i64, _i64, _i, _i, _i, _p, _i, _p], _i),
    "oc_b200_gptq_repack_k": ([_p, _p, _i, _i, _p, _p], _i),
    "oc_b200_gptq_repack_k_ex": ([_p, _p, _i, _i, _i, _p, _p], _i),
    "oc_b200_permute_cols": ([_p, _i64, _i64, _i, _p, _i, _p, _p], _i),
    "oc_b200_gptq_layer_create": ([_p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _i, ctypes.POINTER(_p)], _i),
    "oc_b200_gptq_layer_create_ex": ([_p, _p, _p, _i, _p, _p, _i, _i, _i, _i, _i, _i, _i, ctypes.POINTER(_p)], _i),
    "oc_b200_layer_destroy": ([_p], _i),
    "oc_b200_gptq_gemm_workspace": ([_p, _i64], _sz),
    "oc_b200_gptq_gemm": ([_p, _p, _i, _i64, _i64, _p, _i, _p, _i64, _p, _sz, _p], _i),
    "oc_b200_gptq_gemm_ex": ([_p, _p, _i, _i64, _i64, _p, _i, _p, _i64, _i, _p, _i64, _p, _sz, _p], _i),
    "oc_b200_gptq_gemv_noalloc": ([_p, _p, _i, _i64, _i64, _p, _i, _p, _i64, _p], _i),
    "oc_b200_rows_table_bytes": ([_i], _sz),
    "oc_b200_rows_layer_create": ([_i, _p, _i64, _i, _p, _i, _p, _i, _i64, _i64, _i, _i, _i, _i, _p, _p,
                                   ctypes.POINTER(_p)], _i),
    "oc_b200_rows_gemm": ([_p, _p, _i, _i64, _i64, _p, _p, _i, _p, _i64, _p], _i),
    "oc_b200_rows_gemm_swiglu": ([_p, _p, _i, _i64, _i64, _p, _p, _i64, _p], _i),
    "oc_b200_moe_route": ([_p, _i, _i, _i, _i, _i, _p, _p, _p], _i),
    "oc_b200_moe_permute": ([_p, _i, _i, _i, _p, _p, _p, _p, _p], _i),
    "oc_b200_gather_rows": ([_p, _i64, _p, _i, _i, _p, _i64, _p], _i),
    "oc_b200_silu_mul": ([_p, _p, _i64, _i, _i, _p, _i64, _i, _p], _i),
    "oc_b200_moe_combine": ([_p, _i64, _p, _p, _i, _i, _i, _p, _i64, _p, _i64, _i, _p], _i),
    "oc_b200_im2col_1d": ([_p, _i64, _i64, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _i64, _p], _i),
    "oc_b200_nvls_allreduce_bf16": ([_p, _i64, _p, _i, _i, ctypes.c_uint32, _i, _p], _i),
    "oc_b200_nvls_allreduce_rmsnorm_bf16": ([_p, _i, _i, _p, ctypes.c_float, _p, _i, _i, ctypes.c_uint32, _i, _p],
                                            _i),
}


def lib():
    """Load ``liboc_b200.so`` once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("ONECOMP_B200_LIB", str(LIB_PATH))
        if not Path(path).exists():
            raise RuntimeError(
                f"onecomp_runtime B200 library not found at {path}; build it with "
                "`python onecompression-runtime_b200/build.py` (nvcc, sm_100a)")
        handle = ctypes.CDLL(path)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = res
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    msg = lib().oc_b200_last_error()
    return msg.decode() if msg else ""


def check(rc: int, name: str) -> None:
    if rc != OC_OK:
        raise RuntimeError(f"{name}: {last_error()} (status {rc})")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_b200(device: torch.device) -> None:
    """Raise unless ``device`` is a CUDA sm_100 device and the library loads."""
    if device.type != "cuda":
        raise RuntimeError(
            f"onecomp_runtime (B200) runs on CUDA sm_100 devices only; got device {device}. "
            "There is no CPU fallback.")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    check(lib().oc_b200_device_check(idx), "oc_b200_device_check")


def set_option(key: int, value: int) -> None:
    call("oc_b200_set_option", key, value)


def get_option(key: int) -> int:
    v = _i(0)
    call("oc_b200_get_option", key, ctypes.byref(v))
    return v.value


def read_device_error(device: torch.device) -> int:
    code = _i(0)
    call("oc_b200_read_device_error", ctypes.byref(code), stream_of(device))
    return code.value


# ---------------------------------------------------------------- workspace pool
_ws: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A zero-initialised byte buffer per (device, current stream), grown on demand.

    Kernels on one stream run in order, so layers share it; the split-K tickets
    in its first 8 KiB are left at zero by every call.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_of(device))
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if buf is not None:
            size = max(size, buf.numel() * 2)
        buf = torch.zeros(size, dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf
