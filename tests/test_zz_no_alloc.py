"""oc_b200_gptq_gemv_noalloc: the decode GEMV with its scratch in a fixed device array.

Called through the C ABI; each case runs it twice in a row (the second call reuses the
tickets the first one left at zero) and compares both outputs with oc_b200_gptq_gemm on a
caller workspace. Named to be collected last, so it also runs after every other GPU test
has used the library on the same device.
"""
from __future__ import annotations

import pytest
import torch

from gpu_util import GEMM_TOL

pytestmark = pytest.mark.gpu


def _layer(t, K, N, gs, v1, actorder, device):
    from onecomp_runtime.layers import FusedInt4Linear, FusedInt4LinearAnyGroup, PackedGPTQLinear
    tc = {k: v.to(device) for k, v in t.items()}
    if actorder:
        return PackedGPTQLinear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc["g_idx"], tc.get("bias"), gs, 4,
                                v1)
    cls = FusedInt4Linear if gs == 32 else FusedInt4LinearAnyGroup
    return cls(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc.get("bias"), gs, v1=v1)


def _noalloc(layer, x, out):
    from onecomp_runtime import _lib
    bias = layer.bias
    return _lib.lib().oc_b200_gptq_gemv_noalloc(
        layer._get_handle(), x.data_ptr(), _lib.DT[x.dtype], x.shape[0], x.stride(0),
        None if bias is None else bias.data_ptr(), _lib.DT[bias.dtype] if bias is not None else 0,
        out.data_ptr(), out.stride(0), _lib.stream_of(x.device))


CASES = [
    # M, K, N, gs, v1, act-order, activation dtype
    (1, 3072, 3072, 32, True, False, torch.bfloat16),
    (4, 5120, 8192, 128, False, True, torch.bfloat16),
    (9, 1024, 392, 64, True, False, torch.float16),
    (16, 17408, 5120, 128, False, True, torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"M{c[0]}K{c[1]}N{c[2]}g{c[3]}")
def test_noalloc_matches_workspace_entry(cuda_device, case):
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import activations, gptq_layer
    M, K, N, gs, v1, act, dt = case
    t = gptq_layer(K, N, gs, seed=500 + M, v1=v1, actorder=act, bias=True)
    layer = _layer(t, K, N, gs, v1, act, cuda_device)
    x = activations(M, K, seed=M, dtype=dt).to(cuda_device)
    ref = layer(x)                       # oc_b200_gptq_gemm with a caller workspace
    outs = []
    for _ in range(2):                   # two calls in a row on the same scratch
        out = torch.full((M, N), float("nan"), dtype=dt, device=cuda_device)
        _lib.check(_noalloc(layer, x, out), "oc_b200_gptq_gemv_noalloc")
        outs.append(out)
    torch.cuda.synchronize(cuda_device)
    scale = ref.float().abs().max()
    for out in outs:
        assert torch.isfinite(out.float()).all()
        err = float((out.float() - ref.float()).abs().max() / scale)
        assert err < GEMM_TOL, err
    assert _lib.read_device_error(cuda_device) == 0


def test_noalloc_rejects_oversize(cuda_device):
    """M > 16, and a split plan whose partials exceed the fixed scratch, fail with a message."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import activations, gptq_layer
    K, N = 8192, 16384
    t = gptq_layer(K, N, 128, seed=3, bias=False, device=cuda_device)
    layer = _layer(t, K, N, 128, True, False, cuda_device)
    x = activations(32, K, seed=1).to(cuda_device)
    out = torch.empty((32, N), dtype=torch.bfloat16, device=cuda_device)
    assert _noalloc(layer, x, out) != 0
    assert "M=32" in _lib.last_error()
    saved = {k: _lib.get_option(k) for k in (_lib.OPT_GEMV_IMPL, _lib.OPT_GEMV_CTAS)}
    try:
        # the cp.async GEMV with many splits: 16 rows x 16384 x splits fp32 partials
        _lib.set_option(_lib.OPT_GEMV_IMPL, 2)
        _lib.set_option(_lib.OPT_GEMV_CTAS, 16)
        assert _noalloc(layer, x[:16], out[:16]) != 0
        assert "bytes of scratch" in _lib.last_error()
    finally:
        for k, v in saved.items():   # whatever was set before this test
            _lib.set_option(k, v)
    _lib.check(_noalloc(layer, x[:16], out[:16]), "oc_b200_gptq_gemv_noalloc")
    ref = layer(x[:16]).float()
    err = float((out[:16].float() - ref).abs().max() / ref.abs().max())
    assert err < GEMM_TOL, err
