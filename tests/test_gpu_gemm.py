"""GEMM parity on the GPU: split-K GEMV (M <= 16) and the tcgen05 kernel against the oracle.

Reference: fp64-accumulated ``x @ W.T + b`` where ``W`` is the oracle's exact
dequantized weight (bit-identical to quant_utils.dequant_gptq_to_fp); the bar is
max-abs-relative error <= 2e-2 (north star), and the tests also bound it to
1e-2 to catch layout bugs that stay inside the loose bound.
"""
from __future__ import annotations

import pytest
import torch

from conftest import GPTQ_CASES, load_golden
from gpu_util import GEMM_TOL, NAME, TDT, max_abs_rel, oracle_weight, reference_output, to_torch
from oracle import eager, gptq

pytestmark = pytest.mark.gpu


@pytest.fixture
def path_option():
    from onecomp_runtime import _lib
    yield lambda v: _lib.set_option(_lib.OPT_GEMM_PATH, v)
    _lib.set_option(_lib.OPT_GEMM_PATH, 0)
    _lib.set_option(_lib.OPT_TC_TILE, 0)


def _module(t, K, N, gs, v1, kind, device):
    from onecomp_runtime.layers import FusedInt4Linear, FusedInt4LinearAnyGroup, PackedGPTQLinear
    tc = {k: v.to(device) for k, v in t.items()}
    if kind == "fused":
        return FusedInt4Linear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc.get("bias"), 32, v1=v1)
    if kind == "any":
        return FusedInt4LinearAnyGroup(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc.get("bias"), gs, v1=v1)
    return PackedGPTQLinear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc["g_idx"], tc.get("bias"), gs,
                            4, v1)


@pytest.mark.parametrize("case", [c for c in GPTQ_CASES if load_golden(c)["meta"]["M"]])
@pytest.mark.parametrize("path", [1, 2])
def test_golden_cases(cuda_device, case, path, path_option):
    d = load_golden(case)
    m = d["meta"]
    if path == 1 and m["M"] > 16:
        pytest.skip("GEMV path takes M <= 16")
    path_option(path)
    from onecomp_runtime.layers import PackedGPTQLinear
    qw = torch.from_numpy(d["qweight"]).to(cuda_device)
    qz = torch.from_numpy(d["qzeros"]).to(cuda_device)
    s = to_torch(d["scales"], m["scales_dtype"])
    gi = torch.from_numpy(d["g_idx"]).to(cuda_device)
    bias = to_torch(d["bias_f16"], "f16") if "bias_f16" in d else None
    layer = PackedGPTQLinear(m["K"], m["N"], qw, s, qz, gi, bias, m["gs"], m["wbits"], m["v1"])
    for od in m["out_dtypes"]:
        x = to_torch(d[f"x_{od}"], od)
        y = layer(x)
        assert y.dtype == TDT[od] and y.shape == (m["M"], m["N"])
        ref = reference_output(x, d[f"w_{od}"], od, bias)
        err = max_abs_rel(y, ref)
        assert err < 1e-2, (case, od, err)
        # and against the reference's own eager (CPU bf16 nn.Linear) output
        from oracle.fp import to_f32
        assert eager.max_abs_rel(y.float().cpu().numpy(), to_f32(d[f"y_{od}"], od)) < GEMM_TOL


SHAPES = [
    # M, K, N, gs, v1, actorder, act dtype, scales dtype, bias
    (1, 256, 128, 32, True, False, torch.bfloat16, torch.float16, True),
    (5, 512, 200, 32, True, False, torch.bfloat16, torch.float16, True),
    (8, 384, 136, 128, False, True, torch.bfloat16, torch.bfloat16, False),
    (9, 1024, 256, 32, True, False, torch.float16, torch.float16, True),
    (16, 2048, 384, 128, False, True, torch.bfloat16, torch.float16, True),
    (17, 512, 256, 32, True, False, torch.bfloat16, torch.float16, True),
    (100, 768, 392, 64, True, False, torch.float16, torch.bfloat16, True),
    (193, 1024, 256, 32, True, False, torch.bfloat16, torch.float16, False),
    (300, 520, 128, 26, True, False, torch.bfloat16, torch.float16, True),
    (512, 1536, 640, 128, False, True, torch.bfloat16, torch.bfloat16, True),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"M{s[0]}K{s[1]}N{s[2]}g{s[3]}")
@pytest.mark.parametrize("path", [0, 2])
def test_shapes(cuda_device, shape, path, path_option):
    M, K, N, gs, v1, act, adt, sdt, has_bias = shape
    from onecomp_runtime.testing import gptq_layer, activations
    path_option(path)
    t = gptq_layer(K, N, gs, seed=M * 7 + K, v1=v1, actorder=act, bias=has_bias, scales_dtype=sdt)
    kind = "packed" if (act or gs % 8) else ("fused" if gs == 32 else "any")
    if gs % 8:
        from onecomp_runtime.layers import FusedInt4LinearPaddedGroups
        tc = {k: v.to(cuda_device) for k, v in t.items()}
        layer = FusedInt4LinearPaddedGroups(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc.get("bias"), gs, v1=v1)
    else:
        layer = _module(t, K, N, gs, v1, kind, cuda_device)
    x = activations(M, K, seed=M, dtype=adt).to(cuda_device)
    y = layer(x)
    w = oracle_weight(t, K, N, NAME[adt], v1=v1)
    ref = reference_output(x, w, NAME[adt], layer.bias)
    err = max_abs_rel(y, ref)
    assert err < 1e-2, err


SHAPES8 = [
    # M, K, N, gs, v1, act dtype, scales dtype, bias
    (1, 4096, 4096, 128, True, torch.bfloat16, torch.bfloat16, False),
    (3, 1000, 256, 32, True, torch.bfloat16, torch.float16, True),     # K not a multiple of the 64-k stage
    (8, 2048, 384, 64, False, torch.float16, torch.float16, True),
    (9, 1536, 640, 192, True, torch.bfloat16, torch.bfloat16, True),   # 3 stages per group
    (16, 4096, 1024, 32, False, torch.float16, torch.bfloat16, False),
    (4, 2048, 256, 256, False, torch.bfloat16, torch.bfloat16, True),  # a group spans 4 stages
    # M > 16: the tcgen05 GEMM with 8-bit stages (128- and 384-token presets)
    (17, 512, 256, 32, True, torch.bfloat16, torch.float16, True),
    (96, 640, 256, 64, False, torch.bfloat16, torch.bfloat16, False),
    (200, 1024, 384, 32, True, torch.float16, torch.float16, True),
    (700, 2048, 512, 128, False, torch.bfloat16, torch.float16, True),
]


@pytest.mark.parametrize("shape", SHAPES8, ids=lambda s: f"M{s[0]}K{s[1]}N{s[2]}g{s[3]}")
def test_gemv_8bit(cuda_device, shape):
    """8-bit PackedGPTQLinear (decode GEMV for M <= 16, tcgen05 GEMM above) against the oracle weights."""
    M, K, N, gs, v1, adt, sdt, has_bias = shape
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import activations, gptq_layer
    t = gptq_layer(K, N, gs, seed=M * 13 + K, v1=v1, bias=has_bias, scales_dtype=sdt, wbits=8)
    tc = {k: v.to(cuda_device) for k, v in t.items()}
    layer = PackedGPTQLinear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc["g_idx"], tc.get("bias"), gs, 8, v1)
    x = activations(M, K, seed=M, dtype=adt).to(cuda_device)
    assert layer._use_kernel8(x, M)  # every SHAPES8 M is within the kernels' range
    y = layer(x)
    assert y.dtype == adt and y.shape == (M, N)
    w = oracle_weight(t, K, N, NAME[adt], v1=v1, wbits=8)
    ref = reference_output(x, w, NAME[adt], layer.bias)
    err = max_abs_rel(y, ref)
    assert err < 1e-2, err
    assert _lib.read_device_error(cuda_device) == 0
    # a second call on the same workspace (split-K tickets re-armed) gives the same result
    assert torch.equal(layer(x), y)


@pytest.mark.parametrize("shape", [(1, 4096, 1024, 128), (9, 2048, 384, 64), (64, 2048, 512, 128),
                                   (700, 1536, 256, 32)], ids=lambda s: f"M{s[0]}K{s[1]}N{s[2]}g{s[3]}")
def test_gptq_8bit_act_order(cuda_device, shape):
    """8-bit act-order layers (g_idx a permutation of k // groupsize) run the 8-bit decode GEMV or
    tcgen05 GEMM on rows re-laid out by group (oc_b200_gptq_repack_k_ex) with the activation
    columns gathered; against the oracle's exact weights. A g_idx whose groups do not all hold
    groupsize rows keeps the dequant + F.linear path, also within tolerance."""
    M, K, N, gs = shape
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import activations, gptq_layer
    t = gptq_layer(K, N, gs, seed=M + K, v1=False, actorder=True, scales_dtype=torch.float16, wbits=8)
    tc = {k: v.to(cuda_device) for k, v in t.items()}
    layer = PackedGPTQLinear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], tc["g_idx"], tc.get("bias"), gs, 8,
                             False)
    x = activations(M, K, seed=M).to(cuda_device)
    assert layer._kperm8 is not None and layer._use_kernel8(x, M)
    y = layer(x)
    w = oracle_weight(t, K, N, "bf16", v1=False, wbits=8)
    assert max_abs_rel(y, reference_output(x, w, "bf16", layer.bias)) < 1e-2
    assert torch.equal(layer(x), y)
    # uneven groups: the first two groups swap one row each way, then one row moves from group 0
    g2 = t["g_idx"].clone()
    g2[int((g2 == 0).nonzero()[0])] = 1
    t2 = dict(t, g_idx=g2)
    layer2 = PackedGPTQLinear(K, N, tc["qweight"], tc["scales"], tc["qzeros"], g2.to(cuda_device), tc.get("bias"),
                              gs, 8, False)
    assert not layer2._kernel8_ok
    w2 = oracle_weight(t2, K, N, "bf16", v1=False, wbits=8)
    assert max_abs_rel(layer2(x), reference_output(x, w2, "bf16", layer2.bias)) < 1e-2
    assert _lib.read_device_error(cuda_device) == 0


def test_gemv_8bit_layer_errors(cuda_device):
    """8-bit handles refuse the layouts their kernels do not cover, with an error (no launch)."""
    import ctypes
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer
    t = {k: v.to(cuda_device) for k, v in gptq_layer(256, 128, 32, wbits=8, scales_dtype=torch.float16).items()}
    lib = _lib.lib()
    h = ctypes.c_void_p()
    kperm = torch.arange(264, dtype=torch.int32, device=cuda_device)
    args = (t["qweight"].data_ptr(), t["qzeros"].data_ptr(), t["scales"].data_ptr(), _lib.DT[torch.float16])
    # a K permutation with padding rows (k_packed > in_features): no 8-bit kernel takes it
    assert lib.oc_b200_gptq_layer_create_ex(*args, kperm.data_ptr(), None, 256, 264, 128, 8, 32, 8, 1,
                                            ctypes.byref(h)) != 0
    assert b"K permutation" in lib.oc_b200_last_error()
    assert lib.oc_b200_gptq_layer_create_ex(*args, None, None, 256, 256, 128, 8, 48, 8, 1, ctypes.byref(h)) != 0
    assert lib.oc_b200_gptq_layer_create_ex(*args, None, None, 256, 256, 128, 8, 32, 6, 1, ctypes.byref(h)) != 0
    assert lib.oc_b200_gptq_layer_create_ex(*args, None, None, 256, 256, 128, 8, 32, 8, 1, ctypes.byref(h)) == 0
    try:
        assert lib.oc_b200_gptq_gemm_workspace(h, 17) >= 1024
    finally:
        lib.oc_b200_layer_destroy(h)


@pytest.mark.parametrize("tile", [128, 192, 256, 384, 448])
def test_tc_tiles(cuda_device, tile, path_option):
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    path_option(2)
    _lib.set_option(_lib.OPT_TC_TILE, tile)
    M, K, N = 700, 1024, 384
    t = gptq_layer(K, N, 32, seed=tile)
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=5).to(cuda_device)
    y = layer(x)
    ref = reference_output(x, oracle_weight(t, K, N, "bf16"), "bf16", layer.bias)
    assert max_abs_rel(y, ref) < 1e-2


def test_cfg0_fused_linear(cuda_device):
    """Config 0: K=N=3072, gs=32, v1, M=256 bf16 through FusedInt4Linear."""
    from onecomp_runtime.testing import gptq_layer, activations
    t = gptq_layer(3072, 3072, 32, seed=0)
    layer = _module(t, 3072, 3072, 32, True, "fused", cuda_device)
    x = activations(256, 3072, seed=1).to(cuda_device)
    y = layer(x)
    ref = reference_output(x, oracle_weight(t, 3072, 3072, "bf16"), "bf16", layer.bias)
    assert max_abs_rel(y, ref) < 1e-2


def _gpu_reference(t, K, N, x, v1, bias=None):
    """fp64 GEMM of the bit-exact GPU-dequantized weight (dequant pinned by test_gpu_dequant)."""
    from onecomp_runtime import quant_utils
    w = quant_utils.dequant_gptq_to_fp(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N, x.dtype, v1=v1)
    ref = x.double() @ w.double().t()
    if bias is not None:
        ref = ref + bias.double()
    return ref


@pytest.mark.parametrize("M", [1, 4, 16])
def test_cfg2_decode_layers(cuda_device, M):
    """Config 2: gptq_v2, gs=128, act-order, scales in bf16 (as backend.build_packed stores them)."""
    from onecomp_runtime.testing import CFG2_LAYERS, gptq_layer, activations
    for i, (name, K, N) in enumerate(CFG2_LAYERS):
        t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 128, seed=2000 + i, v1=False, actorder=True,
                                                         scales_range=(0.001, 0.01), scales_dtype=torch.bfloat16,
                                                         bias=False).items()}
        layer = _module(t, K, N, 128, False, "packed", cuda_device)
        x = activations(M, K, seed=M + i).to(cuda_device)
        y = layer(x)
        ref = _gpu_reference(t, K, N, x, False)
        err = float((y.double() - ref).abs().max() / ref.abs().max())
        assert err < 1e-2, (name, err)


def test_full_size_vs_torch_fp32(cuda_device):
    """Config-1 qkv layer at full M: the tcgen05 kernel vs a torch fp32 GEMM of the exact weight."""
    from onecomp_runtime import quant_utils
    from onecomp_runtime.testing import gptq_layer, activations
    K, N, M = 3072, 9216, 4608
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 32, seed=77, device="cpu").items()}
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=3).to(cuda_device)
    y = layer(x)
    w = quant_utils.dequant_gptq_to_fp(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N, torch.bfloat16)
    ref = x.float() @ w.float().t() + t["bias"].float()
    err = float((y.float() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err


def test_module_api(cuda_device):
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(256, 128, 32, seed=9)
    layer = _module(t, 256, 128, 32, True, "fused", cuda_device)
    x3 = torch.randn(2, 3, 256, device=cuda_device, dtype=torch.bfloat16)
    y3 = layer(x3)
    assert y3.shape == (2, 3, 128)
    torch.testing.assert_close(y3.reshape(6, 128), layer(x3.reshape(6, 256)), rtol=0, atol=0)
    y32 = layer(x3.float())
    assert y32.dtype == torch.float32
    y0 = layer(torch.empty(0, 256, device=cuda_device, dtype=torch.bfloat16))
    assert y0.shape == (0, 128)
    xs = torch.randn(4, 512, device=cuda_device, dtype=torch.bfloat16)[:, ::2]
    torch.testing.assert_close(layer(xs), layer(xs.contiguous()), rtol=0, atol=0)


def test_fused_int4_gemm_functional(cuda_device):
    from onecomp_runtime.layers import fused_int4_gemm
    from onecomp_runtime.testing import gptq_layer, activations
    t = {k: v.to(cuda_device) for k, v in gptq_layer(512, 256, 32, seed=4).items()}
    x = activations(40, 512, seed=2, dtype=torch.float16).to(cuda_device)
    y = fused_int4_gemm(x, t["qweight"], t["scales"], t["qzeros"], t["bias"], 32)
    ref = reference_output(x, oracle_weight({k: v.cpu() for k, v in t.items()}, 512, 256, "f16"), "f16",
                           t["bias"])
    assert y.dtype == torch.float16 and max_abs_rel(y, ref) < 1e-2


def test_no_device_errors_recorded(cuda_device):
    from onecomp_runtime import _lib
    assert _lib.read_device_error(cuda_device) == 0


@pytest.mark.parametrize("M", [3, 16, 300])
@pytest.mark.parametrize("act", [None, "gelu_tanh"])
@pytest.mark.parametrize("residual", ["none", "dense", "strided"])
def test_fused_epilogue(cuda_device, M, act, residual):
    """oc_b200_gptq_gemm_ex: act(x @ W.T + b) + residual computed in the GEMM epilogue
    (GEMV for M <= 16, tcgen05 above) against the fp64 GEMM of the exact weight. A residual
    whose row pitch is not a multiple of 8 elements takes the direct-store epilogue."""
    from onecomp_runtime.testing import gptq_layer, activations
    K, N = 1024, 384
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 32, seed=11 + M).items()}
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=M).to(cuda_device)
    r = None
    if residual == "dense":
        r = activations(M, N, seed=M + 1).to(cuda_device)
    elif residual == "strided":
        r = activations(M, N + 4, seed=M + 1).to(cuda_device)[:, :N]
    y = layer.forward_fused(x, residual=r, activation=act)
    ref = _gpu_reference(t, K, N, x, True, t["bias"])
    if act == "gelu_tanh":
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    if r is not None:
        ref = ref + r.double()
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert y.dtype == x.dtype and y.shape == (M, N)
    assert err < 1e-2, err
    if act is None and r is None:
        torch.testing.assert_close(y, layer(x), rtol=0, atol=0)


@pytest.mark.parametrize("tile", [192, 384, 448])
@pytest.mark.parametrize("M", [200, 1000])
def test_tc_tiles_fused_epilogue(cuda_device, tile, M, path_option):
    """Every tile preset (one and two sub-tiles) with a residual + GELU epilogue, partial last tile."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    path_option(2)
    _lib.set_option(_lib.OPT_TC_TILE, tile)
    K, N = 768, 384
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 32, seed=tile + M).items()}
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=M).to(cuda_device)
    r = activations(M, N, seed=M + 7).to(cuda_device)
    y = layer.forward_fused(x, residual=r, activation="gelu_tanh")
    ref = torch.nn.functional.gelu(_gpu_reference(t, K, N, x, True, t["bias"]), approximate="tanh") + r.double()
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err


GEMV_IMPL_SHAPES = [
    # M, K, N, gs, v1, act-order, scales dtype
    (1, 3072, 3072, 32, True, False, torch.float16),
    (3, 1024, 384, 64, True, False, torch.float16),
    (8, 5120, 1024, 128, False, True, torch.bfloat16),
    (11, 4096, 640, 256, False, False, torch.bfloat16),
    (16, 2176, 512, 128, False, True, torch.float16),
    (2, 6144, 256, 512, True, False, torch.float16),     # a group spans 4 stages
    (5, 4160, 384, 64, True, False, torch.bfloat16),     # K not a multiple of the 128-k stage
    (4, 5120, 17408, 128, False, True, torch.float16),   # config-2 gate shape: several activation pieces
    (13, 8192, 2048, 64, True, False, torch.bfloat16),   # two token tiles, two groups per stage
    (1, 256, 256, 128, False, True, torch.float16),      # fewer units than SMs
    (16, 17408, 512, 128, True, False, torch.float16),   # a run spans many K stages of one tile
]


@pytest.mark.parametrize("impl", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("shape", GEMV_IMPL_SHAPES, ids=lambda s: f"M{s[0]}K{s[1]}N{s[2]}g{s[3]}")
def test_gemv_impls(cuda_device, impl, shape):
    """The five decode kernels for uniform-group layers (tcgen05, TMA + mma.sync split-K, cp.async
    + mma.sync, stream-K with the act-order gather inside -- layers narrower than 256 columns run
    the split-K TMA kernel under 3 --, and the integer-MMA kernel on prepared activation digits)
    against the fp64 GEMM of the exact weight, with a residual + GELU epilogue."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    M, K, N, gs, v1, act, sdt = shape
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, gs, seed=K + N + M, v1=v1, actorder=act,
                                                     scales_dtype=sdt).items()}
    layer = _module(t, K, N, gs, v1, "packed" if act else ("fused" if gs == 32 else "any"), cuda_device)
    x = activations(M, K, seed=M).to(cuda_device)
    r = activations(M, N, seed=M + 3).to(cuda_device)
    saved = _lib.get_option(_lib.OPT_GEMV_IMPL)
    _lib.set_option(_lib.OPT_GEMV_IMPL, impl)
    try:
        y = layer(x)
        yf = layer.forward_fused(x, residual=r, activation="gelu_tanh")
    finally:
        _lib.set_option(_lib.OPT_GEMV_IMPL, saved)
    ref = _gpu_reference(t, K, N, x, v1, t["bias"])
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    reff = torch.nn.functional.gelu(ref, approximate="tanh") + r.double()
    errf = float((yf.double() - reff).abs().max() / reff.abs().max())
    assert errf < 1e-2, errf
    assert _lib.read_device_error(cuda_device) == 0


@pytest.fixture
def pair_option():
    from onecomp_runtime import _lib
    yield lambda v: _lib.set_option(_lib.OPT_TC_PAIR, v)
    _lib.set_option(_lib.OPT_TC_PAIR, 1)


@pytest.mark.parametrize("tile", [256, 384, 448])
@pytest.mark.parametrize("M", [200, 1000])
def test_tc_pairs(cuda_device, tile, M, path_option, pair_option):
    """The tcgen05 GEMM on CTA pairs (cta_group::2, 256 features per pair tile, half of each
    activation sub-tile per CTA): plain and residual + GELU epilogues, partial last tiles, a
    pair tile whose second half lies past N."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    path_option(2)
    pair_option(2)
    _lib.set_option(_lib.OPT_TC_TILE, tile)
    K, N = 768, 384
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 32, seed=3 * tile + M).items()}
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=M + 1).to(cuda_device)
    r = activations(M, N, seed=M + 9).to(cuda_device)
    ref = _gpu_reference(t, K, N, x, True, t["bias"])
    y = layer(x)
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    yf = layer.forward_fused(x, residual=r, activation="gelu_tanh")
    reff = torch.nn.functional.gelu(ref, approximate="tanh") + r.double()
    errf = float((yf.double() - reff).abs().max() / reff.abs().max())
    assert errf < 1e-2, errf
    assert _lib.read_device_error(cuda_device) == 0


def test_tc_pairs_full_size(cuda_device, pair_option):
    """Config-1 qkv layer at M = 4608 on CTA pairs vs a torch fp32 GEMM of the exact weight."""
    from onecomp_runtime import _lib, quant_utils
    from onecomp_runtime.testing import gptq_layer, activations
    pair_option(2)
    K, N, M = 3072, 9216, 4608
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 32, seed=78, device="cpu").items()}
    layer = _module(t, K, N, 32, True, "fused", cuda_device)
    x = activations(M, K, seed=4).to(cuda_device)
    y = layer(x)
    w = quant_utils.dequant_gptq_to_fp(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N, torch.bfloat16)
    ref = x.float() @ w.float().t() + t["bias"].float()
    err = float((y.float() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    assert _lib.read_device_error(cuda_device) == 0


I8_PREP_SHAPES = [
    # K, N, gs, v1, act-order, scales dtype. One token without act-order: K splits of up to 20 stages
    # take the in-GEMV preparation; the others (a 43-stage split, act-order, M = 2) take the launch
    # whatever the option, which the test checks gives the same bits too
    (5120, 8192, 128, False, False, torch.float16),   # config-2 q/k/v shape: 4 splits, workspace reduction
    (17408, 5120, 128, False, False, torch.float16),  # config-2 down shape: 7 splits
    (5120, 17408, 128, False, False, torch.float16),  # config-2 gate shape: 2 splits reduced in a cluster
    (3072, 1024, 32, True, False, torch.bfloat16),    # four groups per stage
    (4160, 384, 64, True, False, torch.bfloat16),     # K not a multiple of the 128-k stage
    (5504, 19200, 128, False, False, torch.float16),  # 150 column tiles, one split of 43 stages
    (5120, 8192, 128, False, True, torch.float16),    # act-order
]


@pytest.mark.parametrize("shape", I8_PREP_SHAPES, ids=lambda s: f"K{s[0]}N{s[1]}g{s[2]}a{int(s[4])}")
@pytest.mark.parametrize("M", [1, 2])
def test_gemv_i8_prep_in_kernel_matches_launch(cuda_device, shape, M):
    """The integer decode GEMV prepares the activations of its K split inside each CTA for one token
    without act-order (OC_OPT_GEMV_PREP = 1, the default) instead of a separate preparation launch
    into the workspace (0): the same bits, NaN tokens included; both against the fp64 GEMM of the
    exact weight."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    K, N, gs, v1, act, sdt = shape
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, gs, seed=K + N, v1=v1, actorder=act,
                                                     scales_dtype=sdt).items()}
    layer = _module(t, K, N, gs, v1, "packed" if act else ("fused" if gs == 32 else "any"), cuda_device)
    x = activations(M, K, seed=K + M).to(cuda_device)
    r = activations(M, N, seed=M + 5).to(cuda_device)
    saved = (_lib.get_option(_lib.OPT_GEMV_IMPL), _lib.get_option(_lib.OPT_GEMV_PREP))
    outs = {}
    try:
        _lib.set_option(_lib.OPT_GEMV_IMPL, 4)
        for prep in (1, 0):
            _lib.set_option(_lib.OPT_GEMV_PREP, prep)
            outs[prep] = (layer(x), layer.forward_fused(x, residual=r, activation="gelu_tanh"))
        xn = x.clone()   # a NaN in the last token poisons that token's outputs only, on both paths
        xn[M - 1, K // 3] = float("nan")
        for prep in (1, 0):
            _lib.set_option(_lib.OPT_GEMV_PREP, prep)
            outs[prep] += (layer(xn),)
    finally:
        _lib.set_option(_lib.OPT_GEMV_IMPL, saved[0])
        _lib.set_option(_lib.OPT_GEMV_PREP, saved[1])
    for a, b in zip(outs[1], outs[0]):
        torch.testing.assert_close(a, b, rtol=0, atol=0, equal_nan=True)
    ref = _gpu_reference(t, K, N, x, v1, t["bias"])
    err = float((outs[1][0].double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    yn = outs[1][2]
    assert torch.isnan(yn[M - 1]).all()
    if M == 2:
        assert not torch.isnan(yn[0]).any()
        torch.testing.assert_close(yn[0], outs[1][0][0], rtol=0, atol=0)
    assert _lib.read_device_error(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [1, 6, 16])
def test_gemv_i8_activation_range(cuda_device, dtype, M):
    """The integer decode GEMV represents activations as 16-bit fixed point per 128-k stage. Per
    token (each against its own largest reference output): an outlier 1000x the others, 256 input
    columns scaled to about 1e-30 (bf16) / 1e-6 (fp16), then those columns alone (stages holding
    only tiny values), an all-zero token and a NaN token, which must give NaN in every column as
    the reference's F.linear does. Two calls in a row give identical bits."""
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import gptq_layer, activations
    K, N = 5120, 1024
    t = {k: v.to(cuda_device) for k, v in gptq_layer(K, N, 128, seed=91, v1=False, actorder=True,
                                                     scales_dtype=torch.float16, bias=False).items()}
    layer = _module(t, K, N, 128, False, "packed", cuda_device)
    x = activations(M, K, seed=17).to(cuda_device).to(dtype)
    x[0, 300] = 1000.0
    tiny = 1e-30 if dtype == torch.bfloat16 else 1e-6
    x[0, 1024:1280] *= tiny
    if M > 2:
        x[1].zero_()
        x[2, 77] = float("nan")
    saved = _lib.get_option(_lib.OPT_GEMV_IMPL)
    _lib.set_option(_lib.OPT_GEMV_IMPL, 4)
    try:
        ys = [layer(x) for _ in range(2)]
    finally:
        _lib.set_option(_lib.OPT_GEMV_IMPL, saved)
    torch.testing.assert_close(ys[0], ys[1], rtol=0, atol=0, equal_nan=True)
    y = ys[0].double()
    ref = _gpu_reference(t, K, N, x, False)
    for m in range(M):
        if M > 2 and m == 2:
            assert torch.isnan(y[m]).all()
            continue
        if M > 2 and m == 1:
            assert (y[m] == 0).all()
            continue
        err = float((y[m] - ref[m]).abs().max() / ref[m].abs().max())
        assert err < 1e-2, (m, err)
    # the tiny stage alone, in its own scale: zero every other column of token 0
    xt = torch.zeros_like(x[:1])
    xt[0, 1024:1280] = x[0, 1024:1280]
    _lib.set_option(_lib.OPT_GEMV_IMPL, 4)
    try:
        yt = layer(xt).double()
    finally:
        _lib.set_option(_lib.OPT_GEMV_IMPL, saved)
    reft = _gpu_reference(t, K, N, xt, False)
    err = float((yt - reft).abs().max() / reft.abs().max())
    assert err < 1e-2, err
    assert _lib.read_device_error(cuda_device) == 0
