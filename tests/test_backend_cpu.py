"""Host-side logic of the drop-in boundary: backend resolution, build ladder, K re-layout plans."""
from __future__ import annotations

import pytest
import torch

from onecomp_runtime import backend
from onecomp_runtime.layers._gptq_base import plan_k_layout
from onecomp_runtime.testing import entry


def test_resolve_backend():
    assert backend.resolve_backend("auto") == "b200"
    assert backend.resolve_backend(None) == "b200"
    for b in ("b200", "B200", "fused", "packed", "eager"):
        assert backend.resolve_backend(b) == b.lower()
    assert backend.resolve_backend("fused", use_fused=False) == "eager"
    with pytest.raises(ValueError, match="unknown backend"):
        backend.resolve_backend("triton")
    for b in ("gemlite", "a8w4", "nvfp4_ffn"):
        with pytest.raises(RuntimeError):
            backend.resolve_backend(b)


def test_resolve_dtype():
    assert backend.resolve_dtype("bf16") is torch.bfloat16
    assert backend.resolve_dtype("float16") is torch.float16
    assert backend.resolve_dtype(torch.float32) is torch.float32
    with pytest.raises(ValueError):
        backend.resolve_dtype("int8")


@pytest.mark.parametrize("e,fused,anyg,padded", [
    (entry("a", 3072, 3072, 32), True, True, False),
    (entry("a", 3072, 3072, 32, actorder=True), False, False, False),
    (entry("a", 5120, 8192, 128), False, True, False),
    (entry("a", 520, 64, 26), False, True, True),
    (entry("a", 3072, 3072, 32, wbits=8), False, False, False),
    (entry("a", 3072, 3076, 32), False, False, False),
    (entry("a", 3080, 3072, 32), False, True, False),
])
def test_can_use_ladder(e, fused, anyg, padded):
    assert backend.can_use_fused(e) is fused
    assert backend.can_use_fused_any_group(e) is anyg
    assert backend.can_use_fused_padded_groups(e) is padded


def test_plan_natural():
    kp, kperm, wg, gs = plan_k_layout(3072, 32, 96, None)
    assert (kp, kperm, wg, gs) == (3072, None, None, 32)


def test_plan_actorder_sorts_groups():
    K, gs = 512, 128
    g = torch.Generator().manual_seed(0)
    g_idx = (torch.arange(K) // gs)[torch.randperm(K, generator=g)]
    kp, kperm, wg, gse = plan_k_layout(K, gs, K // gs, g_idx)
    assert kp == K and wg is None and gse == gs
    assert sorted(kperm.tolist()) == list(range(K))
    # every kernel row k' belongs to group k' // gs
    assert torch.equal(g_idx[kperm.long()], torch.arange(K) // gs)


def test_plan_odd_groupsize_pads_to_8():
    K, gs = 520, 26
    kp, kperm, wg, gse = plan_k_layout(K, gs, K // gs, None)
    assert kp == 20 * 32 and gse == 32 and wg is None
    real = kperm[kperm >= 0]
    assert real.tolist() == list(range(K))
    assert int((kperm < 0).sum()) == 20 * 6


def test_plan_irregular_uses_word_groups():
    g_idx = torch.tensor([0] * 5 + [1] * 12 + [2] * 7)
    kp, kperm, wg, gse = plan_k_layout(24, 8, 3, g_idx)
    assert gse == 0 and wg is not None
    assert kp == 8 + 16 + 8
    assert wg.tolist() == [0, 1, 1, 2]


def test_plan_rejects_bad_g_idx():
    with pytest.raises(ValueError):
        plan_k_layout(16, 8, 2, torch.tensor([0] * 8 + [2] * 8))
    with pytest.raises(ValueError):
        plan_k_layout(16, 8, 2, torch.zeros(15, dtype=torch.long))


def test_no_cpu_fallback():
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(64, 64, 32, seed=1)
    layer = FusedInt4Linear(64, 64, t["qweight"], t["scales"], t["qzeros"], t["bias"])
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        layer(torch.zeros(2, 64, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        backend.build_quant_layer(entry("x", 64, 64, 32), t, "b200", torch.bfloat16, torch.device("cpu"))


def test_fused_requires_groupsize_32():
    from onecomp_runtime.layers import FusedInt4Linear, FusedInt4LinearPaddedGroups
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(128, 64, 64, seed=2)
    with pytest.raises(AssertionError):
        FusedInt4Linear(128, 64, t["qweight"], t["scales"], t["qzeros"], groupsize=64)
    with pytest.raises(ValueError):
        FusedInt4LinearPaddedGroups(128, 64, t["qweight"], t["scales"], t["qzeros"], groupsize=32)


def test_apply_keeps_packed_int32():
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(64, 64, 32, seed=3)
    layer = FusedInt4Linear(64, 64, t["qweight"], t["scales"], t["qzeros"], t["bias"]).to(torch.float32)
    assert layer.qweight.dtype == torch.int32 and layer.qzeros.dtype == torch.int32
    assert layer.scales.dtype == torch.float16
    layer = layer.to(torch.bfloat16)
    assert layer.scales.dtype == torch.bfloat16 and layer.qweight.dtype == torch.int32


def test_synthetic_packers_match_oracle():
    import numpy as np
    from oracle import gptq
    from onecomp_runtime.testing import pack_along_k, pack_along_n
    g = torch.Generator().manual_seed(4)
    codes = torch.randint(0, 16, (24, 64), generator=g)
    np.testing.assert_array_equal(pack_along_k(codes).numpy(), gptq.pack_int_weights(codes.numpy(), 4))
    z = torch.randint(0, 16, (3, 32), generator=g)
    np.testing.assert_array_equal(pack_along_n(z).numpy(), gptq.pack_zeros(z.numpy(), 4))


@pytest.mark.parametrize("K,N,gs,actorder,ok", [
    (512, 256, 128, False, True),    # Qwen3.6-style 8-bit layer: uniform groups of 128
    (1000, 256, 32, False, True),    # K not a multiple of the 64-k stage
    (512, 256, 48, False, False),    # groups of 48: neither 32 nor a multiple of 64
    (512, 64, 128, False, False),    # N below one 128-column tile
    (512, 256, 128, True, True),     # act-order, every group 128 rows: kernels after a K re-layout
    (512, 256, 128, "uneven", False),  # act-order with unequal groups: dequant + F.linear
])
def test_packed_gptq_8bit_kernel_eligibility(K, N, gs, actorder, ok):
    """Which 8-bit PackedGPTQLinear layers take the 8-bit kernels (decided at construction, no GPU);
    act-order layers get their group-sorted row order."""
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(K, N, gs, seed=1, actorder=bool(actorder), wbits=8, bias=False)
    g_idx = t["g_idx"].clone()
    if actorder == "uneven":
        g_idx[int((g_idx == 0).nonzero()[0])] = 1
    layer = PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], g_idx, None, gs, 8, True)
    assert layer._kernel8_ok is ok
    if actorder is True:
        kp = layer._kperm8.long()
        assert torch.equal(g_idx[kp], torch.arange(K) // gs)   # rows sorted by group
        assert torch.equal(torch.sort(kp).values, torch.arange(K))
    assert layer.qweight.shape == (K // 4, N) and layer.qzeros.shape == (t["scales"].shape[0], N // 4)
