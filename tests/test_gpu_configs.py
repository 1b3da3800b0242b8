"""Parity at the benchmark configurations' own shapes (3 and 4).

* config 2: the five decode layers (gptq_v2, act-order gs128, fp16 scales) at M = 1, 4, 16;
* config 4: the four video-DiT layer shapes at M = 32768 tokens;
* config 3: the packed MoE layer at full size (256 int2 experts, top-8, H = 4096, F = 2048,
  T = 2048, int4 gs128 shared expert with fractional zeros), checked on a seeded subset of
  64 tokens against fp64 SwiGLU experts.

References are fp64 / fp32 GEMMs of the exact dequantized weights. The GPU dequant kernels that
produce those weights are pinned here against the numpy oracle on a slice of each layer (the
dequant is elementwise, so a slice checks the same code paths in seconds).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import NAME, oracle_weight, to_bits
from oracle import dsv4

pytestmark = pytest.mark.gpu


def _rel(y: torch.Tensor, ref: torch.Tensor) -> float:
    return float((y.double() - ref.double()).abs().max() / ref.double().abs().max())


def _pin_gptq(t: dict, K: int, N: int, w: torch.Tensor, v1: bool, ns: int = 512):
    """The first `ns` output features of a GPU-dequantized weight equal the oracle's, bit for bit."""
    per = 32 // 4
    ts = {"qweight": t["qweight"][:, :ns].cpu(), "scales": t["scales"][:, :ns].cpu(),
          "qzeros": t["qzeros"][:, :ns // per].cpu(), "g_idx": t["g_idx"].cpu()}
    ref = oracle_weight(ts, K, ns, NAME[w.dtype], v1=v1)
    np.testing.assert_array_equal(to_bits(w[:ns]), ref)


# ----------------------------------------------------------------------------------- config 2
@pytest.mark.parametrize("M", [1, 4, 16])
def test_cfg2_layers_fp16_scales(cuda_device, M):
    """Config 2 as stated: gptq_v2 (zeros unshifted), gs128, act-order, fp16 scales U[0.001, 0.01]."""
    from onecomp_runtime import quant_utils
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import CFG2_LAYERS, activations, gptq_layer
    for i, (name, K, N) in enumerate(CFG2_LAYERS):
        t = gptq_layer(K, N, 128, seed=2000 + i, v1=False, actorder=True, scales_range=(0.001, 0.01),
                       scales_dtype=torch.float16, bias=False, device=cuda_device)
        layer = PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], None, 128, 4, False)
        x = activations(M, K, seed=M + 10 * i, device=cuda_device)
        y = layer(x)
        w = quant_utils.dequant_gptq_to_fp(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N,
                                           torch.bfloat16, v1=False)
        if M == 1:
            _pin_gptq(t, K, N, w, v1=False, ns=256)
        ref = x.double() @ w.double().t()
        err = _rel(y, ref)
        assert err < 1e-2, (name, M, err)


# ----------------------------------------------------------------------------------- config 4
def test_cfg4_layers_full_m(cuda_device):
    """Config 4's four layer shapes (GPTQ v1 gs32) at M = 32768 through the tcgen05 GEMM, against a
    torch fp32 GEMM of the exact weight (TF32 off)."""
    from onecomp_runtime import quant_utils
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.testing import CFG4, CFG4_LAYERS, activations, gptq_layer
    assert not torch.backends.cuda.matmul.allow_tf32
    M = CFG4["M"]
    for i, (name, K, N) in enumerate(CFG4_LAYERS):
        t = gptq_layer(K, N, 32, seed=4000 + i, device=cuda_device)
        layer = FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t["bias"], 32)
        x = activations(M, K, seed=40 + i, device=cuda_device)
        y = layer(x)
        w = quant_utils.dequant_gptq_to_fp(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N,
                                           torch.bfloat16)
        if i == 0:
            _pin_gptq(t, K, N, w, v1=True)
        ref = torch.addmm(t["bias"].float(), x.float(), w.float().t())
        err = _rel(y, ref)
        del ref, x, y, w
        assert err < 1e-2, (name, err)


# ----------------------------------------------------------------------------------- config 3
def _pin_dsv4(p: dict, w: torch.Tensor, rows: int = 256):
    """The first `rows` output rows of a GPU-dequantized DSV4 weight equal the oracle's."""
    ref = dsv4.dequant_dsv4(p["qweight_packed"][:rows].cpu().numpy(),
                            p["scales"][:rows].cpu().numpy().view(np.uint16), "f16",
                            p["qzeros"][:rows].cpu().numpy().view(np.uint16), "f16", p["wbits"],
                            p["groupsize"], p["in_features"], "bf16")
    np.testing.assert_array_equal(to_bits(w[:rows]), ref)


def test_cfg3_moe_full_size(cuda_device):
    """Config 3 at full size through PackedMoE: routing kernel vs the stated convention on all 2048
    tokens; outputs of 64 seeded tokens vs fp64 experts (SwiGLU, top-8 weighted sum, shared expert)
    built from the exact dequantized weights."""
    from onecomp_runtime import _lib
    from onecomp_runtime.layers.dsv4_packed_linear import dequant_dsv4_packed
    from onecomp_runtime.moe import PackedMoE, route_reference
    from onecomp_runtime.testing import CFG3, dsv4_packed
    E, k, H, F, T = CFG3["E"], CFG3["k"], CFG3["H"], CFG3["F"], CFG3["T"]
    wb, gs = CFG3["expert_wbits"], CFG3["expert_gs"]
    dev = cuda_device
    experts = [{"gate": dsv4_packed(F, H, wb, gs, seed=3 * e, device=dev),
                "up": dsv4_packed(F, H, wb, gs, seed=3 * e + 1, device=dev),
                "down": dsv4_packed(H, F, wb, gs, seed=3 * e + 2, device=dev)} for e in range(E)]
    sw, sgs = CFG3["shared_wbits"], CFG3["shared_gs"]
    shared = {n: dsv4_packed(*shape, sw, sgs, seed=9000 + j, zero=None, scales_range=(0.002, 0.02), device=dev)
              for j, (n, shape) in enumerate((("gate", (F, H)), ("up", (F, H)), ("down", (H, F))))}
    g = torch.Generator(device=dev).manual_seed(77)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g, device=dev)
    moe = PackedMoE(experts, shared, k=k, device=dev)
    y = moe(x, logits)

    ids, w = moe.route(logits, k)
    rid, rw = route_reference(logits, k)
    assert torch.equal(ids.long().cpu(), rid.long().cpu())
    torch.testing.assert_close(w.cpu(), rw.cpu(), rtol=1e-5, atol=1e-6)

    def weight(p):
        return dequant_dsv4_packed(p, dtype=torch.bfloat16, device=dev)

    # the dequant feeding the reference, pinned to the oracle (an expert's three matrices and the
    # shared expert's gate, whose zeros are fractional)
    for p in (experts[5]["gate"], experts[5]["up"], experts[5]["down"], shared["gate"]):
        _pin_dsv4(p, weight(p))

    def ffn(mats, xx):
        wg, wu, wd = (weight(mats[n]).double() for n in ("gate", "up", "down"))
        return (torch.nn.functional.silu(xx @ wg.t()) * (xx @ wu.t())) @ wd.t()

    sel = torch.randperm(T, generator=torch.Generator().manual_seed(3))[:64].to(dev)
    xs = x[sel].double()
    ref = ffn(shared, xs)
    sid, swt = rid.to(dev)[sel], rw.to(dev)[sel].double()
    for e in torch.unique(sid).tolist():
        rows, slots = (sid == e).nonzero(as_tuple=True)
        ref[rows] += swt[rows, slots].unsqueeze(1) * ffn(experts[e], xs[rows])
    err = _rel(y[sel], ref)
    assert err < 2e-2, err
    assert _lib.read_device_error(dev) == 0


# ------------------------------------------------------------------ exact GEMM operand, edge scales
def test_gptq_operand_exact_f16_act_tiny_bf16_scales(cuda_device):
    """fp16 activations with bf16 scales below fp16's normal range (the scale split is inexact
    there, so the kernel takes the fp32 formula): one-hot activation rows make the tcgen05 GEMM's
    output W^T exactly, compared bit for bit with the oracle's dequant."""
    from onecomp_runtime.layers import FusedInt4LinearAnyGroup
    from onecomp_runtime.testing import gptq_layer
    K, N = 512, 256
    t = gptq_layer(K, N, 64, seed=21, scales_range=(1e-8, 2e-5), scales_dtype=torch.bfloat16, bias=False,
                   device=cuda_device)
    layer = FusedInt4LinearAnyGroup(K, N, t["qweight"], t["scales"], t["qzeros"], None, 64)
    y = layer(torch.eye(K, device=cuda_device, dtype=torch.float16))
    got = to_bits(y.t().contiguous())
    ref = oracle_weight({n: v.cpu() for n, v in t.items()}, K, N, "f16")
    # Products that underflow keep the sign of q - z (-0 in the weight), but the one-hot sum adds
    # +0 products of the other rows and returns +0: the sign of a zero is not observable here.
    zero = lambda b: np.where((b & 0x7FFF) == 0, 0, b)  # noqa: E731
    assert ((ref & 0x7FFF) == 0).sum() > 0      # the case does reach fp16 underflow
    np.testing.assert_array_equal(zero(got), zero(ref))
