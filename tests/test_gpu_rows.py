"""Row-packed GEMMs on the GPU: RTN nibble layers, DSV4 int2/int4 layers, the packed MoE.

References: the reference's own RTN outputs (golden), and fp64 GEMMs of the oracle's
bit-exact dequantized weights. Bar: max-abs-relative error < 1e-2 (north star 2e-2).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import RTN_CASES, load_golden
from gpu_util import GEMM_TOL, TDT, max_abs_rel, to_torch
from oracle import dsv4, eager
from oracle.fp import to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", RTN_CASES)
def test_rtn_linear_golden(cuda_device, case):
    from onecomp_runtime.layers import PackedRTNLinear
    d = load_golden(case)
    m = d["meta"]
    q = torch.from_numpy(d["qweight_u8"]).to(cuda_device)
    s = to_torch(d["scales"], m["scales_dtype"])
    z = to_torch(d["zeros"], m["zeros_dtype"])
    bias = torch.from_numpy(d["bias_f32"]).to(cuda_device)
    layer = PackedRTNLinear(m["in_f"], m["out_f"], q, s, z, bias)
    for od in ("bf16", "f16"):
        x = to_torch(d[f"x_{od}"], od)
        y = layer(x)
        b_od = to_f32(d["bias_f32"].astype(np.float32), "f32")
        from oracle.fp import round_to
        ref, _ = eager.linear_ref(d[f"x_{od}"], od, d[f"w_{od}"], od, round_to(b_od, od), od)
        assert max_abs_rel(y, ref) < 1e-2, (case, od)
        assert eager.max_abs_rel(y.float().cpu().numpy(), to_f32(d[f"y_{od}"], od)) < GEMM_TOL


def _dsv4_layer(out_f, in_f, wbits, gs, seed, zeros="half"):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 1 << wbits, size=(out_f, in_f))
    packed = dsv4.pack_codes(codes, wbits)
    G = (in_f + gs - 1) // gs if gs > 0 else 1
    s = rng.uniform(0.005, 0.05, size=(out_f, G)).astype(np.float16)
    if zeros == "half":
        z = np.full((out_f, G), 1.5 if wbits == 2 else 7.5, np.float16)
    else:
        z = rng.uniform(0, (1 << wbits) - 1, size=(out_f, G)).astype(np.float16)
    return {"qweight_packed": torch.from_numpy(packed), "scales": torch.from_numpy(s),
            "qzeros": torch.from_numpy(z), "wbits": wbits, "groupsize": gs, "in_features": in_f}


def _dsv4_weight(p, od):
    return dsv4.dequant_dsv4(p["qweight_packed"].numpy(), p["scales"].numpy().view(np.uint16), "f16",
                             p["qzeros"].numpy().view(np.uint16), "f16", p["wbits"], p["groupsize"],
                             p["in_features"], od)


@pytest.mark.parametrize("wbits,gs,zeros", [(2, 64, "half"), (4, 128, "half"), (4, 64, "rand"), (2, 0, "rand")])
@pytest.mark.parametrize("M", [3, 200])
def test_dsv4_linear_fused(cuda_device, wbits, gs, zeros, M):
    from onecomp_runtime.layers import Dsv4PackedLinear
    p = _dsv4_layer(192, 512, wbits, gs, seed=wbits * 10 + M, zeros=zeros)
    layer = Dsv4PackedLinear(p, buffer_device=cuda_device)
    assert layer._rows_handle() is not None
    x = torch.randn(M, 512, device=cuda_device).to(torch.bfloat16)
    y = layer(x)
    w = _dsv4_weight(p, "bf16")
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    ref, _ = eager.linear_ref(xb, "bf16", w, "bf16")
    assert max_abs_rel(y, ref) < 1e-2


@pytest.mark.parametrize("wbits,gs", [(2, 64), (4, 128), (2, 0)])
@pytest.mark.parametrize("adt", ["bf16", "f16"])
def test_dsv4_weights_bit_exact_through_gemm(cuda_device, wbits, gs, adt):
    """One-hot activation rows make y = W^T exactly (one nonzero product per output, fp32 sum,
    one exact rounding), so the weights the kernel decodes into the MMA operand are compared bit
    for bit with the oracle. Half-integer zeros: the exact mode's domain. bf16 activations take
    the split-scale path (fp16 scales), f16 activations the single-multiply path."""
    from onecomp_runtime.layers import Dsv4PackedLinear
    K, N = 512, 192
    p = _dsv4_layer(N, K, wbits, gs, seed=wbits + gs, zeros="half")
    layer = Dsv4PackedLinear(p, buffer_device=cuda_device)
    assert layer._rows_handle() is not None
    y = layer(torch.eye(K, device=cuda_device, dtype=TDT[adt]))
    got = y.t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, _dsv4_weight(p, adt))


def test_dsv4_host_buffers_match_fused(cuda_device):
    from onecomp_runtime.layers import Dsv4PackedLinear
    p = _dsv4_layer(128, 256, 2, 64, seed=5)
    x = torch.randn(7, 256, device=cuda_device).to(torch.bfloat16)
    y_host = Dsv4PackedLinear(p, buffer_device="cpu")(x)       # per-call copy + dequant + F.linear
    y_dev = Dsv4PackedLinear(p, buffer_device=cuda_device)(x)  # fused row-packed kernel
    ref = y_host.float()
    assert float((y_dev.float() - ref).abs().max() / ref.abs().max()) < 1e-2


def _moe_setup(E=8, H=256, F=128, seed=0):
    experts = [{"gate": _dsv4_layer(F, H, 2, 64, seed + 3 * e), "up": _dsv4_layer(F, H, 2, 64, seed + 3 * e + 1),
                "down": _dsv4_layer(H, F, 2, 64, seed + 3 * e + 2)} for e in range(E)]
    shared = {"gate": _dsv4_layer(F, H, 4, 128, 900), "up": _dsv4_layer(F, H, 4, 128, 901),
              "down": _dsv4_layer(H, F, 4, 128, 902)}
    return experts, shared


def _moe_reference(experts, shared, x, logits, k):
    from onecomp_runtime.moe import route_reference
    ids, w = route_reference(logits.cpu(), k)
    xf = x.double().cpu()

    def ffn(mats, xx):
        wg = torch.from_numpy(to_f32(_dsv4_weight(mats["gate"], "bf16"), "bf16")).double()
        wu = torch.from_numpy(to_f32(_dsv4_weight(mats["up"], "bf16"), "bf16")).double()
        wd = torch.from_numpy(to_f32(_dsv4_weight(mats["down"], "bf16"), "bf16")).double()
        g = xx @ wg.t()
        return (torch.nn.functional.silu(g) * (xx @ wu.t())) @ wd.t()

    out = ffn(shared, xf)
    for t in range(x.shape[0]):
        for j in range(k):
            out[t] += float(w[t, j]) * ffn(experts[int(ids[t, j])], xf[t:t + 1])[0]
    return out, ids, w


def test_moe_route_kernel_matches_convention(cuda_device):
    from onecomp_runtime.moe import PackedMoE, route_reference
    experts, shared = _moe_setup(E=8)
    moe = PackedMoE(experts, None, k=2, device=cuda_device)
    logits = torch.randn(40, 8, device=cuda_device)
    ids, w = moe.route(logits, 2)
    rid, rw = route_reference(logits, 2)
    assert torch.equal(ids.cpu(), rid.cpu())
    torch.testing.assert_close(w.cpu(), rw.cpu(), rtol=1e-5, atol=1e-6)


def test_moe_forward(cuda_device):
    from onecomp_runtime.moe import PackedMoE
    experts, shared = _moe_setup(E=8)
    moe = PackedMoE(experts, shared, k=2, device=cuda_device)
    x = torch.randn(20, 256, device=cuda_device).to(torch.bfloat16)
    logits = torch.randn(20, 8, device=cuda_device)
    y = moe(x, logits)
    ref, _, _ = _moe_reference(experts, shared, x, logits, 2)
    err = float((y.double().cpu() - ref).abs().max() / ref.abs().max())
    assert err < 2e-2, err


def test_moe_expert_parallel_single_rank(cuda_device):
    """The EP orchestration with the B200 grouped FFN as the local expert step (world size 1)."""
    from onecomp_runtime.moe import ExpertParallelMoE, PackedMoE
    experts, _ = _moe_setup(E=8)
    moe = PackedMoE(experts, None, k=2, device=cuda_device)
    ep = ExpertParallelMoE(8, 2, moe.expert_ffn, route=moe.route)
    x = torch.randn(16, 256, device=cuda_device).to(torch.bfloat16)
    logits = torch.randn(16, 8, device=cuda_device)
    y_ep = ep(x, logits)
    y = moe(x, logits)
    ref = y.float()
    assert float((y_ep.float() - ref).abs().max() / ref.abs().max()) < 1e-2


@pytest.mark.parametrize("T", [16, 0])
def test_moe_expert_parallel_combine_and_shared(cuda_device, T):
    """World size 1 with the fused combine hook and the shared expert on the side stream:
    the same kernels as PackedMoE.forward, so the same result."""
    from onecomp_runtime.moe import ExpertParallelMoE, PackedMoE
    experts, shared = _moe_setup(E=8)
    moe = PackedMoE(experts, shared, k=2, device=cuda_device)
    ep = ExpertParallelMoE(8, 2, moe.expert_ffn, route=moe.route,
                           shared=moe.shared_ffn, combine=moe.combine)
    g = torch.Generator(device=cuda_device).manual_seed(T + 3)
    x = torch.randn(T, 256, generator=g, device=cuda_device).to(torch.bfloat16)
    logits = torch.randn(T, 8, generator=g, device=cuda_device)
    for _ in range(2):  # the second call reuses the cached side stream
        y_ep = ep(x, logits)
        assert y_ep.shape == (T, 256) and y_ep.dtype == torch.bfloat16
        if T:
            ref = moe(x, logits).float()
            assert float((y_ep.float() - ref).abs().max() / ref.abs().max()) < 1e-2


def test_no_device_errors_recorded(cuda_device):
    from onecomp_runtime import _lib
    assert _lib.read_device_error(cuda_device) == 0
