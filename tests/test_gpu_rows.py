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


def _dsv4_layer(out_f, in_f, wbits, gs, seed, zeros="half", sdt=np.float16):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 1 << wbits, size=(out_f, in_f))
    packed = dsv4.pack_codes(codes, wbits)
    G = (in_f + gs - 1) // gs if gs > 0 else 1
    s = rng.uniform(0.005, 0.05, size=(out_f, G)).astype(sdt)
    if zeros == "half":
        z = np.full((out_f, G), 1.5 if wbits == 2 else 7.5, np.float16)
    elif zeros == "mixed":  # half-integer zeros except in a few rows: per-warp choice of decode path
        z = np.full((out_f, G), 1.5 if wbits == 2 else 7.5, np.float16)
        z[::37] = rng.uniform(0, (1 << wbits) - 1, size=z[::37].shape).astype(np.float16)
    else:
        z = rng.uniform(0, (1 << wbits) - 1, size=(out_f, G)).astype(np.float16)
    return {"qweight_packed": torch.from_numpy(packed), "scales": torch.from_numpy(s),
            "qzeros": torch.from_numpy(z), "wbits": wbits, "groupsize": gs, "in_features": in_f}


def _bits_and_name(t: torch.Tensor):
    if t.dtype == torch.float32:
        return t.numpy(), "f32"
    return t.numpy().view(np.uint16), "f16"


def _dsv4_weight(p, od):
    s, sn = _bits_and_name(p["scales"])
    z, zn = _bits_and_name(p["qzeros"])
    return dsv4.dequant_dsv4(p["qweight_packed"].numpy(), s, sn, z, zn, p["wbits"], p["groupsize"],
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


@pytest.mark.parametrize("wbits,gs,zeros,sdt", [
    (2, 64, "half", np.float16), (4, 128, "half", np.float16), (2, 0, "half", np.float16),
    (2, 64, "rand", np.float16), (4, 64, "rand", np.float16), (2, 0, "rand", np.float16),
    (4, 128, "mixed", np.float16), (4, 64, "half", np.float32), (2, 128, "rand", np.float32)],
    ids=lambda v: v.__name__ if isinstance(v, type) else str(v))
@pytest.mark.parametrize("adt", ["bf16", "f16"])
def test_dsv4_weights_bit_exact_through_gemm(cuda_device, wbits, gs, zeros, sdt, adt):
    """One-hot activation rows make y = W^T exactly (one nonzero product per output, fp32 sum,
    one exact rounding), so the weights the kernel decodes into the MMA operand are compared bit
    for bit with the oracle, for any zero point and scale dtype: int2 layers decode through the
    fp32 value table; int4 layers through the pair arithmetic where it is exact (half-integer
    zeros, 16-bit scales) and the fp32 formula elsewhere, chosen per warp."""
    from onecomp_runtime.layers import Dsv4PackedLinear
    K, N = 512, 192
    p = _dsv4_layer(N, K, wbits, gs, seed=wbits + gs, zeros=zeros, sdt=sdt)
    layer = Dsv4PackedLinear(p, buffer_device=cuda_device)
    assert layer._rows_handle() is not None
    y = layer(torch.eye(K, device=cuda_device, dtype=TDT[adt]))
    got = y.t().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, _dsv4_weight(p, adt))


@pytest.mark.parametrize("wbits,gs", [(2, 64), (4, 128)])
def test_dsv4_host_buffers_match_fused(cuda_device, wbits, gs):
    """Host-resident (offloaded) layers copy their packed bytes into the shared staging slot and
    run the same fused kernel: identical output to device-resident buffers, also when two layers
    of one shape take turns on the slot; and within tolerance of the oracle."""
    from onecomp_runtime.layers import Dsv4PackedLinear
    p = _dsv4_layer(128, 256, wbits, gs, seed=5)
    p2 = _dsv4_layer(128, 256, wbits, gs, seed=6)
    x = torch.randn(7, 256, device=cuda_device).to(torch.bfloat16)
    host, host2 = Dsv4PackedLinear(p, buffer_device="cpu"), Dsv4PackedLinear(p2, buffer_device="cpu")
    y_host, y_host2, y_host_again = host(x), host2(x), host(x)
    y_dev = Dsv4PackedLinear(p, buffer_device=cuda_device)(x)
    y_dev2 = Dsv4PackedLinear(p2, buffer_device=cuda_device)(x)
    assert torch.equal(y_host, y_dev) and torch.equal(y_host_again, y_dev) and torch.equal(y_host2, y_dev2)
    xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
    ref, _ = eager.linear_ref(xb, "bf16", _dsv4_weight(p, "bf16"), "bf16")
    assert max_abs_rel(y_host, ref) < 1e-2


def test_rtn_padded_layouts(cuda_device):
    """RTN layers whose packed row stride is not a multiple of 16 bytes, or whose in_features is
    not a multiple of 8 (one group per row), run the fused kernel on a zero-padded copy."""
    from onecomp_runtime.layers import PackedRTNLinear
    from oracle import rtn
    rng = np.random.default_rng(9)
    for K, G in ((208, 2), (100, 1), (75, 1)):
        N = 96
        codes = rng.integers(0, 16, size=(N, K))
        q = np.zeros((N, (K + 1) // 2), np.uint8)
        q[:, :] = (codes[:, 0::2] | (np.pad(codes[:, 1::2], ((0, 0), (0, K % 2))) << 4)).astype(np.uint8)
        s = rng.uniform(0.01, 0.1, size=(N, G)).astype(np.float16)
        z = rng.integers(0, 16, size=(N, G)).astype(np.float16)
        layer = PackedRTNLinear(K, N, torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device),
                                torch.from_numpy(z).to(cuda_device))
        assert layer._rows_handle() is not None
        x = torch.randn(33, K, device=cuda_device).to(torch.bfloat16)
        y = layer(x)
        w = rtn.dequant_rtn(q, s.view(np.uint16), "f16", z.view(np.uint16), "f16", K, N, "bf16")
        xb = x.cpu().view(torch.int16).numpy().view(np.uint16)
        ref, _ = eager.linear_ref(xb, "bf16", w, "bf16")
        assert max_abs_rel(y, ref) < 1e-2, (K, G)


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


@pytest.mark.parametrize("fuse", [True, "shared", False])
def test_moe_forward(cuda_device, fuse):
    from onecomp_runtime.moe import PackedMoE
    experts, shared = _moe_setup(E=8)
    moe = PackedMoE(experts, shared, k=2, device=cuda_device, fuse_gate_up=fuse)
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


@pytest.mark.parametrize("grouped", [True, False])
def test_swiglu_launch_matches_separate_gemms(cuda_device, grouped):
    """The fused gate|up launch (oc_b200_rows_gemm_swiglu) gives the same bits as the gate and up
    GEMMs run separately followed by the silu-mul kernel: grouped over 8 int2 gs64 experts with
    ragged segments (an empty expert and one of 150 rows: two m-tiles), and dense on the int4 gs128
    shared expert."""
    from onecomp_runtime import _lib
    from onecomp_runtime.layers._rows_base import MODE_EXACT, RowsHandle, group_major
    from onecomp_runtime.moe import PackedMoE
    experts, shared = _moe_setup(E=8, H=256, F=384)
    moe = PackedMoE(experts, shared, k=2, device=cuda_device, fuse_gate_up=True)
    hs = moe._h if grouped else moe._shared
    assert "gate_up" in hs
    mats = experts if grouped else [shared]
    counts = [20, 0, 150, 7, 33, 64, 1, 90] if grouped else [77]
    P = sum(counts)
    offsets = torch.tensor([0] + list(np.cumsum(counts)), dtype=torch.int32, device=cuda_device)
    x = torch.randn(P, 256, generator=torch.Generator(device=cuda_device).manual_seed(5),
                    device=cuda_device).to(torch.bfloat16)
    m0 = mats[0]["gate"]
    wbits, gs, K, F = int(m0["wbits"]), int(m0["groupsize"]), int(m0["in_features"]), 384

    def handle(name):
        dev = cuda_device
        return RowsHandle([m[name]["qweight_packed"].to(dev).contiguous() for m in mats],
                          [group_major(m[name]["scales"].to(dev), F, K, gs) for m in mats],
                          [group_major(m[name]["qzeros"].to(dev), F, K, gs) for m in mats],
                          wbits, gs, K, F, MODE_EXACT, 1, F)

    off = offsets if grouped else None
    g = torch.empty((P, 2 * F), dtype=torch.bfloat16, device=cuda_device)
    handle("gate").gemm(x, g[:, :F], off)
    handle("up").gemm(x, g[:, F:], off)
    ref = torch.empty((P, F), dtype=torch.bfloat16, device=cuda_device)
    st = _lib.stream_of(cuda_device)
    _lib.call("oc_b200_silu_mul", g.data_ptr(), g[:, F:].data_ptr(), g.stride(0), P, F, ref.data_ptr(),
              ref.stride(0), _lib.DT[torch.bfloat16], st)
    h = torch.full((P, F), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    _lib.call("oc_b200_rows_gemm_swiglu", hs["gate_up"].h, x.data_ptr(), _lib.DT[torch.bfloat16], P, x.stride(0),
              None if off is None else off.data_ptr(), h.data_ptr(), h.stride(0), st)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(h.view(torch.int16), ref.view(torch.int16))
    assert _lib.read_device_error(cuda_device) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_mul_and_combine_vector_paths_match_scalar(cuda_device, dtype):
    """silu-mul and the weighted combine take 8 columns per thread when rows are 16-byte aligned
    and a scalar path otherwise (odd row pitch): the same bits either way, and silu-mul against
    torch's silu within a bf16/fp16 ulp."""
    from onecomp_runtime import _lib
    st = _lib.stream_of(cuda_device)
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    P, F, T, k, H = 97, 264, 40, 3, 264
    dt = _lib.DT[dtype]

    def silu_mul(pitch):
        gu = torch.randn(P, pitch, generator=gen, device=cuda_device).mul(4).to(dtype)
        g, u = gu[:, :F], gu[:, F:2 * F]
        outs = []
        for ld_out in (F, F + 1):   # 16-byte rows (vector path) and an odd pitch (scalar path)
            h = torch.zeros(P, ld_out, dtype=dtype, device=cuda_device)
            _lib.call("oc_b200_silu_mul", g.data_ptr(), u.data_ptr(), gu.stride(0), P, F, h.data_ptr(), ld_out,
                      dt, st)
            outs.append(h[:, :F])
        return g, u, outs

    g, u, (hv, hs) = silu_mul(2 * F)
    assert torch.equal(hv.view(torch.int16), hs.view(torch.int16))
    ref = (torch.nn.functional.silu(g.float()) * u.float())
    assert float(((hv.float() - ref).abs() / ref.abs().clamp_min(1e-3)).max()) < 2.0 ** -6
    y = torch.randn(T * k, H, generator=gen, device=cuda_device).to(dtype)
    slot = torch.randperm(T * k, generator=gen, device=cuda_device).to(torch.int32)
    w = torch.rand(T, k, generator=gen, device=cuda_device)
    sh = torch.randn(T, H, generator=gen, device=cuda_device).to(dtype)
    y_odd = torch.zeros(T * k, H + 1, dtype=dtype, device=cuda_device)
    y_odd[:, :H] = y
    outs = []
    for yy, ldy in ((y, H), (y_odd, H + 1)):
        o = torch.zeros(T, H, dtype=dtype, device=cuda_device)
        _lib.call("oc_b200_moe_combine", yy.data_ptr(), ldy, slot.data_ptr(), w.data_ptr(), T, k, H, sh.data_ptr(),
                  H, o.data_ptr(), H, dt, st)
        outs.append(o)
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    assert _lib.read_device_error(cuda_device) == 0


def test_no_device_errors_recorded(cuda_device):
    from onecomp_runtime import _lib
    assert _lib.read_device_error(cuda_device) == 0
