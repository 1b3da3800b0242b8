"""Bit-exact dequant parity on the GPU against the reference's golden vectors and the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import DSV4_CASES, GPTQ_CASES, RTN_CASES, load_golden
from gpu_util import TDT, to_bits, to_torch
from oracle import gptq

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", GPTQ_CASES)
def test_gptq_dequant_golden(cuda_device, case):
    from onecomp_runtime import quant_utils
    d = load_golden(case)
    m = d["meta"]
    qw = torch.from_numpy(d["qweight"]).to(cuda_device)
    qz = torch.from_numpy(d["qzeros"]).to(cuda_device)
    s = to_torch(d["scales"], m["scales_dtype"])
    gi = torch.from_numpy(d["g_idx"]).to(cuda_device)
    for od in m["out_dtypes"]:
        w = quant_utils.dequant_gptq_to_fp(qw, s, qz, gi, m["K"], m["N"], TDT[od], v1=m["v1"], wbits=m["wbits"])
        np.testing.assert_array_equal(to_bits(w), d[f"w_{od}"])
    # fp32 output: the exact product
    w32 = quant_utils.dequant_gptq_to_fp(qw, s, qz, gi, m["K"], m["N"], torch.float32, v1=m["v1"], wbits=m["wbits"])
    ref32 = gptq.dequant_gptq(d["qweight"], d["scales"], m["scales_dtype"], d["qzeros"], d["g_idx"], m["K"], m["N"],
                              "f32", v1=m["v1"], wbits=m["wbits"])
    np.testing.assert_array_equal(w32.cpu().numpy(), ref32)


@pytest.mark.parametrize("case", RTN_CASES)
def test_rtn_dequant_golden(cuda_device, case):
    from onecomp_runtime import quant_utils
    d = load_golden(case)
    m = d["meta"]
    q = torch.from_numpy(d["qweight_u8"]).to(cuda_device)
    s = to_torch(d["scales"], m["scales_dtype"])
    z = to_torch(d["zeros"], m["zeros_dtype"])
    for od in ("bf16", "f16"):
        w = quant_utils.dequant_extra_u8_to_weight(q, s, z, m["in_f"], m["out_f"], TDT[od])
        np.testing.assert_array_equal(to_bits(w), d[f"w_{od}"])


@pytest.mark.parametrize("case", DSV4_CASES)
def test_dsv4_dequant_golden(cuda_device, case):
    from onecomp_runtime.layers import dequant_dsv4_packed
    d = load_golden(case)
    m = d["meta"]
    p = {"qweight_packed": torch.from_numpy(d["qweight_packed"]), "scales": to_torch(d["scales"], "f16", "cpu"),
         "qzeros": to_torch(d["qzeros"], "f16", "cpu"), "wbits": m["wbits"], "groupsize": m["gs"],
         "in_features": m["in_f"]}
    for od in ("bf16", "f16"):
        w = dequant_dsv4_packed(p, dtype=TDT[od], device=cuda_device)
        np.testing.assert_array_equal(to_bits(w), d[f"w_{od}"])


def test_unpack_pack_roundtrip(cuda_device):
    from onecomp_runtime import quant_utils
    from onecomp_runtime.layers.fused_int4_linear import _pack_int4_weights
    d = load_golden("gptq_v1_gs32")
    m = d["meta"]
    qw = torch.from_numpy(d["qweight"]).to(cuda_device)
    w_int = quant_utils.unpack_int_weights(qw, 4, (m["N"], m["K"]))
    np.testing.assert_array_equal(w_int.cpu().numpy(), gptq.unpack_int_weights(d["qweight"], 4, (m["N"], m["K"])))
    assert torch.equal(_pack_int4_weights(w_int), qw)
    qz = torch.from_numpy(d["qzeros"]).to(cuda_device)
    z = quant_utils.unpack_zeros(qz, 4, m["N"])
    np.testing.assert_array_equal(z.cpu().numpy(), gptq.unpack_zeros(d["qzeros"], 4, m["N"]))
    with pytest.raises(ValueError):
        quant_utils.unpack_int_weights(qw, 3, (m["N"], m["K"]))


@pytest.mark.parametrize("cfg", ["cfg0", "cfg2_gate"])
def test_dequant_full_size_bit_exact(cuda_device, cfg):
    """Config-sized layers: the GPU dequant equals the oracle bit for bit."""
    from onecomp_runtime import quant_utils
    from onecomp_runtime.testing import gptq_layer
    from gpu_util import oracle_weight
    if cfg == "cfg0":
        K, N, gs, v1, act, sr = 3072, 3072, 32, True, False, (0.002, 0.02)
    else:
        K, N, gs, v1, act, sr = 5120, 17408, 128, False, True, (0.001, 0.01)
    t = gptq_layer(K, N, gs, seed=11, v1=v1, actorder=act, scales_range=sr)
    tc = {k: v.to(cuda_device) for k, v in t.items()}
    w = quant_utils.dequant_gptq_to_fp(tc["qweight"], tc["scales"], tc["qzeros"], tc["g_idx"], K, N,
                                       torch.bfloat16, v1=v1)
    # the oracle checks the first 2048 output features of the full-size dequant
    # (dequant is elementwise; this keeps the CPU side to seconds)
    ns = min(N, 2048)
    ts = {"qweight": t["qweight"][:, :ns], "scales": t["scales"][:, :ns], "qzeros": t["qzeros"][:, :ns // 8],
          "g_idx": t["g_idx"]}
    ref = oracle_weight(ts, K, ns, "bf16", v1=v1)
    np.testing.assert_array_equal(to_bits(w[:ns]), ref)


def test_no_device_errors_recorded(cuda_device):
    from onecomp_runtime import _lib
    assert _lib.read_device_error(cuda_device) == 0
