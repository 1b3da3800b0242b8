"""Pin the CPU oracle against golden vectors produced by the reference itself."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import EMB_CASES, CONV_CASES, DSV4_CASES, GPTQ_CASES, RTN_CASES, load_golden
from oracle import dsv4, eager, gptq, rtn


@pytest.mark.parametrize("case", GPTQ_CASES)
def test_gptq_dequant_bit_exact(case):
    d = load_golden(case)
    m = d["meta"]
    for od in m["out_dtypes"]:
        w = gptq.dequant_gptq(d["qweight"], d["scales"], m["scales_dtype"], d["qzeros"],
                              d["g_idx"], m["K"], m["N"], od, v1=m["v1"], wbits=m["wbits"])
        np.testing.assert_array_equal(w, d[f"w_{od}"])


@pytest.mark.parametrize("case", [c for c in GPTQ_CASES if load_golden(c)["meta"]["M"]])
def test_gptq_eager_linear_within_tolerance(case):
    d = load_golden(case)
    m = d["meta"]
    for od in m["out_dtypes"]:
        w = gptq.dequant_gptq(d["qweight"], d["scales"], m["scales_dtype"], d["qzeros"],
                              d["g_idx"], m["K"], m["N"], od, v1=m["v1"], wbits=m["wbits"])
        bias = d.get("bias_f16")
        # the eager nn.Linear keeps its bias in the compute dtype (backend.py:263)
        if bias is not None:
            from oracle.fp import round_to, to_f32
            bias = round_to(to_f32(bias, "f16"), od)
        y32, _ = eager.linear_ref(d[f"x_{od}"], od, w, od, bias, od if bias is not None else None)
        from oracle.fp import to_f32
        ref = to_f32(d[f"y_{od}"], od)
        assert eager.max_abs_rel(ref, y32) < 1e-2


def test_pack_roundtrip():
    rng = np.random.default_rng(0)
    for wbits in (4, 8):
        codes = rng.integers(0, 1 << wbits, size=(24, 64))
        q = gptq.pack_int_weights(codes, wbits)
        assert q.dtype == np.int32 and q.shape == (64 // (32 // wbits), 24)
        np.testing.assert_array_equal(gptq.unpack_int_weights(q, wbits, (24, 64)), codes)
        z = rng.integers(0, 1 << wbits, size=(3, 16))
        np.testing.assert_array_equal(gptq.unpack_zeros(gptq.pack_zeros(z, wbits), wbits, 16), z)


def test_pack_matches_golden_layout():
    d = load_golden("gptq_v1_gs32")
    m = d["meta"]
    codes = gptq.unpack_int_weights(d["qweight"], 4, (m["N"], m["K"]))
    np.testing.assert_array_equal(gptq.pack_int_weights(codes, 4), d["qweight"])


@pytest.mark.parametrize("case", RTN_CASES)
def test_rtn_dequant_bit_exact(case):
    d = load_golden(case)
    m = d["meta"]
    for od in ("bf16", "f16"):
        w = rtn.dequant_rtn(d["qweight_u8"], d["scales"], m["scales_dtype"], d["zeros"],
                            m["zeros_dtype"], m["in_f"], m["out_f"], od)
        np.testing.assert_array_equal(w, d[f"w_{od}"])


@pytest.mark.parametrize("case", DSV4_CASES)
def test_dsv4_dequant_bit_exact(case):
    d = load_golden(case)
    m = d["meta"]
    for od in ("bf16", "f16"):
        w = dsv4.dequant_dsv4(d["qweight_packed"], d["scales"], "f16", d["qzeros"], "f16",
                              m["wbits"], m["gs"], m["in_f"], od)
        np.testing.assert_array_equal(w, d[f"w_{od}"])


def test_dsv4_pack_roundtrip():
    rng = np.random.default_rng(1)
    for wbits in (2, 4):
        codes = rng.integers(0, 1 << wbits, size=(8, 37))
        p = dsv4.pack_codes(codes, wbits)
        np.testing.assert_array_equal(dsv4.unpack_codes(p, wbits, 37), codes)


def test_rtn_pack_roundtrip():
    rng = np.random.default_rng(2)
    codes = rng.integers(0, 16, size=(8, 33))
    np.testing.assert_array_equal(rtn.unpack_u8_nibbles(rtn.pack_u8_nibbles(codes), 33), codes)


def test_bf16_rounding_ties_and_nan():
    from oracle.fp import f32_to_bf16_bits, bf16_bits_to_f32
    x = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -2.5, np.inf, 0.0, -0.0], dtype=np.float32)
    b = f32_to_bf16_bits(x)
    np.testing.assert_array_equal(bf16_bits_to_f32(b)[:4], np.array([1.0, 1.0, 1.0 + 2**-6, -2.5], np.float32))
    assert np.isinf(bf16_bits_to_f32(b)[4])
    assert np.isnan(bf16_bits_to_f32(f32_to_bf16_bits(np.array([np.nan], np.float32))))[0]


@pytest.mark.parametrize("case", EMB_CASES)
def test_embedding_oracle_bit_exact(case):
    d = load_golden(case)
    m = d["meta"]
    y = rtn.embedding_rtn(d["ids"], d["qweight_u8"], d["scales"], m["scales_dtype"], d["zeros"], m["zeros_dtype"],
                          m["dim"], m["out_dtype"])
    np.testing.assert_array_equal(y, d["y"])


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_codec_oracle_bit_exact(case):
    """The conv codec's encoder and its weight dequant (the RTN arithmetic) against the
    reference's own outputs."""
    d = load_golden(case)
    m = d["meta"]
    w2 = d["weight_f32"].reshape(d["weight_f32"].shape[0], -1)
    q, s16, z16, cols = rtn.quantize_conv_weight_f32(w2, m["groupsize"])
    assert cols == m["cols"]
    np.testing.assert_array_equal(q, d["qweight"])
    np.testing.assert_array_equal(s16, d["scales"])
    np.testing.assert_array_equal(z16, d["zeros"])
    for od in ("bf16", "f16"):
        w = rtn.dequant_rtn(d["qweight"], d["scales"], "f16", d["zeros"], "f16", cols, q.shape[0], od)
        np.testing.assert_array_equal(w, d[f"w_{od}"])


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_quantizer_matches_reference(case):
    """The package's host-side quantize_conv_weight (torch, CPU) reproduces the reference's."""
    import torch
    from onecomp_runtime.layers import quantize_conv_weight
    d = load_golden(case)
    w2 = torch.from_numpy(d["weight_f32"].reshape(d["weight_f32"].shape[0], -1))
    q, s, z, cols = quantize_conv_weight(w2, groupsize=d["meta"]["groupsize"])
    np.testing.assert_array_equal(q.numpy(), d["qweight"])
    np.testing.assert_array_equal(s.view(torch.int16).numpy().view(np.uint16), d["scales"])
    np.testing.assert_array_equal(z.view(torch.int16).numpy().view(np.uint16), d["zeros"])


def test_conv_nibble_pack_roundtrip():
    import torch
    from onecomp_runtime.layers.packed_conv import pack_int4_nibbles, unpack_int4_nibbles
    codes = torch.randint(0, 16, (5, 37), generator=torch.Generator().manual_seed(3))
    packed = pack_int4_nibbles(codes)
    assert packed.shape == (5, 19) and packed.dtype == torch.uint8
    assert torch.equal(unpack_int4_nibbles(packed, 37).to(torch.int64), codes)


@pytest.mark.parametrize("case", GPTQ_CASES)
def test_gptq_torch_restatement_matches(case):
    """The torch restatement used to prepare the CPU baseline's weights equals the numpy oracle."""
    import torch
    d = load_golden(case)
    m = d["meta"]
    s = d["scales"]
    if m["scales_dtype"] == "f32":
        st = torch.from_numpy(s.astype(np.float32))
    else:
        st = torch.from_numpy(s.view(np.int16).copy()).view(
            torch.bfloat16 if m["scales_dtype"] == "bf16" else torch.float16)
    out = gptq.dequant_gptq_torch(torch.from_numpy(d["qweight"]), st, torch.from_numpy(d["qzeros"]),
                                  torch.from_numpy(d["g_idx"]), m["K"], m["N"], torch.bfloat16, v1=m["v1"],
                                  wbits=m["wbits"])
    ref = gptq.dequant_gptq(d["qweight"], d["scales"], m["scales_dtype"], d["qzeros"], d["g_idx"], m["K"], m["N"],
                            "bf16", v1=m["v1"], wbits=m["wbits"])
    np.testing.assert_array_equal(out.view(torch.int16).numpy().view(np.uint16), ref)
