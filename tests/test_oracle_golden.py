"""Pin the CPU oracle against golden vectors produced by the reference itself."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import DSV4_CASES, GPTQ_CASES, RTN_CASES, load_golden
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
            from oracle.fp import quantize, to_f32, round_to
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
