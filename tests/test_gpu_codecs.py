"""RTN packed embedding (oc_b200_rtn_embedding) and the int4 conv codecs on the GPU, against
golden vectors produced by the reference (PackedEmbedding, PackedInt4Conv1d / ConvTranspose1d)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import CONV_CASES, EMB_CASES, load_golden
from gpu_util import to_torch
from oracle import rtn

pytestmark = pytest.mark.gpu

_TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous()
    if t.dtype == torch.float32:
        return t.view(torch.int32).cpu().numpy().view(np.uint32)
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _ref_bits(a: np.ndarray) -> np.ndarray:
    return a.view(np.uint32) if a.dtype == np.float32 else a


@pytest.mark.parametrize("case", EMB_CASES)
def test_embedding_bit_exact(cuda_device, case):
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedEmbedding
    d = load_golden(case)
    m = d["meta"]
    s = to_torch(d["scales"], m["scales_dtype"], cuda_device)
    z = to_torch(d["zeros"], m["zeros_dtype"], cuda_device)
    emb = PackedEmbedding(m["vocab"], m["dim"], torch.from_numpy(d["qweight_u8"]).to(cuda_device), s, z)
    y = emb(torch.from_numpy(d["ids"]).to(cuda_device))
    assert y.dtype == _TDT[m["out_dtype"]] and tuple(y.shape) == tuple(d["ids"].shape) + (m["dim"],)
    np.testing.assert_array_equal(_bits(y), _ref_bits(d["y"]))
    assert _lib.read_device_error(cuda_device) == 0


def test_embedding_out_of_range_ids(cuda_device):
    """Ids outside [-vocab, vocab) give zero rows and a device error code (no fault)."""
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedEmbedding
    vocab, dim = 10, 64
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randint(0, 256, (vocab, dim // 2), generator=g, dtype=torch.uint8).to(cuda_device)
    s = (torch.rand(vocab, 2, generator=g) * 0.05 + 0.01).half().to(cuda_device)
    z = torch.full((vocab, 2), 7.0).half().to(cuda_device)
    emb = PackedEmbedding(vocab, dim, q, s, z)
    y = emb(torch.tensor([1, 12, -3, -11], device=cuda_device))
    assert torch.equal(y[1], torch.zeros_like(y[1])) and torch.equal(y[3], torch.zeros_like(y[3]))
    ref = emb(torch.tensor([1, 7], device=cuda_device))
    assert torch.equal(y[0], ref[0]) and torch.equal(y[2], ref[1])
    assert _lib.read_device_error(cuda_device) != 0
    assert _lib.read_device_error(cuda_device) == 0   # reading clears the word


def _conv_module(d, device):
    from onecomp_runtime.layers import PackedInt4Conv1d, PackedInt4ConvTranspose1d
    m = d["meta"]
    cls = PackedInt4ConvTranspose1d if m["transpose"] else PackedInt4Conv1d
    return cls(m["cin"], m["cout"], m["k"], stride=m["stride"], dilation=m["dilation"], groups=m["groups"],
               qweight=torch.from_numpy(d["qweight"]), scales=to_torch(d["scales"], "f16", "cpu"),
               zeros=to_torch(d["zeros"], "f16", "cpu"), cols=m["cols"], bias=torch.from_numpy(d["bias_f32"]),
               causal=m["causal"], pad_mode=m["pad_mode"]).to(device)


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv_codec(cuda_device, case):
    """Weight dequant bit-exact; conv output (cuDNN) within 1e-2 of the reference's CPU conv."""
    d = load_golden(case)
    m = d["meta"]
    mod = _conv_module(d, cuda_device)
    assert mod.qweight.dtype == torch.uint8 and mod.scales.dtype == torch.float16
    for od in ("bf16", "f16"):
        w = mod._materialize(_TDT[od])
        np.testing.assert_array_equal(_bits(w).reshape(-1), d[f"w_{od}"].reshape(-1))
    # fp32 models materialize in fp32 (the oracle's restatement of the same arithmetic)
    w32 = rtn.dequant_rtn(d["qweight"], d["scales"], "f16", d["zeros"], "f16", m["cols"], d["qweight"].shape[0], "f32")
    np.testing.assert_array_equal(_bits(mod._materialize(torch.float32)).reshape(-1), _ref_bits(w32).reshape(-1))
    x = torch.from_numpy(d["x_f32"]).to(cuda_device, torch.bfloat16)
    y = mod(x)
    ref = to_torch(d["y_bf16"], "bf16").float()
    assert tuple(y.shape) == tuple(ref.shape)
    err = float((y.float() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err


def test_replace_conv_with_packed(cuda_device):
    from onecomp_runtime.layers import PackedInt4Conv1d, PackedInt4ConvTranspose1d, replace_conv_with_packed
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Conv1d(8, 16, 3, padding=1), torch.nn.GELU(),
                                torch.nn.ConvTranspose1d(16, 8, 4, stride=2, padding=1))
    x = torch.randn(2, 8, 20)
    stats = replace_conv_with_packed(model, groupsize=8, cast_remaining_to=torch.float16)
    assert stats["replaced"] == 2 and 0 < stats["ratio"] < 0.5
    assert isinstance(model[0], PackedInt4Conv1d) and isinstance(model[2], PackedInt4ConvTranspose1d)
    model = model.to(cuda_device)
    y = model(x.to(cuda_device, torch.float16))
    w0 = model[0]._materialize(torch.float32).reshape(16, 8, 3)
    w2 = model[2]._materialize(torch.float32).reshape(16, 8, 4)
    xr = x.to(cuda_device)
    ref = torch.nn.functional.conv_transpose1d(
        torch.nn.functional.gelu(torch.nn.functional.conv1d(xr, w0, model[0].bias.float(), padding=1)),
        w2, model[2].bias.float(), stride=2, padding=1)
    err = float((y.float() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err


CONV_GEMM_CASES = [
    # cin, cout, k, stride, dilation, padding, batch (None: unbatched), length, groupsize, dtype
    (64, 128, 7, 1, 1, 3, 2, 300, 32, torch.bfloat16),
    (96, 64, 3, 2, 1, 0, 3, 257, 32, torch.float16),
    (32, 96, 3, 1, 9, 9, 1, 200, 8, torch.bfloat16),     # dilated residual-unit shape
    (13, 40, 5, 1, 1, 2, None, 128, -1, torch.bfloat16),  # C k = 65: K padded to 72, per-row groups
]


@pytest.mark.parametrize("case", CONV_GEMM_CASES, ids=lambda c: f"c{c[0]}o{c[1]}k{c[2]}s{c[3]}d{c[4]}")
def test_conv1d_runs_as_im2col_gemm(cuda_device, case):
    """Ungrouped PackedInt4Conv1d on the GPU: im2col + the row-packed RTN GEMM (no cuDNN), against
    the fp64 convolution of the bit-exact dequantized weight."""
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedInt4Conv1d
    from onecomp_runtime.layers.packed_conv import quantize_conv_weight
    cin, cout, k, stride, dil, pad, batch, L, gs, dt = case
    g = torch.Generator().manual_seed(cin * 7 + k)
    w = torch.randn(cout, cin, k, generator=g) * 0.1
    q, s, z, cols = quantize_conv_weight(w.reshape(cout, -1), groupsize=gs)
    bias = torch.randn(cout, generator=g) * 0.1
    mod = PackedInt4Conv1d(cin, cout, k, stride=stride, padding=pad, dilation=dil, qweight=q, scales=s, zeros=z,
                           cols=cols, bias=bias, pad_mode="none").to(cuda_device)
    shape = (cin, L) if batch is None else (batch, cin, L)
    x = torch.randn(*shape, generator=g).to(cuda_device, dt)
    y = mod(x)
    assert mod.__dict__.get("_lin") is not None and mod.__dict__["_lin"]._rows_handle() is not None
    wq = mod._materialize(dt).double()
    ref = torch.nn.functional.conv1d(x.double(), wq, bias.to(dt).double().to(cuda_device), stride, pad, dil)
    assert y.dtype == dt and tuple(y.shape) == tuple(ref.shape)
    err = float((y.double() - ref).abs().max() / ref.abs().max())
    assert err < 1e-2, err
    assert _lib.read_device_error(cuda_device) == 0
