"""Loader: the streaming safetensors reader and load_int4_model's integrity checks
(reference diffusion.py:110-114, 160-161, 190-205), on the CPU."""
from __future__ import annotations

import json

import pytest
import torch
from safetensors.torch import load_file, save_file

from onecomp_runtime import _io
from onecomp_runtime.diffusion import load_int4_model
from onecomp_runtime.testing import TinyDiT, write_int4_checkpoint

CFG = dict(in_channels=16, hidden=64, mlp=128, blocks=2)


def test_reader_matches_safetensors(tmp_path):
    g = torch.Generator().manual_seed(0)
    tensors = {
        "a": torch.randn(7, 5, generator=g).to(torch.bfloat16),
        "b": torch.randint(-2**31, 2**31 - 1, (33,), generator=g, dtype=torch.int64).to(torch.int32),
        "c": torch.randn(3, generator=g).half(),
        "empty": torch.empty(0, 4),
        "big": torch.randn(3000, generator=g),
        "u8": torch.randint(0, 256, (17,), generator=g, dtype=torch.uint8),
    }
    p = tmp_path / "t.safetensors"
    save_file(tensors, str(p), metadata={"k": "v"})
    infos, meta = _io.read_header(str(p))
    assert meta == {"k": "v"} and set(infos) == set(tensors)
    # small chunks: several chunks, and "big" larger than a chunk
    st = _io.DeviceStreamer(str(p), "cpu", chunk_bytes=4096, threads=3)
    got = st.load(list(tensors))
    ref = load_file(str(p))
    for k, v in ref.items():
        assert got[k].dtype == v.dtype and got[k].shape == v.shape and torch.equal(got[k], v), k
        if got[k].numel():  # 256-byte offsets within a chunk; host chunks start 64-byte aligned
            assert got[k].data_ptr() % 64 == 0
    with pytest.raises(KeyError):
        st.load(["nope"])


def test_reader_rejects_non_safetensors(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        _io.read_header(str(p))


def _load(path, **kw):
    kw.setdefault("device", "cpu")
    kw.setdefault("warmup", False)
    return load_int4_model(str(path), TinyDiT, **kw)


def test_missing_metadata(tmp_path):
    p = tmp_path / "m.safetensors"
    save_file({"x": torch.zeros(2)}, str(p))
    with pytest.raises(ValueError, match="quant_layers_json"):
        _load(p)


@pytest.mark.parametrize("io", ["stream", "simple"])
def test_missing_parent(tmp_path, io):
    p = tmp_path / "p.safetensors"
    write_int4_checkpoint(p, CFG)
    infos, meta = _io.read_header(str(p))
    entries = json.loads(meta["quant_layers_json"])
    entries.insert(0, dict(entries[0], name="nowhere.qkv"))
    tensors = load_file(str(p))
    save_file(tensors, str(p), metadata=dict(meta, quant_layers_json=json.dumps(entries)))
    with pytest.raises(KeyError, match="nowhere"):
        _load(p, io=io)


@pytest.mark.parametrize("io", ["stream", "simple"])
def test_unexpected_key(tmp_path, io):
    p = tmp_path / "u.safetensors"
    write_int4_checkpoint(p, CFG, extra={"bogus.weight": torch.zeros(3, dtype=torch.bfloat16)})
    with pytest.raises(RuntimeError, match="unexpected keys"):
        _load(p, io=io, quant_layer_filter=lambda n: False)


@pytest.mark.parametrize("io", ["stream", "simple"])
def test_params_left_on_meta(tmp_path, io):
    p = tmp_path / "l.safetensors"
    write_int4_checkpoint(p, CFG)
    with pytest.raises(RuntimeError, match="left on meta"):
        _load(p, io=io, quant_layer_filter=lambda n: False)


def test_bad_io_option(tmp_path):
    p = tmp_path / "b.safetensors"
    write_int4_checkpoint(p, CFG)
    with pytest.raises(ValueError, match="io must be"):
        _load(p, io="mmap")
