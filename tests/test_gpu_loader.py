"""load_int4_model on the GPU: the streaming and the per-tensor readers build identical layers,
and the B200 model matches the eager (dequantize + nn.Linear) model of the same checkpoint."""
from __future__ import annotations

import pytest
import torch

from onecomp_runtime.diffusion import load_int4_model
from onecomp_runtime.testing import TinyDiT, write_int4_checkpoint

pytestmark = pytest.mark.gpu


def _load(path, dev, **kw):
    return load_int4_model(str(path), TinyDiT, device=str(dev), dtype="bfloat16", warmup=False, **kw)


@pytest.mark.parametrize("actorder", [False, True])
def test_stream_and_simple_loaders_agree(cuda_device, tmp_path, actorder):
    cfg = dict(in_channels=64, hidden=256, mlp=512, blocks=2)
    p = tmp_path / "ck.safetensors"
    write_int4_checkpoint(p, cfg, groupsize=64 if actorder else 32, actorder=actorder, v1=not actorder)
    a = _load(p, cuda_device, io="stream")
    b = _load(p, cuda_device, io="simple")
    sa, sb = a.state_dict(), b.state_dict()
    assert sa.keys() == sb.keys()
    for k in sa:
        assert sa[k].device.type == "cuda" and torch.equal(sa[k], sb[k]), k
    kind = type(a.blocks[0].qkv).__name__
    assert kind == ("PackedGPTQLinear" if actorder else "FusedInt4Linear"), kind
    x = torch.randn(2, 37, cfg["in_channels"], device=cuda_device).to(torch.bfloat16)
    with torch.no_grad():
        ya, yb = a(x), b(x)
    assert torch.equal(ya, yb)
    e = _load(p, cuda_device, backend="eager", io="simple")
    with torch.no_grad():
        ye = e(x)
    err = float((ya.float() - ye.float()).abs().max() / ye.float().abs().max())
    assert err < 2e-2, err
