"""Edge cases across the layer types on the GPU: empty inputs (no launch, right shape) and
leading batch dimensions (same result as the flattened call)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(dev):
    from onecomp_runtime.layers import Dsv4PackedLinear, PackedGPTQLinear, PackedRTNLinear
    from onecomp_runtime.testing import dsv4_packed, gptq_layer
    K, N = 512, 256
    out = {}
    t4 = {k: v.to(dev) for k, v in gptq_layer(K, N, 128, seed=1, v1=False, actorder=True).items()}
    out["gptq4_actorder"] = PackedGPTQLinear(K, N, t4["qweight"], t4["scales"], t4["qzeros"], t4["g_idx"], t4["bias"],
                                             128, 4, False)
    t8 = {k: v.to(dev) for k, v in gptq_layer(K, N, 64, seed=2, wbits=8).items()}
    out["gptq8"] = PackedGPTQLinear(K, N, t8["qweight"], t8["scales"], t8["qzeros"], t8["g_idx"], t8["bias"], 64, 8,
                                    True)
    g = torch.Generator().manual_seed(3)
    q = torch.randint(0, 256, (N, K // 2), generator=g, dtype=torch.uint8)
    s = (torch.rand(N, 4, generator=g) * 0.02 + 0.002).half()
    z = torch.randint(0, 16, (N, 4), generator=g).half()
    out["rtn"] = PackedRTNLinear(K, N, q.to(dev), s.to(dev), z.to(dev))
    out["dsv4_int2"] = Dsv4PackedLinear(dsv4_packed(N, K, 2, 64, seed=4), buffer_device=dev)
    return K, N, out


@pytest.mark.parametrize("name", ["gptq4_actorder", "gptq8", "rtn", "dsv4_int2"])
def test_empty_and_batched_inputs(cuda_device, name):
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import activations
    K, N, layers = _layers(cuda_device)
    layer = layers[name]
    for shape in ((0, K), (2, 0, K)):
        y = layer(torch.empty(shape, dtype=torch.bfloat16, device=cuda_device))
        assert y.shape == shape[:-1] + (N,) and y.dtype == torch.bfloat16
    for M in (3, 40):  # decode and prefill paths
        x = activations(2 * M, K, seed=M).to(cuda_device)
        y2 = layer(x)
        y3 = layer(x.reshape(2, M, K))
        assert y3.shape == (2, M, N)
        torch.testing.assert_close(y3.reshape(2 * M, N), y2, rtol=0, atol=0)
    assert _lib.read_device_error(cuda_device) == 0


def test_embedding_empty_ids(cuda_device):
    from onecomp_runtime.layers import PackedEmbedding
    vocab, dim = 16, 64
    g = torch.Generator().manual_seed(5)
    q = torch.randint(0, 256, (vocab, dim // 2), generator=g, dtype=torch.uint8).to(cuda_device)
    s = (torch.rand(vocab, 1, generator=g) * 0.05 + 0.01).half().to(cuda_device)
    z = torch.full((vocab, 1), 8.0).half().to(cuda_device)
    emb = PackedEmbedding(vocab, dim, q, s, z)
    for shape in ((0,), (3, 0)):
        y = emb(torch.empty(shape, dtype=torch.long, device=cuda_device))
        assert y.shape == shape + (dim,) and y.dtype == torch.float16
