"""A bounded wait that runs out: the kernel reports it and the next calls are correct.

The decode GEMV's failure-test options make the first CTA leave one pipeline stage unissued
(its full barrier is armed by nobody), with a 20 ms bound on the pipeline waits. The consumer
warps' wait runs out, the kernel records its error code and returns; every bulk copy that was
issued is waited for before the CTA exits, the failed CTA still takes its split-K ticket, and
the tile with the failed split is left unwritten. No trap, no fault: the context stays usable,
and the same workspace (or the no-alloc scratch) gives exact results on the following calls.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

WFULL = 0x107  # kDevErrWFull: a consumer's wait for a weight stage gave up


def _layer(device):
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import gptq_layer
    K, N = 5120, 1024   # config-2 style: gptq_v2, act-order gs128, several splits per column tile
    t = gptq_layer(K, N, 128, seed=71, v1=False, actorder=True, bias=True, device=device)
    return PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], t["bias"], 128, 4, False)


def _with_impl(impl, run, device, stall: bool):
    """Run `run()` on decode kernel `impl` (1: split-K TMA GEMV, 3: stream-K GEMV, 4: integer-MMA
    split-K GEMV), with the stall
    options set when `stall`, restoring the previous option values. Returns the device error word."""
    from onecomp_runtime import _lib
    keys = (_lib.OPT_WAIT_US, _lib.OPT_TEST_STALL, _lib.OPT_GEMV_IMPL, _lib.OPT_GEMM_PATH)
    saved = {k: _lib.get_option(k) for k in keys}
    try:
        _lib.set_option(_lib.OPT_GEMV_IMPL, impl)
        _lib.set_option(_lib.OPT_GEMM_PATH, 0)
        if stall:
            _lib.set_option(_lib.OPT_WAIT_US, 20000)  # 20 ms
            _lib.set_option(_lib.OPT_TEST_STALL, 1)   # the first stage of the first CTA is never issued
        out = run()
        torch.cuda.synchronize(device)
    finally:
        for k, v in saved.items():
            _lib.set_option(k, v)
    return out, _lib.read_device_error(device)


def _stalled(run, device):
    return _with_impl(1, run, device, stall=True)[1]


# Columns the first CTA's failure leaves unwritten: split-K (impl 1) one 128-column tile; stream-K
# (impl 3) the 256-column tile its run starts in (5120 x 1024 at gs128: 160 units, 2 per CTA).
@pytest.mark.parametrize("impl,cols", [(1, 128), (3, 256), (4, 128)])
def test_wait_runs_out_then_workspace_calls_are_exact(cuda_device, impl, cols):
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import activations
    layer = _layer(cuda_device)
    x = activations(1, layer.in_features, seed=5).to(cuda_device)
    ref, code = _with_impl(impl, lambda: layer(x), cuda_device, stall=False)
    assert code == 0
    out = torch.full_like(ref, float("nan"))
    _, code = _with_impl(impl, lambda: layer._gemm_2d(x, out), cuda_device, stall=True)
    assert code == WFULL, hex(code)
    assert torch.isnan(out[:, :cols].float()).all()          # the failed tile is not written
    torch.testing.assert_close(out[:, cols:], ref[:, cols:], rtol=0, atol=0)
    for _ in range(2):                                     # same workspace, tickets re-armed
        y, code = _with_impl(impl, lambda: layer(x), cuda_device, stall=False)
        assert code == 0
        torch.testing.assert_close(y, ref, rtol=0, atol=0)


def test_wait_runs_out_then_noalloc_calls_are_exact(cuda_device):
    from onecomp_runtime import _lib
    from onecomp_runtime.testing import activations
    layer = _layer(cuda_device)
    x = activations(1, layer.in_features, seed=6).to(cuda_device)
    ref, _ = _with_impl(1, lambda: layer(x), cuda_device, stall=False)   # the kernel the no-alloc entry runs
    h = layer._get_handle()
    bias = layer.bias

    def noalloc(out):
        return _lib.lib().oc_b200_gptq_gemv_noalloc(
            h, x.data_ptr(), _lib.DT[x.dtype], 1, x.stride(0), bias.data_ptr(), _lib.DT[bias.dtype],
            out.data_ptr(), out.stride(0), _lib.stream_of(cuda_device))

    _lib.check(noalloc(torch.empty_like(ref)), "oc_b200_gptq_gemv_noalloc")  # scratch set up
    torch.cuda.synchronize(cuda_device)
    out = torch.full_like(ref, float("nan"))
    code = _stalled(lambda: _lib.check(noalloc(out), "oc_b200_gptq_gemv_noalloc"), cuda_device)
    assert code == WFULL, hex(code)
    assert torch.isnan(out[:, :128].float()).all()
    for _ in range(2):                                     # the shared scratch's tickets are zero again
        y = torch.full_like(ref, float("nan"))
        _lib.check(noalloc(y), "oc_b200_gptq_gemv_noalloc")
        torch.testing.assert_close(y, ref, rtol=0, atol=0)
    torch.cuda.synchronize(cuda_device)
    assert _lib.read_device_error(cuda_device) == 0


PEER = 0x110  # kDevErrPeer: a cross-rank barrier of the NVLS all-reduce gave up


@pytest.mark.parametrize("fused_norm", [False, True])
def test_nvls_allreduce_peer_that_never_arrives(cuda_device, fused_norm):
    """The NVLS all-reduce's entry barrier (plain, or with the RMS norm) waits for a rank that does
    not exist: a two-rank call on one GPU whose second flag array is a local buffer nobody writes.
    With a 20 ms bound the kernel records the peer-wait code and returns before any multicast
    access (the buffer is never touched, so no multicast object is needed), and the context stays
    usable."""
    from onecomp_runtime import _lib
    blocks, world = 2, 2
    flags = [torch.zeros(2 * blocks * world, dtype=torch.int32, device=cuda_device) for _ in range(world)]
    ptrs = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=cuda_device)
    buf = torch.full((64, 8), 3.0, dtype=torch.bfloat16, device=cuda_device)
    saved = _lib.get_option(_lib.OPT_WAIT_US)
    try:
        _lib.set_option(_lib.OPT_WAIT_US, 20000)
        if fused_norm:
            _lib.call("oc_b200_nvls_allreduce_rmsnorm_bf16", buf.data_ptr(), buf.shape[0], buf.shape[1], None, 1e-6,
                      ptrs.data_ptr(), 0, world, 1, blocks, _lib.stream_of(cuda_device))
        else:
            _lib.call("oc_b200_nvls_allreduce_bf16", buf.data_ptr(), buf.numel(), ptrs.data_ptr(), 0, world, 1,
                      blocks, _lib.stream_of(cuda_device))
        torch.cuda.synchronize(cuda_device)
    finally:
        _lib.set_option(_lib.OPT_WAIT_US, saved)
    assert _lib.read_device_error(cuda_device) == PEER
    assert torch.equal(buf, torch.full_like(buf, 3.0))
    # this rank's own arrival was recorded in the other rank's array, and nothing else
    assert int(flags[1][0 * blocks * world + 0 * world + 0]) == 1
    assert int(flags[0].sum()) == 1 * blocks  # its own slot of each block, from itself
    y = buf.float() * 2                         # the context is still usable
    torch.cuda.synchronize(cuda_device)
    assert float(y[0, 0]) == 6.0
    assert _lib.read_device_error(cuda_device) == 0
