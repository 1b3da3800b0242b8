"""Tensor-parallel sharding + all-reduce orchestration on CPU (gloo, 2 ranks).

The B200 kernels need a GPU, so the local linear here is an oracle-backed CPU
stand-in (exact dequant in numpy, fp32 matmul). What is tested is the host-side
logic: column/row sharding of packed GPTQ tensors, head-aligned qkv shards,
bias-once for row-parallel layers, chunked asynchronous all-reduce, and that a
rank failing fast is reported to the others by the process-group timeout.
"""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import gptq


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleLinear(torch.nn.Module):
    """CPU stand-in: x @ dequant(W).T + b in fp32 via the numpy oracle."""

    def __init__(self, t: dict, K: int, N: int, gs: int):
        super().__init__()
        s_bits = t["scales"].view(torch.int16).numpy().view(np.uint16)
        gi = np.arange(K) // gs
        w = gptq.dequant_gptq(t["qweight"].numpy(), s_bits, "f16", t["qzeros"].numpy(), gi, K, N, "f32")
        self.w = torch.from_numpy(np.ascontiguousarray(w))
        self.b = t["bias"].float() if t.get("bias") is not None else None
        self.in_features, self.out_features = K, N

    def forward(self, x):
        y = x.float() @ self.w.t()
        return y + self.b if self.b is not None else y

    def forward_fused(self, x, residual=None, activation=None):
        y = self.forward(x)
        if activation == "gelu_tanh":
            y = torch.nn.functional.gelu(y, approximate="tanh")
        return y + residual if residual is not None else y


LAYERS = (("qkv", 256, 768), ("out", 256, 256), ("fc1", 256, 512), ("fc2", 512, 256))
GS = 32


def _tensors():
    from onecomp_runtime.testing import gptq_layer
    return {name: gptq_layer(K, N, GS, seed=50 + i) for i, (name, K, N) in enumerate(LAYERS)}


def _block_forward(blk, x, hidden, local_q):
    qkv = blk["qkv"](x)
    h = x + blk["out"](qkv[:, :local_q])
    f = torch.nn.functional.gelu(blk["fc1"](h), approximate="tanh")
    return h + blk["fc2"](f)


def _block_forward_fused(blk, x, local_q):
    """The same block with the residual adds and the GELU folded into the linears' epilogues."""
    qkv = blk["qkv"](x)
    h = blk["out"](qkv[:, :local_q], residual=x)
    f = blk["fc1"](h, activation="gelu_tanh")
    return blk["fc2"](f, residual=h)


def _block_forward_pipelined(blk, x, local_q, chunks):
    """The fused block pipelined over row chunks with forward_async: every chunk's out-projection
    reduction is started before any is waited for, then fc1 / fc2 per chunk."""
    step = (x.shape[0] + chunks - 1) // chunks
    xs = [x[c0:c0 + step] for c0 in range(0, x.shape[0], step)]
    qkv = [blk["qkv"](xc) for xc in xs]
    pend = [blk["out"].forward_async(q[:, :local_q], residual=xc) for q, xc in zip(qkv, xs)]
    pend2 = []
    for o, w in pend:
        if w is not None:
            w.wait()
        f = blk["fc1"](o, activation="gelu_tanh")
        pend2.append(blk["fc2"].forward_async(f, residual=o))
    ys = []
    for o, w in pend2:
        if w is not None:
            w.wait()
        ys.append(o)
    return torch.cat(ys)


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from onecomp_runtime.tensor_parallel import build_tp_block
    tens = _tensors()
    blk = build_tp_block(tens, LAYERS, rank, world, GS, lambda t, K, N: OracleLinear(t, K, N, GS), chunks=3)
    x = torch.randn(10, 256, generator=torch.Generator().manual_seed(0))
    y = _block_forward(blk, x, 256, 256 // world)
    y_fused = _block_forward_fused(blk, x, 256 // world)
    y_pipe = _block_forward_pipelined(blk, x, 256 // world, chunks=3)
    if rank == 0:
        torch.save((y, y_fused, y_pipe), out_path)
    dist.barrier()
    dist.destroy_process_group()


def test_tp_block_matches_single_rank(tmp_path):
    world = 2
    out = tmp_path / "y.pt"
    mp.spawn(_worker, args=(world, _free_port(), str(out)), nprocs=world, join=True)
    y_tp, y_tp_fused, y_tp_pipe = torch.load(out)
    tens = _tensors()
    full = {name: OracleLinear(tens[name], K, N, GS) for name, K, N in LAYERS}
    x = torch.randn(10, 256, generator=torch.Generator().manual_seed(0))
    y_ref = _block_forward(full, x, 256, 256)
    torch.testing.assert_close(y_tp, y_ref, rtol=1e-4, atol=1e-4)
    # residual added once (rank 0's epilogue) before the reduction, GELU in the column shard
    torch.testing.assert_close(y_tp_fused, y_ref, rtol=1e-4, atol=1e-4)
    # chunk pipeline: reductions started per chunk and waited for later give the same block
    torch.testing.assert_close(y_tp_pipe, y_ref, rtol=1e-4, atol=1e-4)


def test_column_and_row_shards_cover_the_layer():
    from onecomp_runtime.tensor_parallel import shard_gptq_columns, shard_gptq_rows
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(256, 192, 32, seed=3)
    cols = [shard_gptq_columns(t, r, 2) for r in range(2)]
    assert torch.equal(torch.cat([c["qweight"] for c in cols], 1), t["qweight"])
    assert torch.equal(torch.cat([c["qzeros"] for c in cols], 1), t["qzeros"])
    assert torch.equal(torch.cat([c["bias"] for c in cols]), t["bias"])
    rows = [shard_gptq_rows(t, r, 4, 32) for r in range(4)]
    assert torch.equal(torch.cat([r["qweight"] for r in rows], 0), t["qweight"])
    assert torch.equal(torch.cat([r["scales"] for r in rows], 0), t["scales"])
    assert "bias" in rows[0] and all("bias" not in r for r in rows[1:])
    with pytest.raises(ValueError):
        shard_gptq_rows(t, 0, 3, 32)
    with pytest.raises(ValueError):
        shard_gptq_columns(t, 0, 5)
    # head-aligned qkv shard: rank r holds q_r | k_r | v_r
    qkv = gptq_layer(64, 288, 32, seed=4)
    sh = shard_gptq_columns(qkv, 1, 2, parts=3)
    n = qkv["scales"].shape[1] // 3 // 2
    expect = torch.cat([qkv["scales"][:, p * 2 * n + n:p * 2 * n + 2 * n] for p in range(3)], 1)
    assert torch.equal(sh["scales"], expect)


def _failing_worker(rank, world, port, flag_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)          # leaves between steps: never joins the next collective
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        err = "none"
    except Exception as e:  # the timeout surfaces as an exception, not a hang
        err = type(e).__name__
    with open(flag_path, "w") as f:
        f.write(err)
    os._exit(0)


def test_missing_rank_times_out_cleanly(tmp_path):
    flag = tmp_path / "flag.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(flag))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert flag.exists() and flag.read_text() != "none"


def test_fused_norm_needs_the_nvls_reducer():
    """The RMS norm rides in the NVLS reduction kernel: asking for it without a reducer is an
    error on the host, before any GEMM runs (one process, no process group)."""
    from onecomp_runtime.tensor_parallel import RowParallelInt4Linear
    layer = RowParallelInt4Linear(torch.nn.Identity(), chunks=1)
    with pytest.raises(ValueError, match="NvlsReducer"):
        layer.forward_async(torch.zeros(4, 8), rms_norm_eps=1e-6)
