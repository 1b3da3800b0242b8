"""Tensor- and expert-parallel paths on 2 GPUs over NCCL (skipped with fewer GPUs).

Each test spawns one process per GPU; rank 0 compares the parallel result with the
same layer computed on one GPU with the unsharded weights.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _need_gpus(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    if torch.cuda.get_device_capability(0) != (10, 0):
        pytest.skip("needs sm_100")


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60), device_id=dev)
    return dev


LAYERS = (("qkv", 512, 1536), ("out", 512, 512), ("fc1", 512, 2048), ("fc2", 2048, 512))


def _tp_worker(rank, world, port, out_path):
    dev = _init(rank, world, port)
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.tensor_parallel import build_tp_block
    from onecomp_runtime.testing import gptq_layer

    def make(t, K, N):
        return FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t.get("bias"), 32)

    tens = {n: gptq_layer(K, N, 32, seed=70 + i, device=dev) for i, (n, K, N) in enumerate(LAYERS)}
    x = torch.randn(300, 512, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)

    def fwd(blk, q):
        qkv = blk["qkv"](x)
        h = x + blk["out"](qkv[:, :q])
        return h + blk["fc2"](torch.nn.functional.gelu(blk["fc1"](h), approximate="tanh"))

    def fwd_fused(blk, q):  # residual adds and GELU in the GEMM epilogues, as the benchmark stack runs
        qkv = blk["qkv"](x)
        h = blk["out"](qkv[:, :q], residual=x)
        return blk["fc2"](blk["fc1"](h, activation="gelu_tanh"), residual=h)

    blk = build_tp_block(tens, LAYERS, rank, world, 32, make, chunks=2)
    y, yf = fwd(blk, 512 // world), fwd_fused(blk, 512 // world)
    if rank == 0:
        full = {n: make(tens[n], K, N) for n, K, N in LAYERS}
        ref = fwd(full, 512).float()
        err = max(float((v.float() - ref).abs().max() / ref.abs().max()) for v in (y, yf))
        torch.save(torch.tensor([err]), out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_tp_two_gpus(tmp_path):
    _need_gpus(2)
    out = tmp_path / "err.pt"
    mp.spawn(_tp_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    assert float(torch.load(out)[0]) < 2e-2


def _nvls_worker(rank, world, port, out_path):
    """NvlsReducer (the library's multimem all-reduce kernel): two row ranges of its buffer summed
    over the ranks, each element within one bf16 ulp of the exact sum; then a tensor-parallel
    block whose row-parallel outputs go through it, against the same block on one GPU."""
    dev = _init(rank, world, port)
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.tensor_parallel import NvlsReducer, build_tp_block
    from onecomp_runtime.testing import gptq_layer
    try:
        red = NvlsReducer(300, 512, blocks=8)
    except RuntimeError:
        torch.save(torch.tensor([-1.0, -1.0]), out_path) if rank == 0 else None
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        return
    vals = [torch.randn(300, 512, generator=torch.Generator(device=dev).manual_seed(40 + r), device=dev)
            .to(torch.bfloat16) for r in range(world)]
    red.buffer.copy_(vals[rank])
    pend = [red.all_reduce_async(red.view(0, 128)), red.all_reduce_async(red.view(128, 300))]
    for w in pend:
        w.wait()
    exact = sum(v.float() for v in vals)
    # the switch's bf16 addition: within one bf16 ulp (2^-7 relative at most) of the exact sum
    mismatch = float(((red.buffer.float() - exact).abs() > exact.abs() * 2.0 ** -7 + 1e-30).sum())

    def make(t, K, N):
        return FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t.get("bias"), 32)

    tens = {n: gptq_layer(K, N, 32, seed=70 + i, device=dev) for i, (n, K, N) in enumerate(LAYERS)}
    x = torch.randn(300, 512, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    blk = build_tp_block(tens, LAYERS, rank, world, 32, make, chunks=2)
    r1, r2 = red, NvlsReducer(300, 512, blocks=8)
    spans = [(0, 160), (160, 300)]
    outs = [blk["out"].forward_async(blk["qkv"](x[a:b])[:, :512 // world], residual=x[a:b], out=r1.view(a, b),
                                     reducer=r1) for a, b in spans]
    ys = []
    for (o, w), (a, b) in zip(outs, spans):
        w.wait()
        f = blk["fc1"](o, activation="gelu_tanh")
        y, w2 = blk["fc2"].forward_async(f, residual=o, out=r2.view(a, b), reducer=r2)
        w2.wait()
        ys.append(y.clone())
    y = torch.cat(ys)
    torch.cuda.synchronize(dev)
    if rank == 0:
        full = {n: make(tens[n], K, N) for n, K, N in LAYERS}
        qkv = full["qkv"](x)
        h = x + full["out"](qkv[:, :512])
        ref = (h + full["fc2"](torch.nn.functional.gelu(full["fc1"](h), approximate="tanh"))).float()
        err = float((y.float() - ref).abs().max() / ref.abs().max())
        torch.save(torch.tensor([mismatch, err]), out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_nvls_allreduce_two_gpus(tmp_path):
    _need_gpus(2)
    out = tmp_path / "nvls.pt"
    mp.spawn(_nvls_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    mismatch, err = (float(v) for v in torch.load(out))
    if mismatch < 0:
        pytest.skip("no NVLink multicast on these GPUs")
    assert mismatch == 0
    assert err < 2e-2, err


def _nvls_norm_worker(rank, world, port, out_path):
    """The NVLS all-reduce with the RMS norm in the same kernel: against torch's rms_norm of the
    plain NVLS sum of the same rows (one bf16 ulp), with and without a gain, on a 4096-wide buffer
    (the config-4 hidden size) and a 520-wide one (a partial last vector per lane); rows outside
    the normalized range stay as they were; then a tensor-parallel block whose two reductions
    normalize, against the block on one GPU."""
    dev = _init(rank, world, port)
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.tensor_parallel import NvlsReducer, build_tp_block
    from onecomp_runtime.testing import gptq_layer
    F = torch.nn.functional
    try:
        reds = [NvlsReducer(300, 4096, blocks=8), NvlsReducer(37, 520, blocks=4)]
    except RuntimeError:
        torch.save(torch.tensor([-1.0, -1.0, -1.0]), out_path) if rank == 0 else None
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        return
    bad = 0.0
    for i, red in enumerate(reds):
        R, C = red.buffer.shape
        vals = [torch.randn(R, C, generator=torch.Generator(device=dev).manual_seed(60 + 7 * i + r), device=dev)
                .mul(3.0).to(torch.bfloat16) for r in range(world)]
        gain = torch.rand(C, generator=torch.Generator(device=dev).manual_seed(99 + i), device=dev).add(0.5) \
            .to(torch.bfloat16)
        red.buffer.copy_(vals[rank])
        red.all_reduce_async(red.buffer).wait()
        s = red.buffer.clone()                                   # the switch's bf16 sum
        for g in (None, gain):
            red.buffer.copy_(vals[rank])
            r0 = 5 if R > 100 else 0
            red.all_reduce_async(red.view(r0, R), rms_norm_eps=1e-6, gain=g).wait()
            ref = F.rms_norm(s[r0:].float(), (C,), eps=1e-6)
            if g is not None:
                ref = ref * g.float()
            y = red.buffer[r0:].float()
            bad += float(((y - ref).abs() > ref.abs() * 2.0 ** -7 + 1e-30).sum())
            bad += float((red.buffer[:r0] != vals[rank][:r0]).sum())   # rows outside the range untouched
    torch.cuda.synchronize(dev)
    bad += _lib.read_device_error(dev)

    def make(t, K, N):
        return FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t.get("bias"), 32)

    tens = {n: gptq_layer(K, N, 32, seed=70 + i, device=dev) for i, (n, K, N) in enumerate(LAYERS)}
    x = torch.randn(300, 512, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    blk = build_tp_block(tens, LAYERS, rank, world, 32, make, chunks=2)
    r1, r2 = NvlsReducer(300, 512, blocks=8), NvlsReducer(300, 512, blocks=8)
    ys = []
    for a, b in ((0, 160), (160, 300)):
        o, w = blk["out"].forward_async(blk["qkv"](x[a:b])[:, :512 // world], residual=x[a:b], out=r1.view(a, b),
                                        reducer=r1, rms_norm_eps=1e-6)
        w.wait()
        y, w2 = blk["fc2"].forward_async(blk["fc1"](o, activation="gelu_tanh"), residual=o, out=r2.view(a, b),
                                         reducer=r2, rms_norm_eps=1e-6)
        w2.wait()
        ys.append(y.clone())
    y = torch.cat(ys)
    torch.cuda.synchronize(dev)
    if rank == 0:
        full = {n: make(tens[n], K, N) for n, K, N in LAYERS}
        h = F.rms_norm((x + full["out"](full["qkv"](x)[:, :512])).float(), (512,), eps=1e-6).to(torch.bfloat16)
        ref = F.rms_norm((h + full["fc2"](F.gelu(full["fc1"](h), approximate="tanh"))).float(), (512,), eps=1e-6)
        err = float((y.float() - ref).abs().max() / ref.abs().max())
        torch.save(torch.tensor([bad, err, 0.0]), out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_nvls_allreduce_rmsnorm_two_gpus(tmp_path):
    _need_gpus(2)
    out = tmp_path / "nvls_norm.pt"
    mp.spawn(_nvls_norm_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    bad, err, _ = (float(v) for v in torch.load(out))
    if bad < 0:
        pytest.skip("no NVLink multicast on these GPUs")
    assert bad == 0
    assert err < 2e-2, err


def _ep_worker(rank, world, port, out_path, with_shared):
    dev = _init(rank, world, port)
    from onecomp_runtime.moe import ExpertParallelMoE, PackedMoE
    from onecomp_runtime.testing import dsv4_packed
    E, k, H, F, T = 8, 2, 256, 128, 24
    experts = [{"gate": dsv4_packed(F, H, 2, 64, seed=3 * e, device=dev),
                "up": dsv4_packed(F, H, 2, 64, seed=3 * e + 1, device=dev),
                "down": dsv4_packed(H, F, 2, 64, seed=3 * e + 2, device=dev)} for e in range(E)]
    shared = None
    if with_shared:
        shared = {"gate": dsv4_packed(F, H, 4, 128, seed=900, device=dev),
                  "up": dsv4_packed(F, H, 4, 128, seed=901, device=dev),
                  "down": dsv4_packed(H, F, 4, 128, seed=902, device=dev)}
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=dev)
    el = E // world
    local = PackedMoE(experts[rank * el:(rank + 1) * el], shared, k=k, device=dev)
    sh_fn = local.shared_ffn if with_shared else None
    # with the shared expert: every device hook (permute, gather, combine); without: the torch ones
    hooks = dict(combine=local.combine, permute=local.permute, gather=local.gather) if with_shared else {}
    ep = ExpertParallelMoE(E, k, local.expert_ffn, route=local.route, shared=sh_fn, **hooks)
    sh = T // world
    y = ep(x[rank * sh:(rank + 1) * sh], logits[rank * sh:(rank + 1) * sh])
    ys = [torch.empty_like(y) for _ in range(world)]
    torch.distributed.all_gather(ys, y)
    if rank == 0:
        ref = PackedMoE(experts, shared, k=k, device=dev)(x, logits)
        y = torch.cat(ys)
        err = float((y.float() - ref.float()).abs().max() / ref.float().abs().max())
        torch.save(torch.tensor([err]), out_path)
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


@pytest.mark.parametrize("with_shared", [False, True])
def test_ep_two_gpus(tmp_path, with_shared):
    """Without a shared expert: the torch combine; with one: the fused combine kernel and the
    shared expert on the side stream."""
    _need_gpus(2)
    out = tmp_path / "err.pt"
    mp.spawn(_ep_worker, args=(2, _free_port(), str(out), with_shared), nprocs=2, join=True)
    assert float(torch.load(out)[0]) < 1e-2
