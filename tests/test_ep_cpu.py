"""Expert-parallel MoE orchestration on CPU (gloo, 2 and 4 ranks) against a single-rank run.

Experts are DSV4 byte-packed int2 (dequantized by the oracle, fp32 math) so only
the host-side logic is under test: routing convention, stable expert-major
permutation, split-size exchange, all-to-all dispatch/return, combine.
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

from oracle import dsv4

E, K_TOP, H, F, T = 8, 2, 64, 32, 12


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _experts():
    rng = np.random.default_rng(0)
    ex = []
    for e in range(E):
        mats = {}
        for name, (o, i) in {"gate": (F, H), "up": (F, H), "down": (H, F)}.items():
            codes = rng.integers(0, 4, size=(o, i))
            packed = dsv4.pack_codes(codes, 2)
            s = rng.uniform(0.005, 0.05, size=(o, i // 16)).astype(np.float16).view(np.uint16)
            z = np.full((o, i // 16), 1.5, np.float16).view(np.uint16)
            w = dsv4.dequant_dsv4(packed, s, "f16", z, "f16", 2, 16, i, "f32")
            mats[name] = torch.from_numpy(np.ascontiguousarray(w))
        ex.append(mats)
    return ex


def _ffn_factory(experts, first):
    def ffn(xs, offsets):
        out = torch.zeros((xs.shape[0], H), dtype=torch.float32)
        off = offsets.tolist()
        for le in range(len(off) - 1):
            a, b = off[le], off[le + 1]
            if b > a:
                m = experts[first + le]
                xx = xs[a:b].float()
                h = torch.nn.functional.silu(xx @ m["gate"].t()) * (xx @ m["up"].t())
                out[a:b] = h @ m["down"].t()
        return out
    return ffn


def _inputs():
    g = torch.Generator().manual_seed(1)
    return torch.randn(T, H, generator=g), torch.randn(T, E, generator=g)


def _shared(xx):
    return 0.5 * xx


def _combine(y_sorted, slot_pos, w, shared_out):
    y_tk = y_sorted.index_select(0, slot_pos.long()).view(w.shape[0], w.shape[1], -1)
    out = (y_tk * w.unsqueeze(-1)).sum(1)
    return out if shared_out is None else out + shared_out


def _worker(rank, world, port, out_path, hooks=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from onecomp_runtime.moe import ExpertParallelMoE
    x, logits = _inputs()
    shard = T // world
    xs, ls = x[rank * shard:(rank + 1) * shard], logits[rank * shard:(rank + 1) * shard]
    extra = {"shared": _shared, "combine": _combine} if hooks else {}
    moe = ExpertParallelMoE(E, K_TOP, _ffn_factory(_experts(), rank * (E // world)), **extra)
    y = moe(xs, ls)
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ys, y)
    if rank == 0:
        torch.save(torch.cat(ys), out_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,hooks", [(2, False), (4, False), (2, True)])
def test_ep_matches_single_rank(tmp_path, world, hooks):
    """hooks: a shared expert and a combine callable, as PackedMoE passes them on the GPU."""
    from onecomp_runtime.moe import ExpertParallelMoE
    out = tmp_path / "y.pt"
    mp.spawn(_worker, args=(world, _free_port(), str(out), hooks), nprocs=world, join=True)
    y_ep = torch.load(out)
    x, logits = _inputs()
    y_ref = ExpertParallelMoE(E, K_TOP, _ffn_factory(_experts(), 0))(x, logits)
    if hooks:
        y_ref = y_ref + 0.5 * x
    torch.testing.assert_close(y_ep, y_ref, rtol=1e-5, atol=1e-5)


def test_combine_and_shared_hooks_single_process():
    """The combine hook receives (y_sorted, slot_pos, w, shared_out) and its result is returned;
    without it the shared expert's output is added to the weighted sum."""
    from onecomp_runtime.moe import ExpertParallelMoE
    x, logits = _inputs()
    ffn = _ffn_factory(_experts(), 0)
    shared = _shared
    plain = ExpertParallelMoE(E, K_TOP, ffn)(x, logits)
    with_shared = ExpertParallelMoE(E, K_TOP, ffn, shared=shared)(x, logits)
    torch.testing.assert_close(with_shared, plain + 0.5 * x, rtol=1e-6, atol=1e-6)
    seen = {}

    def combine(y_sorted, slot_pos, w, shared_out):
        seen.update(rows=y_sorted.shape[0], slots=slot_pos.numel(), w=tuple(w.shape))
        y_tk = y_sorted.index_select(0, slot_pos.long()).view(T, K_TOP, -1)
        return (y_tk * w.unsqueeze(-1)).sum(1) + shared_out

    hooked = ExpertParallelMoE(E, K_TOP, ffn, shared=shared, combine=combine)(x, logits)
    assert seen == {"rows": T * K_TOP, "slots": T * K_TOP, "w": (T, K_TOP)}
    torch.testing.assert_close(hooked, with_shared, rtol=1e-6, atol=1e-6)


def test_routing_convention_and_permutation():
    from onecomp_runtime.moe import permute_reference, route_reference
    logits = torch.tensor([[0.0, 2.0, 1.0, 2.0], [3.0, 0.0, 0.0, 0.0]])
    ids, w = route_reference(logits, 2)
    assert ids.tolist() == [[1, 3], [0, 1]]            # ties go to the lower expert id
    torch.testing.assert_close(w.sum(-1), torch.ones(2))
    off, st, sp = permute_reference(ids, 4)
    assert off.tolist() == [0, 1, 3, 3, 4]
    assert st.tolist() == [1, 0, 1, 0]                 # expert 0: t1; expert 1: t0, t1; expert 3: t0
    assert sp.tolist() == [1, 3, 0, 2]


def test_packed_moe_shared_ffn_hook():
    """PackedMoE.shared_ffn feeds the shared expert's handles a contiguous [T, H] input (no expert
    offsets) and refuses a module built without a shared expert; host logic only, on a stub."""
    from onecomp_runtime.moe import PackedMoE

    class Stub:
        _shared = {"gate": object()}

        def _ffn(self, handles, xs, offsets):
            return handles, xs, offsets

    stub = Stub()
    x = torch.randn(4, 3).t()
    handles, xs, offsets = PackedMoE.shared_ffn(stub, x)
    assert handles is stub._shared and xs.is_contiguous() and offsets is None
    torch.testing.assert_close(xs, x)
    stub._shared = None
    with pytest.raises(ValueError, match="no shared expert"):
        PackedMoE.shared_ffn(stub, x)
