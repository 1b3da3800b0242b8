"""Property tests (hypothesis) of host-side logic that the GPU paths share: the MoE routing
convention and expert-major permutation, the loader's chunk planning, and tensor-parallel
sharding of packed GPTQ layers (checked through the oracle's dequantization)."""
from __future__ import annotations

import os
import tempfile

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import gptq

_FAST = settings(max_examples=40, deadline=None)


@_FAST
@given(T=st.integers(0, 24), E=st.integers(1, 12), data=st.data())
def test_permute_reference_properties(T, E, data):
    """offsets are the expert histogram's prefix sum; slot_pos is a permutation that puts each
    (token, slot) inside its expert's segment at a row holding that token; segments keep token
    order (stable)."""
    from onecomp_runtime.moe import permute_reference
    K = data.draw(st.integers(1, E))
    g = torch.Generator().manual_seed(data.draw(st.integers(0, 2**31 - 1)))
    rows = [torch.randperm(E, generator=g)[:K] for _ in range(T)]
    ids = (torch.stack(rows) if rows else torch.empty((0, K), dtype=torch.int64)).to(torch.int32)
    off, tok, pos = permute_reference(ids, E)
    counts = torch.bincount(ids.reshape(-1).long(), minlength=E).to(torch.int32)
    assert int(off[0]) == 0 and int(off[-1]) == T * K
    assert torch.equal(off[1:] - off[:-1], counts)
    assert sorted(pos.tolist()) == list(range(T * K))
    for t in range(T):
        for j in range(K):
            p, e = int(pos[t * K + j]), int(ids[t, j])
            assert int(tok[p]) == t and int(off[e]) <= p < int(off[e + 1])
    for e in range(E):
        seg = tok[int(off[e]):int(off[e + 1])].tolist()
        assert seg == sorted(seg)


@_FAST
@given(T=st.integers(1, 12), E=st.integers(2, 24), data=st.data())
def test_route_reference_properties(T, E, data):
    """top-k of the fp32 softmax in descending order, ties to the lower expert id, weights
    renormalised to sum 1 (integer logits make ties common)."""
    from onecomp_runtime.moe import route_reference
    K = data.draw(st.integers(1, E))
    g = torch.Generator().manual_seed(data.draw(st.integers(0, 2**31 - 1)))
    logits = torch.randint(-2, 3, (T, E), generator=g).float()
    ids, w = route_reference(logits, K)
    p = torch.softmax(logits, dim=-1)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(p[t, e]), e))[:K]
        assert ids[t].tolist() == order
        chosen = p[t, ids[t].long()]
        torch.testing.assert_close(w[t], chosen / chosen.sum(), rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(w.sum(-1), torch.ones(T), rtol=1e-6, atol=1e-6)


@settings(max_examples=30, deadline=None)
@given(sizes=st.lists(st.integers(0, 3000), min_size=1, max_size=10), chunk=st.integers(1, 4000),
       threads=st.integers(1, 3), data=st.data())
def test_streamer_plan_and_load(sizes, chunk, threads, data):
    """Every requested tensor lands in exactly one chunk at a 256-byte aligned offset, members
    of a chunk do not overlap and fit it (a tensor larger than a chunk gets one of its own), and
    the bytes read back equal the file's."""
    from safetensors.torch import save_file

    from onecomp_runtime import _io
    g = torch.Generator().manual_seed(len(sizes) * 7919 + chunk)
    tensors = {f"t{i}": torch.randint(0, 256, (n,), generator=g, dtype=torch.uint8) for i, n in enumerate(sizes)}
    tensors["f"] = torch.randn(3, 5, generator=g)
    keys = data.draw(st.lists(st.sampled_from(sorted(tensors)), min_size=1, unique=True))
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.safetensors")
        save_file(tensors, path)
        ds = _io.DeviceStreamer(path, "cpu", chunk_bytes=chunk, threads=threads)
        plan = ds._plan(keys)
        placed = [k for members, _ in plan for k, _ in members]
        assert sorted(placed) == sorted(keys)
        for members, size in plan:
            spans = sorted((off, off + ds.infos[k].nbytes) for k, off in members)
            assert all(off % 256 == 0 for off, _ in spans)
            assert all(a_end <= b_off for (_, a_end), (b_off, _) in zip(spans, spans[1:]))
            assert spans[-1][1] == size
            assert size <= chunk or len(members) == 1
        out = ds.load(keys)
        for k in keys:
            assert out[k].dtype == tensors[k].dtype and torch.equal(out[k], tensors[k])


def _dequant(t: dict, K: int, N: int) -> np.ndarray:
    s_bits = t["scales"].view(torch.int16).numpy().view(np.uint16)
    return gptq.dequant_gptq(t["qweight"].numpy(), s_bits, "f16", t["qzeros"].numpy(), t["g_idx"].numpy(), K, N, "f32")


@settings(max_examples=25, deadline=None)
@given(world=st.sampled_from([1, 2, 4]), parts=st.sampled_from([1, 3]), gs=st.sampled_from([32, 64, 128]),
       kmul=st.integers(1, 3), nmul=st.integers(1, 3), seed=st.integers(0, 1000))
def test_tp_shards_dequantize_to_slices(world, parts, gs, kmul, nmul, seed):
    """Each column shard dequantizes to its rows of the full weight (q | k | v blocks kept
    apart when parts = 3), each row shard to its K columns, with bias on rank 0 only."""
    from onecomp_runtime.tensor_parallel import shard_gptq_columns, shard_gptq_rows
    from onecomp_runtime.testing import gptq_layer
    K, N = world * gs * kmul, world * parts * 8 * nmul
    t = gptq_layer(K, N, gs, seed=seed)
    w = _dequant(t, K, N)
    blk, n = N // parts, N // parts // world
    for r in range(world):
        c = shard_gptq_columns(t, r, world, parts=parts)
        rows = np.concatenate([np.arange(p * blk + r * n, p * blk + (r + 1) * n) for p in range(parts)])
        np.testing.assert_array_equal(_dequant(c, K, len(rows)), w[rows])
        rs = shard_gptq_rows(t, r, world, gs)
        k = K // world
        np.testing.assert_array_equal(_dequant(rs, k, N), w[:, r * k:(r + 1) * k])
        assert ("bias" in rs) == (r == 0)


def test_row_shards_reject_act_order():
    from onecomp_runtime.tensor_parallel import shard_gptq_rows
    from onecomp_runtime.testing import gptq_layer
    t = gptq_layer(256, 64, 32, seed=1, actorder=True)
    with pytest.raises(ValueError, match="act-order"):
        shard_gptq_rows(t, 0, 2, 32)
    shard_gptq_rows(t, 0, 1, 32)  # one rank keeps the whole layer


@settings(max_examples=60, deadline=None)
@given(G=st.integers(1, 12), gs=st.sampled_from([8, 16, 26, 32, 64, 128]), kind=st.sampled_from(["natural", "perm", "ragged"]),
       seed=st.integers(0, 10_000))
def test_plan_k_layout_properties(G, gs, kind, seed):
    """The kernels' K layout: every input row k appears once, each group occupies whole 8-row
    words starting on a word boundary, padding rows are -1, and the per-word group table (or the
    uniform groupsize) names the group of every real row."""
    from onecomp_runtime.layers._gptq_base import plan_k_layout
    g = torch.Generator().manual_seed(seed)
    if kind == "ragged":  # irregular group sizes, some groups empty
        gi = torch.sort(torch.randint(0, G, (G * gs,), generator=g)).values
    else:
        gi = torch.arange(G * gs) // gs
        if kind == "perm":
            gi = gi[torch.randperm(G * gs, generator=g)]
    K = gi.numel()
    kp, kperm, word_group, gs_eff = plan_k_layout(K, gs, G, None if kind == "natural" else gi)
    assert kp % 8 == 0 and kp >= K
    if kperm is None:
        assert torch.equal(gi, torch.arange(K) // gs) and gs % 8 == 0 and (kp, word_group, gs_eff) == (K, None, gs)
        return
    perm = kperm.tolist()
    real = [k for k in perm if k >= 0]
    assert sorted(real) == list(range(K)) and len(perm) == kp
    groups = word_group.tolist() if word_group is not None else [w * 8 // gs_eff for w in range(kp // 8)]
    assert len(groups) == kp // 8
    for p, k in enumerate(perm):
        if k >= 0:
            assert int(gi[k]) == groups[p // 8]
    assert groups == sorted(groups)  # groups are contiguous runs of words


@pytest.mark.parametrize("wbits,gs,K,N", [(2, 64, 256, 192), (4, 128, 512, 96), (4, 32, 256, 40)])
def test_gate_up_matrix_dequantizes_to_gate_then_up(wbits, gs, K, N):
    """The [F, 2K] gate|up matrix the fused SwiGLU launch reads dequantizes (oracle restatement of
    the reference's dequant_dsv4_packed) to the gate weights followed by the up weights, row by row,
    bit for bit; layouts it cannot express give None."""
    from oracle import dsv4
    from onecomp_runtime.moe import gate_up_matrix
    from onecomp_runtime.testing import dsv4_packed
    g = dsv4_packed(N, K, wbits, gs, seed=1, zero=None)
    u = dsv4_packed(N, K, wbits, gs, seed=2, zero=None)
    q, s, z = gate_up_matrix(g, u, "cpu")
    G = K // gs
    assert q.shape == (N, 2 * K * wbits // 8) and s.shape == (2 * G, N) and z.shape == (2 * G, N)

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def deq(qq, ss, zz, k):
        return dsv4.dequant_dsv4(qq.numpy(), bits(ss), "f16", bits(zz), "f16", wbits, gs, k, "bf16")

    w_cat = deq(q, s, z, 2 * K)
    w_ref = np.concatenate([deq(g["qweight_packed"], g["scales"], g["qzeros"], K),
                            deq(u["qweight_packed"], u["scales"], u["qzeros"], K)], axis=1)
    np.testing.assert_array_equal(w_cat, w_ref)
    one_group = dsv4_packed(N, K, wbits, K, seed=3)
    assert gate_up_matrix(one_group, one_group, "cpu") is None          # a single group per row
    assert gate_up_matrix(g, dsv4_packed(N, 2 * K, wbits, gs, seed=4), "cpu") is None   # shapes differ
