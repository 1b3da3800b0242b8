"""Packed-expert MoE layer on B200, single GPU and expert-parallel.

The reference keeps DSV4 routed experts packed on the host and, per call,
copies each routed expert to the GPU, dequantizes it and runs ``F.linear``
(``layers/dsv4_packed_linear.py:95-98``, ``models/dsv4/loader.py:115-119``); the
routing itself lives in an unvendored model file. Here experts stay packed in
HBM and one call does:

1. ``route``: softmax over expert logits (fp32), top-k, renormalised weights;
2. ``permute``: stable per-expert ranking -> ``offsets[E+1]``, ``sorted_token``,
   ``slot_pos``; rows of x gathered into expert-contiguous order;
3. ``expert_ffn``: grouped GEMMs over the expert segments -- gate and up, then
   ``silu(gate) * up``, then down;
4. ``combine``: ``y[t] = sum_j w[t,j] * out[slot_pos[t,j]] (+ shared(x)[t])``.

Expert parallelism (``ExpertParallelMoE``): experts are split contiguously
across ranks, tokens are sharded; per layer the routed rows are exchanged with
``all_to_all_single`` (split sizes exchanged first), processed by the local
experts and sent back. Every step is a pluggable callable so the host-side
logic is tested on CPU with gloo.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class Routing:
    ids: torch.Tensor          # [T, K] int32 expert ids
    weights: torch.Tensor      # [T, K] fp32
    offsets: torch.Tensor      # [E + 1] int32, expert segment starts in sorted order
    sorted_token: torch.Tensor  # [T*K] int32 token of each sorted row
    slot_pos: torch.Tensor     # [T*K] int32 sorted position of (t, j)


def route_reference(logits: torch.Tensor, k: int, renorm: bool = True):
    """The routing convention (fp32 softmax, top-k, ties to the lower id, renormalised)."""
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.sort(p, dim=-1, descending=True, stable=True)
    w, ids = w[..., :k], ids[..., :k]
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids.to(torch.int32), w


def permute_reference(ids: torch.Tensor, E: int):
    """Stable expert-major order of the (token, slot) assignments."""
    T, K = ids.shape
    flat = ids.reshape(-1).long()
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E)
    offsets = torch.zeros(E + 1, dtype=torch.int32, device=ids.device)
    offsets[1:] = torch.cumsum(counts, 0).to(torch.int32)
    sorted_token = (order // K).to(torch.int32)
    slot_pos = torch.empty_like(order)
    slot_pos[order] = torch.arange(order.numel(), device=ids.device)
    return offsets, sorted_token, slot_pos.to(torch.int32)


class ExpertParallelMoE(torch.nn.Module):
    """Expert-parallel MoE orchestration over a process group.

    ``expert_ffn(x_sorted, offsets_local) -> y_sorted`` runs the local experts on
    rows sorted by local expert id. ``route`` / ``shared`` are callables on the
    local token shard.
    """

    def __init__(self, num_experts: int, k: int, expert_ffn: Callable, route: Callable = route_reference,
                 shared: Callable | None = None, group=None):
        super().__init__()
        self.E = int(num_experts)
        self.k = int(k)
        self.expert_ffn = expert_ffn
        self.route = route
        self.shared = shared
        self.group = group

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        E, K = self.E, self.k
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        el = E // world
        T, H = x.shape
        ids, w = self.route(logits, K)
        offsets, sorted_token, slot_pos = permute_reference(ids, E)
        x_send = x.index_select(0, sorted_token.long())
        ids_send = ids.reshape(-1).index_select(0, torch.argsort(slot_pos.long()))  # expert of each sorted row
        counts = (offsets[1:] - offsets[:-1]).to(torch.int64)                        # per expert, this rank
        if world == 1:
            y_sorted = self.expert_ffn(x_send, offsets)
        else:
            send_split = counts.view(world, el).sum(1)
            recv_counts = torch.empty_like(counts)
            dist.all_to_all_single(recv_counts, counts, group=self.group)    # [src][local expert]
            recv_counts = recv_counts.view(world, el)
            recv_split = recv_counts.sum(1)
            ss, rs = send_split.tolist(), recv_split.tolist()
            x_recv = x.new_empty((sum(rs), H))
            dist.all_to_all_single(x_recv, x_send.contiguous(), rs, ss, group=self.group)
            e_recv = ids_send.new_empty((sum(rs),))
            dist.all_to_all_single(e_recv, ids_send.contiguous(), rs, ss, group=self.group)
            # rows arrive grouped by source rank; order them by local expert (stable)
            local_e = (e_recv.long() - rank * el)
            order = torch.argsort(local_e, stable=True)
            loc_counts = torch.bincount(local_e, minlength=el)
            loc_off = torch.zeros(el + 1, dtype=torch.int32, device=x.device)
            loc_off[1:] = torch.cumsum(loc_counts, 0).to(torch.int32)
            y_loc = self.expert_ffn(x_recv.index_select(0, order), loc_off)
            y_recv = torch.empty_like(y_loc)
            y_recv[order] = y_loc
            y_sorted = x.new_empty((T * K, y_recv.shape[1]))
            dist.all_to_all_single(y_sorted, y_recv, ss, rs, group=self.group)
        y_tk = y_sorted.index_select(0, slot_pos.long()).view(T, K, -1).float()
        out = (y_tk * w.unsqueeze(-1).float()).sum(1)
        if self.shared is not None:
            out = out + self.shared(x).float()
        return out.to(x.dtype)
