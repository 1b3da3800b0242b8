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
   ``silu(gate) * up``, then down (the dense shared expert runs gate, up and the
   activation as one launch on a [F, 2K] gate|up matrix built at load time);
4. ``combine``: ``y[t] = sum_j w[t,j] * out[slot_pos[t,j]] (+ shared(x)[t])``.

Expert parallelism (``ExpertParallelMoE``): experts are split contiguously
across ranks, tokens are sharded; per layer the routed rows are exchanged with
``all_to_all_single`` (split sizes exchanged first, one host sync for them),
processed by the local experts and sent back. Every step is a pluggable callable
(routing, permutation, row gather, expert FFN, shared expert, combine) so the
host-side logic is tested on CPU with gloo; ``PackedMoE`` supplies device
kernels for each.
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
    local token shard. ``combine(y_sorted, slot_pos, w, shared_out) -> out``, when
    given, replaces the torch weighted sum (``PackedMoE.combine`` is the fused
    kernel). On CUDA the shared expert runs on a side stream, issued before the
    routed rows are exchanged, so it overlaps the all-to-alls and the routed FFN.
    """

    def __init__(self, num_experts: int, k: int, expert_ffn: Callable, route: Callable = route_reference,
                 shared: Callable | None = None, group=None, combine: Callable | None = None,
                 permute: Callable | None = None, gather: Callable | None = None):
        super().__init__()
        self.E = int(num_experts)
        self.k = int(k)
        self.expert_ffn = expert_ffn
        self.route = route
        self.shared = shared
        self.group = group
        self.combine = combine
        # permute(ids [T, k], E) -> (offsets, sorted_token, slot_pos); gather(x, idx) -> x[idx]
        self.permute = permute or permute_reference
        self.gather = gather or (lambda x, idx: x.index_select(0, idx.long()))
        self._side: dict[int, torch.cuda.Stream] = {}

    def _launch_shared(self, x: torch.Tensor):
        """(shared_out, side stream or None): the shared expert, on a side stream on CUDA."""
        if self.shared is None:
            return None, None
        if x.device.type != "cuda":
            return self.shared(x), None
        idx = x.device.index if x.device.index is not None else torch.cuda.current_device()
        side = self._side.get(idx)
        if side is None:
            side = self._side[idx] = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            out = self.shared(x)
        return out, side

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        E, K = self.E, self.k
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        el = E // world
        T, H = x.shape
        shared_out, side = self._launch_shared(x)
        ids, w = self.route(logits, K)
        offsets, sorted_token, slot_pos = self.permute(ids, E)
        x_send = self.gather(x, sorted_token)
        counts = (offsets[1:] - offsets[:-1]).to(torch.int64)                        # per expert, this rank
        if world == 1:
            y_sorted = self.expert_ffn(x_send, offsets)
        else:
            # expert id of each sorted row: the segment its position falls in
            pos = torch.arange(T * K, device=x.device, dtype=offsets.dtype)
            ids_send = torch.searchsorted(offsets[1:].contiguous(), pos, right=True).to(torch.int32)
            send_split = counts.view(world, el).sum(1)
            recv_counts = torch.empty_like(counts)
            dist.all_to_all_single(recv_counts, counts, group=self.group)    # [src][local expert]
            recv_counts = recv_counts.view(world, el)
            recv_split = recv_counts.sum(1)
            splits = torch.cat([send_split, recv_split]).tolist()             # the one host sync
            ss, rs = splits[:world], splits[world:]
            x_recv = x.new_empty((sum(rs), H))
            dist.all_to_all_single(x_recv, x_send.contiguous(), rs, ss, group=self.group)
            e_recv = ids_send.new_empty((sum(rs),))
            dist.all_to_all_single(e_recv, ids_send.contiguous(), rs, ss, group=self.group)
            # rows arrive grouped by source rank; order them by local expert (stable)
            local_e = (e_recv - rank * el).view(-1, 1)
            loc_off, order, back = self.permute(local_e, el)
            y_loc = self.expert_ffn(self.gather(x_recv, order), loc_off)
            y_recv = self.gather(y_loc, back)                                   # back to arrival order
            y_sorted = x.new_empty((T * K, y_recv.shape[1]))
            dist.all_to_all_single(y_sorted, y_recv, ss, rs, group=self.group)
        if side is not None:
            cur = torch.cuda.current_stream(x.device)
            cur.wait_stream(side)
            shared_out.record_stream(cur)
        if self.combine is not None:
            return self.combine(y_sorted, slot_pos, w, shared_out)
        y_tk = y_sorted.index_select(0, slot_pos.long()).view(T, K, -1).float()
        out = (y_tk * w.unsqueeze(-1).float()).sum(1)
        if shared_out is not None:
            out = out + shared_out.float()
        return out.to(x.dtype)


# ----------------------------------------------------------------------------- B200 module
def gate_up_matrix(gate: dict, up: dict, device=None):
    """The [F, 2K] gate|up matrix of one expert for the fused SwiGLU launch
    (``oc_b200_rows_gemm_swiglu``): row n is gate row n followed by up row n (packed bytes
    concatenated along k), scales and zeros group-major ``[2G, F]`` (the gate's groups, then the
    up's). ``gate`` / ``up`` are DSV4 packed dicts of one shape. Returns ``(qweight, scales,
    zeros)``, or None where the layout does not allow it (K a multiple of 64 and of the
    groupsize, more than one group, 16-byte packed rows): then gate and up stay two matrices."""
    from .layers._rows_base import group_major

    def shape(m):
        return (int(m["wbits"]), int(m["groupsize"]), int(m["in_features"]), tuple(m["qweight_packed"].shape))

    if shape(gate) != shape(up):
        return None
    wbits, gs, K, (N, ldb) = shape(gate)
    if K % 64 or not (0 < gs < K) or K % gs or ldb * 8 != K * wbits or ldb % 16:
        return None
    dev = device if device is not None else gate["qweight_packed"].device
    q = torch.cat([gate["qweight_packed"].to(dev), up["qweight_packed"].to(dev)], dim=1).contiguous()
    s = torch.cat([group_major(gate["scales"].to(dev), N, K, gs), group_major(up["scales"].to(dev), N, K, gs)])
    z = torch.cat([group_major(gate["qzeros"].to(dev), N, K, gs), group_major(up["qzeros"].to(dev), N, K, gs)])
    return q, s, z


class PackedMoE(torch.nn.Module):
    """Routed packed experts (+ optional shared expert) on the sm_100a kernels.

    ``experts[e]`` and ``shared`` are dicts ``{"gate", "up", "down"}`` of DSV4
    packed dicts (``qweight_packed``, ``scales``, ``qzeros``, ``wbits``,
    ``groupsize``, ``in_features``), the format ``Dsv4PackedLinear`` takes.
    All routed experts share one shape. ``forward(x [T, H], logits [T, E])``.
    ``fuse_gate_up`` picks where gate, up and silu(gate) * up run as one launch on a gate|up
    matrix (``oc_b200_rows_gemm_swiglu``) instead of two GEMMs and the silu-mul kernel (same
    bits): ``"shared"`` (default) the dense shared expert only, ``True`` the routed experts too,
    ``False`` neither. Measured at config 3 on B200: shared expert 0.45 ms fused against 0.47;
    routed experts 2.77 ms fused against 2.72 (2.84 against 2.65 once the silu-mul pass was
    vectorized), also with the epilogue overlapped.
    """

    def __init__(self, experts: list[dict], shared: dict | None = None, k: int = 8, renorm: bool = True,
                 device="cuda", fuse_gate_up: bool | str = "shared"):
        super().__init__()
        from . import _lib
        from .layers._rows_base import MODE_EXACT, RowsHandle, group_major
        dev = torch.device(device)
        _lib.require_b200(dev)
        self.E = len(experts)
        self.k = int(k)
        self.renorm = bool(renorm)
        self.device = dev

        def shape(m: dict):
            return (int(m["wbits"]), int(m["groupsize"]), int(m["in_features"]), int(m["qweight_packed"].shape[0]),
                    int(m["qweight_packed"].shape[1]))

        def build(mats: list[dict]):
            wbits, gs, K, N, _ = shape(mats[0])
            q = [m["qweight_packed"].to(dev).contiguous() for m in mats]
            # scales / zeros group-major ([G, N]): the kernel stages each block's rows by TMA
            s = [group_major(m["scales"].to(dev), N, K, gs) for m in mats]
            z = [group_major(m["qzeros"].to(dev), N, K, gs) for m in mats]
            return RowsHandle(q, s, z, wbits, gs if gs > 0 else K, K, N, MODE_EXACT, 1, N)

        def gate_up(gates: list[dict], ups: list[dict]):
            """The experts' gate|up matrices as one handle for the fused SwiGLU launch, or None."""
            if any(shape(m) != shape(gates[0]) for m in gates + ups):
                return None
            mats = [gate_up_matrix(g, u, dev) for g, u in zip(gates, ups)]
            if any(m is None for m in mats):
                return None
            q, s, z = ([m[i] for m in mats] for i in range(3))
            if len({t.dtype for t in s}) != 1 or len({t.dtype for t in z}) != 1:
                return None
            wbits, gs, K, N, _ = shape(gates[0])
            return RowsHandle(q, s, z, wbits, gs, 2 * K, N, MODE_EXACT, 1, N)

        def handles(ex: list[dict], fuse: bool) -> dict:
            gu = gate_up([e["gate"] for e in ex], [e["up"] for e in ex]) if fuse else None
            h = {"gate_up": gu} if gu is not None else {n: build([e[n] for e in ex]) for n in ("gate", "up")}
            h["down"] = build([e["down"] for e in ex])
            return h

        if fuse_gate_up not in (True, False, "shared"):
            raise ValueError(f"fuse_gate_up must be True, False or 'shared', not {fuse_gate_up!r}")
        self._h = handles(experts, fuse_gate_up is True)
        self._shared = handles([shared], bool(fuse_gate_up)) if shared else None
        g0 = experts[0]["gate"]
        self.hidden = int(g0["in_features"])
        self.ffn = int(g0["qweight_packed"].shape[0])

    def _ffn(self, handles, xs: torch.Tensor, offsets: torch.Tensor | None) -> torch.Tensor:
        from . import _lib
        P = xs.shape[0]
        if P == 0:
            return xs.new_empty((0, handles["down"].N))
        if "gate_up" in handles:   # gate, up and silu(gate) * up in one grouped launch
            h = torch.empty((P, handles["gate_up"].N), dtype=xs.dtype, device=xs.device)
            handles["gate_up"].gemm_swiglu(xs, h, offsets)
        else:
            F_ = handles["gate"].N
            g = torch.empty((P, 2 * F_), dtype=xs.dtype, device=xs.device)
            handles["gate"].gemm(xs, g[:, :F_], offsets)
            handles["up"].gemm(xs, g[:, F_:], offsets)
            h = torch.empty((P, F_), dtype=xs.dtype, device=xs.device)
            _lib.call("oc_b200_silu_mul", g.data_ptr(), g[:, F_:].data_ptr(), g.stride(0), P, F_, h.data_ptr(),
                      h.stride(0), _lib.DT[xs.dtype], _lib.stream_of(xs.device))
        y = torch.empty((P, handles["down"].N), dtype=xs.dtype, device=xs.device)
        handles["down"].gemm(h, y, offsets)
        return y

    def expert_ffn(self, xs: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
        """Grouped SwiGLU FFN over rows sorted by expert (``offsets`` int32 [E+1] on the device)."""
        if xs.shape[0] == 0:
            return xs.new_empty((0, self._h["down"].N))
        return self._ffn(self._h, xs.contiguous(), offsets.to(device=xs.device, dtype=torch.int32))

    def shared_ffn(self, x: torch.Tensor) -> torch.Tensor:
        """The shared expert's SwiGLU FFN over ``x [T, H]`` (the ``shared`` hook of
        ``ExpertParallelMoE``)."""
        if self._shared is None:
            raise ValueError("this PackedMoE has no shared expert")
        return self._ffn(self._shared, x.contiguous(), None)

    def permute(self, ids: torch.Tensor, E: int):
        """Stable expert-major order of ``ids [T, k]`` on the device (``oc_b200_moe_permute``): the
        ``permute`` hook of ``ExpertParallelMoE`` -> (offsets [E+1], sorted_token, slot_pos)."""
        from . import _lib
        T, k = ids.shape
        dev = ids.device
        ids = ids.to(torch.int32).contiguous()
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        sorted_token = torch.empty(T * k, dtype=torch.int32, device=dev)
        slot_pos = torch.empty(T * k, dtype=torch.int32, device=dev)
        _lib.call("oc_b200_moe_permute", ids.data_ptr(), T, k, E, counts.data_ptr(), offsets.data_ptr(),
                  sorted_token.data_ptr(), slot_pos.data_ptr(), _lib.stream_of(dev))
        return offsets, sorted_token, slot_pos

    def gather(self, x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        """``x[idx]`` for 16-bit rows on the device (``oc_b200_gather_rows``): the ``gather`` hook."""
        from . import _lib
        x = x.contiguous()
        P, H = idx.numel(), x.shape[1]
        out = torch.empty((P, H), dtype=x.dtype, device=x.device)
        if P:
            ii = idx.to(torch.int32).contiguous()
            _lib.call("oc_b200_gather_rows", x.data_ptr(), x.stride(0), ii.data_ptr(), P, H, out.data_ptr(),
                      out.stride(0), _lib.stream_of(x.device))
        return out

    def route(self, logits: torch.Tensor, k: int):
        from . import _lib
        T, E = logits.shape
        ids = torch.empty((T, k), dtype=torch.int32, device=logits.device)
        w = torch.empty((T, k), dtype=torch.float32, device=logits.device)
        if T == 0:
            return ids, w
        lg = logits.contiguous()
        _lib.call("oc_b200_moe_route", lg.data_ptr(), _lib.DT[lg.dtype], T, E, k, int(self.renorm), ids.data_ptr(),
                  w.data_ptr(), _lib.stream_of(lg.device))
        return ids, w

    def combine(self, y_sorted: torch.Tensor, slot_pos: torch.Tensor, w: torch.Tensor,
                shared: torch.Tensor | None = None) -> torch.Tensor:
        """``out[t] = sum_j w[t,j] * y_sorted[slot_pos[t*k+j]] (+ shared[t])`` in one kernel
        (fp32 sum, one rounding), the combine hook of ``ExpertParallelMoE``."""
        from . import _lib
        T, k = w.shape
        H = y_sorted.shape[1]
        dev = y_sorted.device
        y = y_sorted.contiguous()
        sp = slot_pos.to(device=dev, dtype=torch.int32).contiguous()
        ww = w.to(device=dev, dtype=torch.float32).contiguous()
        if y.shape[0] != T * k or sp.numel() != T * k:
            raise ValueError(f"combine: {y.shape[0]} rows and {sp.numel()} slots for {T} tokens x top-{k}")
        if shared is not None:
            if shared.shape != (T, H) or shared.dtype != y.dtype:
                raise ValueError(f"shared output {tuple(shared.shape)} {shared.dtype}, expected {(T, H)} {y.dtype}")
            shared = shared.contiguous()
        out = torch.empty((T, H), dtype=y.dtype, device=dev)
        if T == 0:
            return out
        _lib.call("oc_b200_moe_combine", y.data_ptr(), y.stride(0), sp.data_ptr(), ww.data_ptr(), T, k, H,
                  None if shared is None else shared.data_ptr(), 0 if shared is None else shared.stride(0),
                  out.data_ptr(), out.stride(0), _lib.DT[y.dtype], _lib.stream_of(dev))
        return out

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        from . import _lib
        T, H = x.shape
        dev = x.device
        if T == 0:
            return x.new_empty((0, H))
        st = _lib.stream_of(dev)
        x = x.contiguous()
        ids, w = self.route(logits, self.k)
        TK = T * self.k
        counts = torch.empty(self.E, dtype=torch.int32, device=dev)
        offsets = torch.empty(self.E + 1, dtype=torch.int32, device=dev)
        sorted_token = torch.empty(TK, dtype=torch.int32, device=dev)
        slot_pos = torch.empty(TK, dtype=torch.int32, device=dev)
        _lib.call("oc_b200_moe_permute", ids.data_ptr(), T, self.k, self.E, counts.data_ptr(), offsets.data_ptr(),
                  sorted_token.data_ptr(), slot_pos.data_ptr(), st)
        xs = torch.empty((TK, H), dtype=x.dtype, device=dev)
        _lib.call("oc_b200_gather_rows", x.data_ptr(), x.stride(0), sorted_token.data_ptr(), TK, H, xs.data_ptr(),
                  xs.stride(0), st)
        y = self._ffn(self._h, xs, offsets) if TK else xs.new_empty((0, H))
        shared = self._ffn(self._shared, x, None) if self._shared is not None else None
        out = torch.empty((T, H), dtype=x.dtype, device=dev)
        _lib.call("oc_b200_moe_combine", y.data_ptr(), y.stride(0), slot_pos.data_ptr(), w.data_ptr(), T, self.k, H,
                  None if shared is None else shared.data_ptr(), 0 if shared is None else shared.stride(0),
                  out.data_ptr(), out.stride(0), _lib.DT[x.dtype], st)
        return out
