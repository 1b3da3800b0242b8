"""Tensor-parallel sharding of packed GPTQ int4 linears (one process per GPU, NCCL).

The reference has no distributed code; this is the multi-GPU layer the north
star asks for on the video-DiT stack:

* column-parallel (``shard_gptq_columns``): split N. qweight/scales columns,
  qzeros word-columns (N/world must stay a multiple of 8), bias columns;
* row-parallel (``shard_gptq_rows``): split K. qweight rows (K/world must be a
  multiple of the groupsize and of 8), scales/qzeros rows; the bias is added by
  rank 0 only so the all-reduce sums it once;
* ``RowParallelInt4Linear.forward`` runs the local GEMM in M-chunks, each
  chunk's GEMM writing straight into its rows of the output, and issues an
  asynchronous all-reduce (sum, bf16) per chunk, so the reduction of chunk i
  overlaps the GEMM of chunk i+1; the current stream waits on every chunk's
  reduction before returning. ``forward_async`` does one chunk without the wait,
  for callers that pipeline whole blocks chunk by chunk (the reduction of one
  chunk then overlaps the following layers' GEMMs of the other chunks). A
  residual (the DiT block's skip connection) is added in rank 0's GEMM epilogue
  before the reduction, so the sum carries it once and no separate elementwise
  pass runs;
* ``ColumnParallelInt4Linear.forward(x, activation=...)`` applies an elementwise
  activation (tanh-GELU) in the GEMM epilogue: the shard's outputs are whole
  features, so the activation needs no communication.

Sharding helpers are plain tensor slicing and run on any device; the linears
themselves are the B200 modules (``FusedInt4Linear`` / ``FusedInt4LinearAnyGroup``).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_gptq_columns(t: dict, rank: int, world: int, parts: int = 1) -> dict:
    """Column shard of a packed GPTQ layer (split output features).

    ``parts > 1`` treats the output as ``parts`` equal blocks (e.g. q | k | v) and
    gives each rank its slice of every block, concatenated in block order, so a
    fused qkv shard holds the rank's q, k and v columns.
    """
    N = t["scales"].shape[1]
    if N % (world * parts) or (N // (world * parts)) % 8:
        raise ValueError(f"N={N} does not split into {world}x{parts} shards of a multiple of 8")
    blk = N // parts
    n = blk // world
    spans = [(p * blk + rank * n, p * blk + (rank + 1) * n) for p in range(parts)]

    def cols(x, div=1):
        return torch.cat([x[:, lo // div:hi // div] for lo, hi in spans], dim=1).contiguous()

    out = {"qweight": cols(t["qweight"]), "scales": cols(t["scales"]), "qzeros": cols(t["qzeros"], 8)}
    if t.get("g_idx") is not None:
        out["g_idx"] = t["g_idx"]
    if t.get("bias") is not None:
        out["bias"] = torch.cat([t["bias"][lo:hi] for lo, hi in spans]).contiguous()
    return out


def shard_gptq_rows(t: dict, rank: int, world: int, groupsize: int) -> dict:
    """Row shard of a packed GPTQ layer (split input features); bias kept on rank 0."""
    K = t["qweight"].shape[0] * 8
    if K % world or (K // world) % groupsize or (K // world) % 8:
        raise ValueError(f"K={K} does not split into {world} shards aligned to groupsize {groupsize}")
    k = K // world
    g = k // groupsize
    out = {
        "qweight": t["qweight"][rank * k // 8:(rank + 1) * k // 8].contiguous(),
        "scales": t["scales"][rank * g:(rank + 1) * g].contiguous(),
        "qzeros": t["qzeros"][rank * g:(rank + 1) * g].contiguous(),
    }
    if t.get("g_idx") is not None:
        gi = (t["g_idx"][rank * k:(rank + 1) * k] - rank * g).contiguous()
        if gi.numel() and (int(gi.min()) < 0 or int(gi.max()) >= g):
            raise ValueError(f"g_idx of rank {rank}'s rows reaches groups outside its own {g}: an act-order "
                             "layer does not split along K")
        out["g_idx"] = gi
    if t.get("bias") is not None and rank == 0:
        out["bias"] = t["bias"]
    return out


class ColumnParallelInt4Linear(torch.nn.Module):
    """Local column shard; output stays sharded ([M, N/world])."""

    def __init__(self, local: torch.nn.Module):
        super().__init__()
        self.local = local

    def forward(self, x: torch.Tensor, activation: str | None = None) -> torch.Tensor:
        if activation is None:
            return self.local(x)
        return self.local.forward_fused(x, activation=activation)


class _Pending:
    """An all-reduce started on a side stream: ``wait()`` orders the current stream after it."""

    def __init__(self, done: torch.cuda.Event):
        self.done = done

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.done)


class NvlsReducer:
    """In-place sum over the group's ranks of row ranges of one symmetric bf16 buffer, through
    NVLink SHARP: the library's own kernel (``oc_b200_nvls_allreduce_bf16``) reads each rank's
    slice with ``multimem.ld_reduce`` and writes the sum to every rank with ``multimem.st``.

    ``buffer`` ([rows, cols] bf16) is allocated as symmetric memory (one NVLink multicast object
    across the group); the row-parallel GEMMs write their partial outputs straight into row ranges
    of it (``view``), and ``all_reduce_async`` reduces such a range on a side stream, ordered after
    the current stream's work, returning a handle whose ``wait()`` orders the current stream after
    the reduction. Every rank must make the same calls in the same order. Raises at construction
    when the devices offer no multicast (then use NCCL: ``RowParallelInt4Linear`` without a reducer).
    """

    def __init__(self, rows: int, cols: int, group=None, blocks: int = 8):
        import torch.distributed._symmetric_memory as symm
        from . import _lib
        self._lib = _lib
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.blocks = int(blocks)
        dev = torch.device("cuda", torch.cuda.current_device())
        if not symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, dev.index):
            raise RuntimeError("NvlsReducer: these GPUs offer no NVLink multicast (NVLS)")
        self.buffer = symm.empty((rows, cols), dtype=torch.bfloat16, device=dev)
        self._h = symm.rendezvous(self.buffer, self.group)
        self._mc = int(self._h.multicast_ptr)
        if self._mc == 0:
            raise RuntimeError("NvlsReducer: the symmetric buffer has no multicast mapping")
        self.flags = symm.empty((2 * self.blocks * self.world,), dtype=torch.int32, device=dev)
        self.flags.zero_()
        self._fh = symm.rendezvous(self.flags, self.group)
        self._flag_ptrs = int(self._fh.buffer_ptrs_dev)
        self.epoch = 0
        self.stream = torch.cuda.Stream(dev)
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)  # every rank's flags are zero before any reduction starts

    def view(self, r0: int, r1: int) -> torch.Tensor:
        return self.buffer[r0:r1]

    def _offset(self, t: torch.Tensor) -> int:
        off = t.data_ptr() - self.buffer.data_ptr()
        if not (t.is_contiguous() and 0 <= off and off + t.numel() * 2 <= self.buffer.numel() * 2):
            raise ValueError("NvlsReducer: the tensor must be a contiguous row range of the buffer")
        return off

    def all_reduce_async(self, t: torch.Tensor, rms_norm_eps: float | None = None,
                         gain: torch.Tensor | None = None) -> _Pending:
        """Sum ``t`` (a row range of ``buffer``) over the ranks, in place, on the side stream.

        With ``rms_norm_eps`` the same kernel pass also normalizes every row of the sum,
        ``s * rsqrt(mean(s**2) + eps)`` (times ``gain``, a [cols] bf16 vector, when given), each
        rank normalizing only its share of the rows (``oc_b200_nvls_allreduce_rmsnorm_bf16``).
        """
        off = self._offset(t)
        if rms_norm_eps is not None and (off % (2 * self.buffer.shape[1]) or t.numel() % self.buffer.shape[1]):
            raise ValueError("NvlsReducer: the normalized range must be whole rows of the buffer")
        if rms_norm_eps is not None and gain is not None:
            if gain.dtype != torch.bfloat16 or gain.numel() != self.buffer.shape[1] or not gain.is_contiguous():
                raise ValueError("NvlsReducer: gain must be a contiguous bf16 vector of the buffer's width")
        self.epoch += 1
        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)
        if rms_norm_eps is None:
            self._lib.call("oc_b200_nvls_allreduce_bf16", self._mc + off, t.numel(), self._flag_ptrs, self.rank,
                           self.world, self.epoch & 0xFFFFFFFF, self.blocks, self.stream.cuda_stream)
        else:
            cols = self.buffer.shape[1]
            self._lib.call("oc_b200_nvls_allreduce_rmsnorm_bf16", self._mc + off, t.numel() // cols, cols,
                           None if gain is None else gain.data_ptr(), float(rms_norm_eps), self._flag_ptrs,
                           self.rank, self.world, self.epoch & 0xFFFFFFFF, self.blocks, self.stream.cuda_stream)
            if gain is not None:
                gain.record_stream(self.stream)
        done = torch.cuda.Event()
        done.record(self.stream)
        return _Pending(done)


class RowParallelInt4Linear(torch.nn.Module):
    """Local row shard followed by an all-reduce (sum) of the partial outputs.

    ``chunks`` splits M so each chunk's all-reduce overlaps the next chunk's GEMM.
    """

    def __init__(self, local: torch.nn.Module, group=None, chunks: int = 4):
        super().__init__()
        self.local = local
        self.group = group
        self.chunks = max(1, int(chunks))

    def _local_into(self, x: torch.Tensor, out: torch.Tensor, residual: torch.Tensor | None) -> None:
        """out = x @ W_shard.T (+ bias on rank 0) (+ residual), written in place."""
        if hasattr(self.local, "_gemm_2d") and x.dtype in (torch.float16, torch.bfloat16):
            if x.stride(1) != 1 or x.data_ptr() % 16 or x.stride(0) % 8:
                x = x.contiguous()
            self.local._gemm_2d(x, out, residual)   # residual in the GEMM epilogue
        else:
            out.copy_(self.local(x) if residual is None else self.local(x) + residual)

    def forward_async(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                      out: torch.Tensor | None = None, reducer: "NvlsReducer | None" = None,
                      rms_norm_eps: float | None = None):
        """Start ``all_reduce(x_shard @ W_shard.T) + bias + residual`` for one chunk of rows.

        Runs the local GEMM on the current stream into ``out`` (allocated when None) and issues its
        all-reduce without waiting, so the caller can queue the next chunk's (or the next layer's)
        GEMMs while the reduction crosses NVLink. Returns ``(out, work)``: ``work.wait()`` (None for
        one rank) orders the current stream after the reduction; ``out`` must not be read before.
        The residual is added by rank 0 only, so the sum carries it once. With a ``reducer``,
        ``out`` is a row range of its symmetric buffer and the sum runs on NVLink SHARP
        (``NvlsReducer``) instead of NCCL; ``rms_norm_eps`` (reducer only) makes that reduction also
        RMS-normalize every row, so ``out`` then holds the normalized sum.
        """
        if rms_norm_eps is not None and reducer is None:
            raise ValueError("forward_async: rms_norm_eps needs an NvlsReducer (the norm runs in its kernel)")
        if out is None:
            out = torch.empty((x.shape[0], self.local.out_features), dtype=x.dtype, device=x.device)
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        rank = dist.get_rank(self.group) if world > 1 else 0
        self._local_into(x, out, residual if rank == 0 else None)
        if world == 1:
            return out, None
        if reducer is not None:   # out is a row range of the reducer's symmetric buffer
            return out, reducer.all_reduce_async(out, rms_norm_eps=rms_norm_eps)
        return out, dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """``all_reduce(x_shard @ W_shard.T) + bias + residual``; ``residual`` [M, N] (optional)."""
        M = x.shape[0]
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if world == 1:
            if residual is None:
                return self.local(x)
            return self.local.forward_fused(x, residual=residual)
        out = torch.empty((M, self.local.out_features), dtype=x.dtype, device=x.device)
        step = (M + self.chunks - 1) // self.chunks
        works = []
        for c0 in range(0, M, step):
            c1 = min(M, c0 + step)
            res = residual[c0:c1] if residual is not None else None
            works.append(self.forward_async(x[c0:c1], res, out[c0:c1])[1])
        for w in works:
            w.wait()
        return out


def build_tp_block(tensors: dict, layers, rank: int, world: int, groupsize: int,
                   make_linear: Callable[[dict, int, int], torch.nn.Module], group=None, chunks: int = 4) -> dict:
    """Shard one DiT block: qkv/fc1 column-parallel, out/fc2 row-parallel.

    ``layers`` = ((name, K, N), ...) in the order qkv, out, fc1, fc2; ``make_linear``
    builds the local module from a shard dict and its (K, N).
    """
    (qn, qk, qN), (on, ok, oN), (fn, fk, fN), (gn, gk, gN) = layers
    blk = {}
    blk[qn] = ColumnParallelInt4Linear(make_linear(shard_gptq_columns(tensors[qn], rank, world, parts=3), qk,
                                                   qN // world))
    blk[on] = RowParallelInt4Linear(make_linear(shard_gptq_rows(tensors[on], rank, world, groupsize), ok // world, oN),
                                    group, chunks)
    blk[fn] = ColumnParallelInt4Linear(make_linear(shard_gptq_columns(tensors[fn], rank, world), fk, fN // world))
    blk[gn] = RowParallelInt4Linear(make_linear(shard_gptq_rows(tensors[gn], rank, world, groupsize), gk // world, gN),
                                    group, chunks)
    return blk
