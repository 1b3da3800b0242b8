"""Checkpoint I/O for the loader: safetensors bytes -> pinned host staging -> device, overlapped.

``load_int4_model`` (reference ``diffusion.py:152-186``) reads every tensor through
``safe_open.get_tensor`` into pageable host memory and copies it with a blocking ``.to(device)``.
Here the file's own header gives each tensor's byte range; reader threads ``preadv`` the bytes
straight into a ring of pinned staging buffers, and a side CUDA stream copies each filled buffer
to the device with one ``cudaMemcpyAsync`` while the threads fill the next one. Tensors come
back as 256-byte aligned views into a few large device chunks (one copy per chunk, not per
tensor). On a CPU device the bytes are read into ordinary host tensors.
"""
from __future__ import annotations

import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import torch

# safetensors dtype tags (format specification) -> torch dtypes
_DTYPES = {
    "BOOL": torch.bool, "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "I32": torch.int32,
    "I64": torch.int64, "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
}
_ALIGN = 256
_READ_PIECE = 8 << 20  # bytes per reader-thread job


@dataclass(frozen=True)
class TensorInfo:
    dtype: torch.dtype
    shape: tuple[int, ...]
    begin: int  # absolute file offset
    nbytes: int


def read_header(path: str) -> tuple[dict[str, TensorInfo], dict[str, str]]:
    """Parse a safetensors header: ``({name: TensorInfo}, metadata)``."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header)")
        (n,) = struct.unpack("<Q", head)
        if n > (100 << 20):
            raise ValueError(f"{path}: header of {n} bytes")
        hdr = json.loads(f.read(n))
    data_start = 8 + n
    meta = hdr.pop("__metadata__", None) or {}
    infos = {}
    for name, e in hdr.items():
        if e["dtype"] not in _DTYPES:
            raise TypeError(f"{path}: tensor {name!r} has unsupported dtype {e['dtype']}")
        b, t = e["data_offsets"]
        infos[name] = TensorInfo(_DTYPES[e["dtype"]], tuple(int(d) for d in e["shape"]), data_start + b, t - b)
    return infos, meta


def _align(v: int) -> int:
    return (v + _ALIGN - 1) // _ALIGN * _ALIGN


class DeviceStreamer:
    """Stream tensors of one safetensors file to ``device`` (see the module docstring).

    ``chunk_bytes`` sizes the staging buffers and device chunks (a larger tensor gets a chunk of
    its own, filled piece by piece through the ring), ``buffers`` the depth of the pinned ring,
    ``threads`` the reader threads."""

    def __init__(self, path: str, device: torch.device | str, *, chunk_bytes: int = 16 << 20,
                 buffers: int = 4, threads: int = 8) -> None:
        self.path = str(path)
        self.device = torch.device(device)
        self.infos, self.metadata = read_header(self.path)
        self.chunk_bytes = int(chunk_bytes)
        self.buffers = max(2, int(buffers))
        self.threads = max(1, int(threads))

    # ------------------------------------------------------------------ reads
    def _read_into(self, pool: ThreadPoolExecutor, fd: int, dst: torch.Tensor, jobs) -> None:
        """``jobs``: (dst offset, file offset, nbytes); fills the host uint8 tensor ``dst``."""
        arr = dst.numpy()
        futs = []
        for d_off, f_off, n in jobs:
            for p in range(0, n, _READ_PIECE):
                m = min(_READ_PIECE, n - p)
                futs.append(pool.submit(self._pread, fd, memoryview(arr[d_off + p:d_off + p + m]), f_off + p))
        for fu in futs:
            fu.result()

    @staticmethod
    def _pread(fd: int, mv: memoryview, off: int) -> None:
        got = 0
        while got < len(mv):
            n = os.preadv(fd, [mv[got:]], off + got)
            if n <= 0:
                raise OSError(f"short read at offset {off + got}")
            got += n

    # ------------------------------------------------------------------ plan
    def _plan(self, keys):
        """Chunks of (key, offset in chunk) in file order; a tensor larger than a chunk alone."""
        order = sorted(keys, key=lambda k: self.infos[k].begin)
        chunks, cur, size = [], [], 0
        for k in order:
            n = self.infos[k].nbytes
            if n > self.chunk_bytes:
                chunks.append(([(k, 0)], n))
                continue
            off = _align(size)
            if cur and off + n > self.chunk_bytes:
                chunks.append((cur, size))
                cur, off = [], 0
            cur.append((k, off))
            size = off + n
        if cur:
            chunks.append((cur, size))
        return chunks

    def _views(self, chunk: torch.Tensor, members) -> dict[str, torch.Tensor]:
        out = {}
        for k, off in members:
            info = self.infos[k]
            if info.nbytes == 0:
                out[k] = torch.empty(info.shape, dtype=info.dtype, device=chunk.device)
            else:
                out[k] = chunk[off:off + info.nbytes].view(info.dtype).view(info.shape)
        return out

    # ------------------------------------------------------------------ load
    def load(self, keys) -> dict[str, torch.Tensor]:
        """Tensors ``keys`` on the device, in their stored dtype. On CUDA the current stream is
        made to wait for the copies before this returns."""
        keys = list(dict.fromkeys(keys))
        missing = [k for k in keys if k not in self.infos]
        if missing:
            raise KeyError(f"{self.path}: no tensor {missing[:4]}")
        plan = self._plan(keys)
        out: dict[str, torch.Tensor] = {}
        if not plan:
            return out
        fd = os.open(self.path, os.O_RDONLY)
        try:
            with ThreadPoolExecutor(self.threads) as pool:
                if self.device.type != "cuda":
                    for members, size in plan:
                        chunk = torch.empty(size, dtype=torch.uint8)
                        self._read_into(pool, fd, chunk,
                                        [(off, self.infos[k].begin, self.infos[k].nbytes) for k, off in members])
                        out.update(self._views(chunk.to(self.device), members))
                    return out
                out.update(self._load_cuda(pool, fd, plan))
        finally:
            os.close(fd)
        return out

    def _load_cuda(self, pool, fd, plan) -> dict[str, torch.Tensor]:
        dev = self.device
        stage_bytes = min(self.chunk_bytes, max(size for _, size in plan))
        ring = [torch.empty(stage_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(self.buffers)]
        done = [None] * self.buffers  # event: the last copy out of the buffer has finished
        side = torch.cuda.Stream(device=dev)
        cur = torch.cuda.current_stream(dev)
        side.wait_stream(cur)
        out = {}
        slot = 0

        def pieces(members, size):
            """(chunk offset, jobs) pieces of at most stage_bytes each."""
            if len(members) == 1 and size > stage_bytes:  # one large tensor, piece by piece
                k, _ = members[0]
                info = self.infos[k]
                for p in range(0, info.nbytes, stage_bytes):
                    m = min(stage_bytes, info.nbytes - p)
                    yield p, [(0, info.begin + p, m)], m
            else:
                yield 0, [(off, self.infos[k].begin, self.infos[k].nbytes) for k, off in members], size

        with torch.cuda.device(dev):
            for members, size in plan:
                chunk = torch.empty(size, dtype=torch.uint8, device=dev)
                for c_off, jobs, n in pieces(members, size):
                    buf = ring[slot]
                    if done[slot] is not None:
                        done[slot].synchronize()  # the buffer's previous copy has left it
                    self._read_into(pool, fd, buf, jobs)
                    with torch.cuda.stream(side):
                        chunk[c_off:c_off + n].copy_(buf[:n], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(side)
                    done[slot] = ev
                    slot = (slot + 1) % self.buffers
                chunk.record_stream(side)
                out.update(self._views(chunk, members))
            cur.wait_stream(side)
            for ev in done:
                if ev is not None:
                    ev.synchronize()  # the pinned ring is released on return
        return out
