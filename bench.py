"""Benchmark of the int4 linear hot path on B200 (one JSON line on rank 0).

Default workload (the DiT stack the metric quotes at 1/2/4/8 GPUs): a
video-DiT-shaped stack of 12 blocks, hidden 4096 (qkv 4096->12288, out 4096->4096,
fc1 4096->16384, fc2 16384->4096), AutoGPTQ v1 int4 gs32, M = 32768 bf16 tokens N(0,1),
seeded random packed weights (no checkpoints offline). Tensor parallel over the N ranks of
the job: qkv and fc1 column-parallel, out and fc2 row-parallel with an all-reduce (sum) per
row-parallel linear: the library's NVLS kernel (multimem.ld_reduce / multimem.st over symmetric
memory, on 8 SMs the GEMMs leave free), which also applies the block's RMS norm (each rank
normalizes 1/N of the rows and multicasts them); ``--tp-reduce nccl`` runs NCCL and torch's norm
instead. The stack is pipelined over 3 row chunks: each chunk's reduction runs on a side stream
while the following GEMMs of the other chunks run.
Per block: qkv; its q slice stands in for attention; out (+ residual in rank 0's
epilogue); RMS norm; fc1 (tanh-GELU in the epilogue); fc2 (+ residual); RMS norm.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload cfg4|cfg1|cfg2|cfg3] [--no-nested]

* ``value``: tokens/s of the whole job (the same 32768 tokens whatever N: strong scaling),
  device-timed with CUDA events around K steps, max over ranks. Weights and inputs are
  resident in HBM and larger than the 126 MB L2, so nothing needs flushing.
* ``e2e``: the same steps through the public module API with each step's input copied from
  pinned host memory and its output read back (on every rank), double-buffered on side streams.
* ``roofline``: the tcgen05 GEMM launches of the timed steps, each bracketed by CUDA events on
  the stream that launches it: achieved = sum(2 M K N) / sum(durations), against the measured
  bf16 peak (burst when the SM clock held its maximum during the timed region, sustained
  when it was power capped).
* ``comm`` (N > 1): one step's all-reduces timed alone (no GEMM in between) and their share.
* ``cpu_baseline`` (rank 0, N = 1): the reference's CPU eager path restated in ``oracle/``
  (weights dequantized once, torch CPU bf16 ``F.linear``) on a bounded sample: one block at
  ``--cpu-sample-m`` tokens, the same K and W steps as the reference arm, extrapolated x12.
* ``workloads``: the other configurations, each with its own roofline: ``cfg1`` (FLUX-style
  8-block stack, 4608 tokens per GPU, replicas), ``cfg2`` (decode layer set, M = 1/4/16, HBM
  fraction) and ``cfg3`` (packed MoE layer, expert parallel over the N ranks).
* ``--impl reference``: the CPU eager path above as the reference arm (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "onecompression-runtime_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "DiT-stack tokens/s (video-DiT int4 GPTQ stack, 12 blocks, hidden 4096, 32768 tokens, tensor parallel)"
METRIC_CFG1 = "DiT-stack tokens/s (FLUX-style int4 GPTQ stack, 8 blocks, hidden 3072, 4608 tokens per GPU)"

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the dominant kernel of
# each workload, from one ncu capture (profiles/ holds the command and the per-launch figures).
TC_TRAFFIC_CFG1 = 103_200_000     # cfg1: mean of the qkv, proj, fc1, fc2 launches at M = 4608
TC_TRAFFIC_CFG4 = 1_637_000_000   # cfg4: mean of the qkv, out, fc1, fc2 launches at M = 32768
GEMV_TRAFFIC_BYTES_PER_LAUNCH = 21_847_808   # cfg2: q/k/v layer, M = 1, integer GEMV (algorithmic 21.85 MB)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16": d.get("bf16_tflops"),
                "bf16_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


def tensor_peak(peaks: dict, clk: dict | None) -> tuple[float, str]:
    """The bf16 denominator that matches the clocks seen: the burst figure when the SM clock stayed
    at its maximum (a short region), the sustained (power-capped) one otherwise."""
    burst = clk is not None and clk.get("sm_mhz") and clk.get("sm_max_mhz") and \
        clk["sm_mhz"] >= 0.95 * clk["sm_max_mhz"] and "sw_power_cap" not in clk.get("reasons", [])
    if burst:
        return peaks["bf16"], f"{peaks['source']} bf16_tflops (burst: SM clock at its maximum)"
    return peaks["bf16_sustained"], f"{peaks['source']} bf16_tflops_sustained (power-capped clocks)"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock / throttle-reason sampling during the timed region: NVML polled every 5 ms from a
    thread (reads only; no GPU setting is changed), nvidia-smi at 100 ms if NVML is missing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None
        self.thread = None
        self.rows = []
        self.stop_evt = threading.Event()

    def _nvml_loop(self, nv, h):
        names = (("hw_slowdown", nv.nvmlClocksEventReasonHwSlowdown),
                 ("hw_thermal_slowdown", nv.nvmlClocksEventReasonHwThermalSlowdown),
                 ("sw_thermal_slowdown", nv.nvmlClocksEventReasonSwThermalSlowdown),
                 ("sw_power_cap", nv.nvmlClocksEventReasonSwPowerCap))
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self.stop_evt.is_set():
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.rows.append((sm, mx, [n for n, b in names if bits & b]))
            self.stop_evt.wait(0.005)

    def start(self):
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.thread = threading.Thread(target=self._nvml_loop, args=(nv, h), daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            if not self.rows:
                return None
            sm = [r[0] for r in self.rows]
            reasons = sorted({n for r in self.rows for n in r[2]})
            return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(r[1] for r in self.rows)),
                    "reasons": reasons, "samples": len(self.rows), "source": "nvml 5 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i] and "Not" not in r[5 + i]})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "source": "nvidia-smi 100 ms"}


# ----------------------------------------------------------------------------- plumbing
RMS_EPS = 1e-6


def rms_norm(h: torch.Tensor, eps: float = RMS_EPS) -> torch.Tensor:
    """RMS norm without weight, fp32 statistics (torch's fused rms_norm)."""
    return torch.nn.functional.rms_norm(h, (h.shape[-1],), eps=eps)


class Job:
    """Rank, world and device of this process; NCCL process group when N > 1."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None

    def init_gpu(self):
        import datetime
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1 and not torch.distributed.is_initialized():
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
        from onecomp_runtime import _lib
        _lib.require_b200(self.dev)
        return self

    def barrier(self):
        if self.world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(self.dev)

    def max_over_ranks(self, *vals: float) -> list[float]:
        t = torch.tensor(list(vals), dtype=torch.float64, device=self.dev)
        if self.world > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return [float(v) for v in t]

    def close(self):
        if self.world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


class LaunchTimer:
    """CUDA events around every launch of the instrumented kernels (on the launching stream), with
    their algorithmic flops: the roofline's achieved rate and the count of our launches."""

    def __init__(self):
        self.on = False
        self.rec: list = []
        self.launches = 0

    def wrap_gptq(self, layer):
        orig = layer._gemm_2d

        def timed(a_2d, out, residual=None, act=0):
            if not self.on:
                return orig(a_2d, out, residual, act)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            orig(a_2d, out, residual, act)
            e.record()
            self.rec.append((s, e, 2.0 * a_2d.shape[0] * layer.in_features * layer.out_features))
            self.launches += 1 + (1 if layer._relayout else 0)
        layer._gemm_2d = timed

    def wrap_rows(self, handle):
        orig = handle.gemm

        def timed(a, out, offsets=None, bias=None):
            if not self.on:
                return orig(a, out, offsets, bias)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            orig(a, out, offsets, bias)
            e.record()
            self.rec.append((s, e, 2.0 * a.shape[0] * handle.K * handle.N))
            self.launches += 1
        handle.gemm = timed
        orig_sw = handle.gemm_swiglu

        def timed_sw(a, out, offsets=None):   # gate|up handle: K = 2 x hidden, so 2 M K N counts both
            if not self.on:
                return orig_sw(a, out, offsets)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            orig_sw(a, out, offsets)
            e.record()
            self.rec.append((s, e, 2.0 * a.shape[0] * handle.K * handle.N))
            self.launches += 1
        handle.gemm_swiglu = timed_sw

    def start(self):
        self.rec, self.launches, self.on = [], 0, True

    def stop(self) -> tuple[float, float]:
        """(summed launch milliseconds, summed flops); events must have completed."""
        self.on = False
        return sum(s.elapsed_time(e) for s, e, _ in self.rec), sum(f for _, _, f in self.rec)


def timed_steps(job: Job, fn, steps: int, warmup: int, clocks: bool = True, before=None):
    """(max-over-ranks ms per step, clock record) for `steps` calls of fn after `warmup` calls;
    `before()` runs between the warm-up and the timed calls."""
    for _ in range(warmup):
        fn()
    job.barrier()
    if before is not None:
        before()
    clk = ClockSampler(job.local) if clocks else None
    if clk:
        clk.start()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        fn()
    s1.record()
    job.barrier()
    rec = clk.stop() if clk else None
    ms, = job.max_over_ranks(s0.elapsed_time(s1) / steps)
    return ms, rec


def e2e_steps(job: Job, forward, x_shape, steps: int, dtype=torch.bfloat16):
    """Steps through the public API with host buffers: each step's input is copied from pinned host
    memory and its output read back; copies of step i+1 / i-1 overlap step i (double-buffered).
    Returns (max-over-ranks total ms, h2d bytes per step, d2h bytes per step)."""
    dev = job.dev
    g = torch.Generator().manual_seed(99 + job.rank)
    x_host = [torch.randn(x_shape, generator=g).to(dtype).pin_memory() for _ in range(2)]
    y_host = [None, None]
    x_dev = [torch.empty(x_shape, dtype=dtype, device=dev) for _ in range(2)]
    main = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_bytes = [0]

    def run(n):
        for i in range(n):
            b = i & 1
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(in_free[b])
                x_dev[b].copy_(x_host[b], non_blocking=True)
                in_ready[b].record(s_in)
            main.wait_event(in_ready[b])
            y = forward(x_dev[b])
            in_free[b].record(main)
            out_ready[b].record(main)
            if y_host[b] is None or y_host[b].shape != y.shape:
                y_host[b] = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
            out_bytes[0] = y.numel() * y.element_size()
            with torch.cuda.stream(s_out):
                s_out.wait_event(out_ready[b])
                y_host[b].copy_(y, non_blocking=True)
                y.record_stream(s_out)
        main.wait_stream(s_in)
        main.wait_stream(s_out)

    run(2)
    job.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    run(steps)
    e1.record(main)
    job.barrier()
    ms, = job.max_over_ranks(e0.elapsed_time(e1))
    if not torch.isfinite(y_host[(steps - 1) & 1].float()).all():
        raise RuntimeError("non-finite end-to-end output")
    return ms, x_host[0].numel() * x_host[0].element_size(), out_bytes[0]


def roofline_tensor(ms: float, flops: float, peaks: dict, clk, traffic, kernel: str, step_ms_total: float,
                    steps: int) -> dict:
    achieved = flops / (ms / 1e3) / 1e12 if ms > 0 else 0.0
    peak, src = tensor_peak(peaks, clk)
    return {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_unit": "bytes per launch",
            "kernel": kernel, "peak_source": src,
            "gemm_share_of_step": round(ms / step_ms_total, 4) if step_ms_total else None,
            "gemm_ms_per_step": round(ms / steps, 3)}


# ----------------------------------------------------------------------------- CPU eager baseline
def cpu_eager_block(layers, gs: int, M: int, seed: int):
    """The reference CPU eager path for one DiT block (``backend.build_eager``: dequantize once,
    then ``nn.Linear`` in bf16 on the host cores), restated in ``oracle/``: weights from
    ``oracle.gptq.dequant_gptq_torch`` (load time, not timed), each call the block's four
    ``F.linear`` in bf16 plus the glue. Returns ``(run, threads)``."""
    from oracle import gptq
    from oracle.eager import EagerCPU
    from onecomp_runtime.testing import gptq_layer
    torch.set_num_threads(os.cpu_count() or 1)
    mods = {}
    for li, (name, K, N) in enumerate(layers):
        t = gptq_layer(K, N, gs, seed=seed + li)
        w = gptq.dequant_gptq_torch(t["qweight"], t["scales"], t["qzeros"], t["g_idx"], K, N, torch.bfloat16)
        b_bits = t["bias"].view(torch.int16).numpy().view(np.uint16)
        mods[name] = EagerCPU(w.view(torch.int16).numpy().view(np.uint16), "bf16", b_bits, "f16")
        del w, t
    H = layers[0][1]
    x = torch.randn(M, H, dtype=torch.float32).to(torch.bfloat16)

    def run():
        qkv = mods[layers[0][0]](x)
        h = rms_norm(x + mods[layers[1][0]](qkv[:, :H].contiguous()))
        f = torch.nn.functional.gelu(mods[layers[2][0]](h), approximate="tanh")
        return rms_norm(h + mods[layers[3][0]](f))

    return run, torch.get_num_threads()


def time_cpu(run, warmup: int, steps: int) -> float:
    """Seconds per call."""
    for _ in range(warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(steps):
        run()
    return (time.perf_counter() - t0) / steps


def cpu_baseline_cfg4(args) -> dict:
    from onecomp_runtime.testing import CFG4, CFG4_LAYERS
    m, blocks = args.cpu_sample_m, CFG4["blocks"]
    run, cores = cpu_eager_block(CFG4_LAYERS, CFG4["gs"], m, seed=4000)
    per_block = time_cpu(run, args.warmup, args.steps)
    return {"value": round(m / (per_block * blocks), 1), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"one cfg4 block (4 linears + glue) at M={m} tokens per step, {args.steps} steps after "
                      f"{args.warmup} warm-up, torch CPU bf16 F.linear on weights dequantized once by the oracle's "
                      f"formula; tokens/s = M / (block time x {blocks} blocks)",
            "ms_per_sample": round(per_block * 1e3, 3)}


# ----------------------------------------------------------------------------- cfg4: TP video-DiT stack
class TPStack:
    """12 video-DiT blocks of B200 int4 linears sharded over the job's ranks."""

    def __init__(self, job: Job, blocks: int, timer: LaunchTimer, chunks: int = 1, reduce: str = "nccl",
                 M: int = 0, nvls_blocks: int = 32, fused_norm: bool = True):
        from onecomp_runtime.layers import FusedInt4Linear
        from onecomp_runtime.tensor_parallel import NvlsReducer, build_tp_block
        self.chunks = max(1, chunks)
        self.fused_norm = fused_norm
        self.reducers = None
        self.reduce = "none" if job.world == 1 else "nccl"
        if job.world > 1 and reduce == "nvls":
            try:   # two symmetric buffers: out-projection and fc2 partial outputs
                from onecomp_runtime.testing import CFG4
                self.reducers = (NvlsReducer(M, CFG4["hidden"], blocks=nvls_blocks),
                                 NvlsReducer(M, CFG4["hidden"], blocks=nvls_blocks))
                self.reduce = "nvls"
            except RuntimeError as e:
                print(f"[bench] NVLS all-reduce unavailable ({e}); using NCCL", file=sys.stderr)
        from onecomp_runtime.testing import CFG4, CFG4_LAYERS, gptq_layer
        self.gs, self.H = CFG4["gs"], CFG4["hidden"]
        self.hq = self.H // job.world
        self.blocks = []
        for b in range(blocks):
            tens = {name: gptq_layer(K, N, self.gs, seed=4000 + 10 * b + i, device=job.dev)
                    for i, (name, K, N) in enumerate(CFG4_LAYERS)}
            blk = build_tp_block(tens, CFG4_LAYERS, job.rank, job.world, self.gs,
                                 lambda t, K, N: FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"],
                                                                 t.get("bias"), self.gs))
            for mod in blk.values():
                timer.wrap_gptq(mod.local)
            self.blocks.append(blk)
            del tens

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """The stack, pipelined over ``self.chunks`` row chunks. Per block: qkv of every chunk first
        (attention needs all tokens), then per chunk the out-projection with its all-reduce started;
        per chunk, once its reduction is done, norm, fc1 and fc2 with the second all-reduce started;
        per chunk, once that is done, norm and the next block's qkv. Each reduction crosses NVLink
        while the following chunks' GEMMs run."""
        M = h.shape[0]
        step = (M + self.chunks - 1) // self.chunks
        spans = [(c0, min(M, c0 + step)) for c0 in range(0, M, step)]
        hs = [h[c0:c1] for c0, c1 in spans]
        r1, r2 = self.reducers if self.reducers else (None, None)
        # with the NVLS reducers each all-reduce also applies the block's RMS norm (every rank
        # normalizes 1/N of the rows) instead of every rank normalizing every row afterwards
        eps = RMS_EPS if (r1 is not None and self.fused_norm) else None
        qkv = [self.blocks[0]["qkv"](hc) for hc in hs]
        for b, blk in enumerate(self.blocks):
            pend = [blk["out"].forward_async(q[:, :self.hq], residual=hc, out=r1.view(c0, c1) if r1 else None,
                                             reducer=r1, rms_norm_eps=eps)
                    for q, hc, (c0, c1) in zip(qkv, hs, spans)]
            pend2 = []
            for (o, w), (c0, c1) in zip(pend, spans):
                if w is not None:
                    w.wait()
                hn = o if eps is not None else rms_norm(o)   # the NVLS reduction normalized the rows
                f = blk["fc1"](hn, activation="gelu_tanh")
                pend2.append(blk["fc2"].forward_async(f, residual=hn, out=r2.view(c0, c1) if r2 else None,
                                                      reducer=r2, rms_norm_eps=eps))
            nxt = self.blocks[b + 1] if b + 1 < len(self.blocks) else None
            hs, qkv = [], []
            for o, w in pend2:
                if w is not None:
                    w.wait()
                hc = o if eps is not None else rms_norm(o)
                hs.append(hc)
                if nxt is not None:
                    qkv.append(nxt["qkv"](hc))
        return hs[0] if len(hs) == 1 else torch.cat(hs)


def allreduce_alone(job: Job, M: int, H: int, per_step: int, chunks: int, reducer=None) -> float:
    """Milliseconds of one step's row-parallel all-reduces issued back to back (no GEMMs): NCCL, or
    the NVLS kernel on the reducer's symmetric buffer."""
    buf = reducer.buffer if reducer is not None else torch.zeros((M, H), dtype=torch.bfloat16, device=job.dev)
    step = (M + chunks - 1) // chunks

    def once():
        for _ in range(per_step):
            for c0 in range(0, M, step):
                if reducer is not None:
                    reducer.all_reduce_async(buf[c0:c0 + step]).wait()
                else:
                    torch.distributed.all_reduce(buf[c0:c0 + step])

    once()
    ms, _ = timed_steps(job, once, 3, 1, clocks=False)
    return ms


def bench_cfg4(args, job: Job, peaks: dict, with_cpu: bool) -> dict:
    from onecomp_runtime.testing import CFG4, CFG4_LAYERS
    M, H, blocks = CFG4["M"], CFG4["hidden"], (args.blocks or CFG4["blocks"])
    timer = LaunchTimer()
    # row chunks of the pipeline: more chunks overlap more of the reductions but shrink each GEMM;
    # measured: 3 on 8 GPUs 1.295M tokens/s against 1.251M with 2; on 2 GPUs 496.5k against 492.7k
    chunks = args.tp_chunks if args.tp_chunks > 0 else (1 if job.world == 1 else 3)
    reduce = args.tp_reduce if args.tp_reduce != "auto" else "nvls"
    if job.world > 1:
        # The GEMM CTA holds a whole SM's register file, so a reduction gets only SMs the persistent
        # GEMM leaves free: with NVLS, leave exactly the reduction's blocks (measured best at N = 8).
        sms = torch.cuda.get_device_properties(job.dev).multi_processor_count
        cap = args.tc_max_ctas if args.tc_max_ctas >= 0 else (sms - args.nvls_blocks if reduce == "nvls" else 0)
        args.tc_max_ctas = cap
        if cap:
            from onecomp_runtime import _lib
            _lib.set_option(_lib.OPT_TC_MAX_CTAS, cap)
    stack = TPStack(job, blocks, timer, chunks, reduce, M, args.nvls_blocks, fused_norm=not args.no_fused_norm)
    x = torch.randn((M, H), generator=torch.Generator(device=job.dev).manual_seed(5), device=job.dev).to(torch.bfloat16)
    with torch.no_grad():
        y = stack.forward(x)
        torch.cuda.synchronize(job.dev)
        if not torch.isfinite(y).all():
            raise RuntimeError("non-finite stack output")
        ms, clk = timed_steps(job, lambda: stack.forward(x), args.steps, args.warmup, before=timer.start)
        gemm_ms, gemm_flops = timer.stop()
        launches = timer.launches
        ms_e2e, h2d, d2h = e2e_steps(job, stack.forward, (M, H), args.steps)
    flops_step = blocks * sum(2.0 * M * K * N for _, K, N in CFG4_LAYERS)
    line = {"metric": METRIC, "value": round(M / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": job.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random packed weights, N(0,1) activations)",
            "config": {"workload": "cfg4: video-DiT int4 stack, 12 blocks x (qkv 4096->12288, out 4096->4096, "
                                   "fc1 4096->16384, fc2 16384->4096), GPTQ v1 gs32, M=32768 tokens",
                       "tokens": M, "blocks": blocks, "global_batch_tokens": M,
                       "parallelism": f"tp{job.world} (column qkv/fc1, row out/fc2 + NCCL all-reduce)"
                       if job.world > 1 else "tp1 (one GPU, no collective)",
                       "pipeline_chunks": stack.chunks,
                       "nvls_blocks": args.nvls_blocks if stack.reduce == "nvls" else None,
                       "rms_norm": ("in the NVLS all-reduce kernel (each rank normalizes 1/N of the rows)"
                                    if stack.reduce == "nvls" and stack.fused_norm else "torch F.rms_norm"),
                       "allreduce": {"nvls": "own NVLS kernel (multimem.ld_reduce / multimem.st)",
                                     "nccl": "NCCL", "none": "none"}[stack.reduce],
                       "gemm_ctas": args.tc_max_ctas if (job.world > 1 and args.tc_max_ctas > 0) else "one per SM",
                       "l2_flush": "none needed: weights (1.4 GB packed) and activations exceed the 126 MB L2"},
            "e2e": {"value": round(M * args.steps / (ms_e2e / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "every rank copies the step's input in and its output back"},
            "gpu_launches": launches,
            "roofline": roofline_tensor(gemm_ms, gemm_flops, peaks, clk, TC_TRAFFIC_CFG4,
                                        "gptq_gemm_tc_kernel (tcgen05, A = dequantized weights in TMEM)",
                                        ms * args.steps, args.steps),
            "tflops_step": round(flops_step / (ms / 1e3) / 1e12, 1),
            "clocks": clk}
    if job.world > 1:
        ar_ms = allreduce_alone(job, M, H, 2 * blocks, stack.chunks, stack.reducers[0] if stack.reducers else None)
        nbytes = 2 * blocks * M * H * 2
        line["comm"] = {"allreduce_ms_per_step_alone": round(ar_ms, 3), "allreduce_bytes_per_step": nbytes,
                        "allreduce": line["config"]["allreduce"],
                        "busbw_GBs": round(nbytes * 2 * (job.world - 1) / job.world / (ar_ms / 1e3) / 1e9, 1),
                        "alone_over_step": round(ar_ms / ms, 4),
                        "note": "the step overlaps each chunk's reduction with the next chunk's GEMM"}
    del stack
    torch.cuda.empty_cache()
    if job.world > 1 and args.tc_max_ctas:
        # the cap only makes room for the stack's NVLS reductions: the nested workloads get every SM
        from onecomp_runtime import _lib
        _lib.set_option(_lib.OPT_TC_MAX_CTAS, 0)
    if with_cpu:
        line["cpu_baseline"] = cpu_baseline_cfg4(args)
    return line


# ----------------------------------------------------------------------------- cfg1: FLUX-style stack
class DiTStack:
    """8 FLUX-style blocks of FusedInt4Linear layers (random packed weights), one per GPU."""

    def __init__(self, job: Job, blocks: int, timer: LaunchTimer):
        from onecomp_runtime.layers import FusedInt4Linear
        from onecomp_runtime.testing import CFG1, CFG1_LAYERS, gptq_layer
        gs = CFG1["gs"]
        self.blocks = []
        for b in range(blocks):
            blk = {}
            for li, (name, K, N) in enumerate(CFG1_LAYERS):
                t = gptq_layer(K, N, gs, seed=(1000 + 17 * job.rank) * (b + 1) + li, device=job.dev)
                blk[name] = FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t["bias"], gs)
                timer.wrap_gptq(blk[name])
            self.blocks.append(blk)
        self.hidden = CFG1["hidden"]

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """q = qkv(h)[:, :H]; h = rms(h + proj(q)); h = rms(h + fc2(gelu(fc1(h)))), adds/GELU in epilogues."""
        H = self.hidden
        for blk in self.blocks:
            qkv = blk["qkv"](h)
            h = rms_norm(blk["proj"].forward_fused(qkv[:, :H], residual=h))
            f = blk["fc1"].forward_fused(h, activation="gelu_tanh")
            h = rms_norm(blk["fc2"].forward_fused(f, residual=h))
        return h


def bench_cfg1(args, job: Job, peaks: dict, full_line: bool) -> dict:
    from onecomp_runtime.testing import CFG1
    M, blocks = CFG1["M"], (args.blocks or CFG1["blocks"])
    if args.tc_tile:
        from onecomp_runtime import _lib
        _lib.set_option(_lib.OPT_TC_TILE, args.tc_tile)
    timer = LaunchTimer()
    stack = DiTStack(job, blocks, timer)
    x = torch.randn(M, CFG1["hidden"], generator=torch.Generator(device=job.dev).manual_seed(1234 + job.rank),
                    device=job.dev).to(torch.bfloat16)
    steps = args.steps if full_line else max(args.steps, 10)
    with torch.no_grad():
        ms, clk = timed_steps(job, lambda: stack.forward(x), steps, args.warmup, before=timer.start)
        gemm_ms, gemm_flops = timer.stop()
        launches = timer.launches
        e2e = None
        if full_line:
            ms_e2e, h2d, d2h = e2e_steps(job, stack.forward, (M, CFG1["hidden"]), steps)
            e2e = {"value": round(job.world * M * steps / (ms_e2e / 1e3), 1), "unit": "tokens/s",
                   "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    out = {"metric": METRIC_CFG1, "value": round(job.world * M / (ms / 1e3), 1), "unit": "tokens/s",
           "n_gpus": job.world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
           "data": "synthetic (seeded random packed weights, N(0,1) activations)",
           "config": {"workload": "cfg1: FLUX-style DiT int4 stack, 8 blocks x (qkv 3072->9216, proj 3072->3072, "
                                  "fc1 3072->9216, fc2 9216->3072), GPTQ v1 gs32, M=4608 tokens per GPU",
                      "global_batch_tokens": M * job.world, "tokens_per_gpu": M, "blocks": blocks,
                      "parallelism": f"replicas x{job.world} (weak scaling, no collective)",
                      "l2_flush": "none needed: weights 437 MB packed per stack > 126 MB L2"},
           "gpu_launches": launches,
           "roofline": roofline_tensor(gemm_ms, gemm_flops, peaks, clk, TC_TRAFFIC_CFG1 if not args.blocks else None,
                                       "gptq_gemm_tc_kernel (tcgen05, 384-token tiles = 2 x 192)", ms * steps, steps),
           "clocks": clk}
    if e2e:
        out["e2e"] = e2e
    del stack
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- cfg2: decode layer set
def bench_cfg2(args, job: Job, peaks: dict) -> dict:
    """gptq_v2 gs128 act-order layer set (fp16 scales, bf16 activations), M in {1, 4, 16},
    replayed as one CUDA graph of the five layers; every rank runs its own copy (replicas). ``--wbits 8``:
    the same shapes as 8-bit gs128 layers without act-order, bf16 scales (the Qwen3.6 adapter's 8-bit layers).
    Reported: packed bytes streamed per second (qweight + scales + qzeros + g_idx, + activations)."""
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import CFG2_LAYERS, gptq_layer
    if args.gemv_ctas:
        _lib.set_option(_lib.OPT_GEMV_CTAS, args.gemv_ctas)
    if args.gemv_impl >= 0:
        _lib.set_option(_lib.OPT_GEMV_IMPL, args.gemv_impl)
    if args.gemv_prep >= 0:
        _lib.set_option(_lib.OPT_GEMV_PREP, args.gemv_prep)
    dev = job.dev
    layers, nbytes = [], 0
    w8 = args.wbits == 8
    for i, (name, K, N) in enumerate(CFG2_LAYERS):
        G = (K + 127) // 128
        if w8:
            t = gptq_layer(K, N, 128, seed=2000 + i, v1=True, scales_range=(0.001, 0.01),
                           scales_dtype=torch.bfloat16, bias=False, device=dev, wbits=8)
            layers.append(PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], None, 128, 8,
                                           True))
            nbytes += K * N + 2 * G * N + G * N
        else:
            t = gptq_layer(K, N, 128, seed=2000 + i, v1=False, actorder=True, scales_range=(0.001, 0.01),
                           scales_dtype=torch.float16, bias=False, device=dev)
            layers.append(PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], None, 128, 4,
                                           False))
            nbytes += K * N // 2 + 2 * G * N + G * N // 2 + 4 * K
    per_m = {}
    clk = None
    for M in (1, 4, 16):
        xs = [torch.randn(M, K, device=dev).to(torch.bfloat16) for _, K, _ in CFG2_LAYERS]
        act = sum(2 * M * K + 2 * M * N for _, K, N in CFG2_LAYERS)
        for _ in range(3):
            [lay(x) for lay, x in zip(layers, xs)]
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = [lay(x) for lay, x in zip(layers, xs)]
        reps = max(args.steps, 1) * 20   # the set is ~30-150 us; 200+ replays stream 35 GB > L2
        ms, c = timed_steps(job, g.replay, reps, args.warmup, clocks=(M == 16))
        clk = c or clk
        us = ms * 1e3
        gbs = (nbytes + act) / (us * 1e-6) / 1e9
        per_m[str(M)] = {"us_per_set": round(us, 2), "GB_s": round(gbs, 1), "frac_hbm": round(gbs / peaks["hbm_gbs"], 4)}
        del g, outs
    top = per_m["1"]
    kind = "gptq v1 gs128 8-bit" if w8 else "gptq_v2 gs128 act-order"
    out = {"metric": f"decode GB/s ({kind} layer set, M=1)", "value": top["GB_s"], "unit": "GB/s",
           "n_gpus": job.world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "cfg2: q/k/v 5120->8192, o 6144->5120, gate/up 5120->17408, down 17408->5120"
                                  + (", 8-bit codes" if w8 else ", fp16 scales"),
                      "packed_bytes_per_set": nbytes, "graph": "CUDA graph of the 5 layers, replayed",
                      "parallelism": f"replicas x{job.world} (per-GPU figures, max time over ranks)",
                      "l2_flush": "none needed: each replay streams 177 MB of weights > 126 MB L2"},
           "per_m": per_m,
           "roofline": {"bound": "hbm", "achieved": top["GB_s"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": top["frac_hbm"], "traffic": None if w8 else GEMV_TRAFFIC_BYTES_PER_LAUNCH,
                        "traffic_unit": "bytes per launch (q/k/v layer)",
                        "kernel": ("gptq_gemv_tma_kernel (split-K decode GEMV)" if w8 else
                                   "gptq_gemv_i8_kernel (integer-MMA split-K decode GEMV; M = 16: gptq_gemv_tma_kernel)"),
                        "peak_source": f"{peaks['source']} hbm_gbs"},
           "clocks": clk}
    del layers
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- cfg0: one GPTQ linear
def bench_cfg0(args, job: Job, peaks: dict) -> dict:
    """BASELINE config 0 on the GPU: one AutoGPTQ v1 gs32 linear, K = N = 3072, M = 256 bf16 tokens
    (the reference's CPU-runnable case). Its packed weights (5.5 MB) fit L2, so C copies with their
    own weights (> 126 MB in all) run back to back in one CUDA graph; time per linear = graph / C."""
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.testing import CFG0, gptq_layer
    dev = job.dev
    K, N, gs, M = CFG0["K"], CFG0["N"], CFG0["gs"], CFG0["M"]
    per = K * N // 2 + 2 * (K // gs) * N + (K // gs) * N // 2
    C = -(-160_000_000 // per)
    layers = []
    for c in range(C):
        t = gptq_layer(K, N, gs, seed=c, device=dev)
        layers.append(FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t["bias"], gs))
    x = torch.randn((M, K), generator=torch.Generator(device=dev).manual_seed(0), device=dev).to(torch.bfloat16)
    with torch.no_grad():
        for _ in range(3):
            [lay(x) for lay in layers]
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = [lay(x) for lay in layers]
        ms, clk = timed_steps(job, g.replay, max(args.steps, 1) * 5, args.warmup)
    us = ms * 1e3 / C
    tflops = 2.0 * M * K * N / (us * 1e-6) / 1e12
    peak, src = tensor_peak(peaks, clk)
    out = {"metric": "GPTQ int4 linear TFLOP/s (config 0: K=N=3072, gs32, M=256)", "value": round(tflops, 1),
           "unit": "TFLOP/s", "n_gpus": job.world, "steps": args.steps, "warmup": args.warmup,
           "us_per_linear": round(us, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "cfg0", "copies_per_graph": C,
                      "l2_flush": f"none needed: the graph streams {C} copies of 5.5 MB of packed weights"},
           "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tflops / peak, 4), "traffic": None,
                        "kernel": "gptq_gemm_tc_kernel (24 column tiles of 128: 24 of 148 SMs at M = 256)",
                        "peak_source": src},
           "clocks": clk}
    del g, outs, layers
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- cfg3: packed MoE
def bench_cfg3(args, job: Job, peaks: dict) -> dict:
    """256 int2 experts (top-8) + int4 shared expert, T=2048 tokens per rank. N ranks:
    experts split contiguously, each rank routes its own tokens and exchanges rows with NCCL all_to_all
    (weak scaling). value = tokens/s over all ranks."""
    from onecomp_runtime.moe import ExpertParallelMoE, PackedMoE
    from onecomp_runtime.testing import CFG3, dsv4_packed
    dev, world, rank = job.dev, job.world, job.rank
    E, k, H, F, T = CFG3["E"], CFG3["k"], CFG3["H"], CFG3["F"], CFG3["T"]
    E = args.moe_experts or E  # profiling only: a smaller case with the same rows per expert
    T = args.moe_tokens or T
    el = E // world
    wb, gs = CFG3["expert_wbits"], CFG3["expert_gs"]
    experts = [{"gate": dsv4_packed(F, H, wb, gs, seed=3 * e, device=dev),
                "up": dsv4_packed(F, H, wb, gs, seed=3 * e + 1, device=dev),
                "down": dsv4_packed(H, F, wb, gs, seed=3 * e + 2, device=dev)} for e in range(rank * el, (rank + 1) * el)]
    sw, sgs = CFG3["shared_wbits"], CFG3["shared_gs"]
    shared = {"gate": dsv4_packed(F, H, sw, sgs, seed=9000, zero=None, scales_range=(0.002, 0.02), device=dev),
              "up": dsv4_packed(F, H, sw, sgs, seed=9001, zero=None, scales_range=(0.002, 0.02), device=dev),
              "down": dsv4_packed(H, F, sw, sgs, seed=9002, zero=None, scales_range=(0.002, 0.02), device=dev)}
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g, device=dev)
    timer = LaunchTimer()
    moe = PackedMoE(experts, shared, k=k, device=dev, fuse_gate_up=False if args.moe_no_fuse else "shared")
    for h in list(moe._h.values()) + list((moe._shared or {}).values()):
        timer.wrap_rows(h)
    if world == 1:
        fn = lambda: moe(x, logits)  # noqa: E731
    else:
        ep = ExpertParallelMoE(E, k, moe.expert_ffn, route=moe.route, shared=moe.shared_ffn, combine=moe.combine,
                               permute=moe.permute, gather=moe.gather)
        fn = lambda: ep(x, logits)  # noqa: E731
    with torch.no_grad():
        ms, clk = timed_steps(job, fn, args.steps, args.warmup, before=timer.start)
        gemm_ms, gemm_flops = timer.stop()
    flops = 2 * T * k * 3 * H * F + 2 * T * 3 * H * F
    # packed bytes a rank must read once per layer: its experts' int2 codes + fp16 scales and zeros, the
    # shared expert's int4 codes + scales/zeros, activations in and out
    G_e = (H + gs - 1) // gs
    exp_bytes = el * (2 * F * H * wb // 8 + H * F * wb // 8 + 2 * (2 * F * G_e + 2 * H * ((F + gs - 1) // gs)) * 2)
    sh_bytes = 3 * F * H * sw // 8 + 2 * 2 * (2 * F * ((H + sgs - 1) // sgs) + H * ((F + sgs - 1) // sgs))
    act_bytes = 2 * T * H * 2
    nbytes = exp_bytes + sh_bytes + act_bytes
    gbs = nbytes / (ms / 1e3) / 1e9
    rt = roofline_tensor(gemm_ms, gemm_flops, peaks, clk, None,
                         "rows_gemm_tc_kernel (tcgen05, grouped over experts, int2 table decode)", ms * args.steps,
                         args.steps)
    rt["layer_tflops"] = round(flops / (ms / 1e3) / 1e12, 1)
    rt["layer_frac_tensor"] = round(rt["layer_tflops"] / rt["peak"], 4)
    rt["hbm"] = {"achieved_GBs": round(gbs, 1), "peak": peaks["hbm_gbs"], "frac": round(gbs / peaks["hbm_gbs"], 4),
                 "bytes_per_layer": nbytes}
    out = {"metric": "packed-MoE layer tokens/s (256 int2 experts top-8 + int4 shared)",
           "value": round(world * T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
           "config": {"workload": "cfg3", "tokens_per_gpu": T, "experts_per_gpu": el,
                      "parallelism": f"expert parallel x{world} (NCCL all_to_all)" if world > 1 else "1 GPU",
                      "gate_up": {"routed": "one SwiGLU launch" if "gate_up" in moe._h else "two GEMMs + silu-mul",
                                  "shared": "one SwiGLU launch" if "gate_up" in (moe._shared or {}) else
                                            "two GEMMs + silu-mul"},
                      "l2_flush": "none needed: 2 GB of packed experts per layer > 126 MB L2"},
           "roofline": rt, "clocks": clk}
    del moe, experts, shared
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- reference arm
def reference_arm(args, job: Job):
    """The reference's CPU eager path (oracle port) on the host cores, rank 0 only."""
    if job.rank != 0:
        return
    if args.workload == "cfg1":
        from onecomp_runtime.testing import CFG1, CFG1_LAYERS
        m, blocks, layers, gs, tokens, seed = args.cpu_sample_m, CFG1["blocks"], CFG1_LAYERS, CFG1["gs"], CFG1["M"], 1000
        metric, cfg = METRIC_CFG1, {"workload": "cfg1", "tokens_per_gpu": tokens, "blocks": blocks}
    else:
        from onecomp_runtime.testing import CFG4, CFG4_LAYERS
        m, blocks, layers, gs, tokens, seed = args.cpu_sample_m, CFG4["blocks"], CFG4_LAYERS, CFG4["gs"], CFG4["M"], 4000
        metric, cfg = METRIC, {"workload": "cfg4: video-DiT int4 stack, 12 blocks, hidden 4096, GPTQ v1 gs32, "
                                           "M=32768 tokens", "tokens": tokens, "blocks": blocks}
    run, cores = cpu_eager_block(layers, gs, m, seed)
    per_block = time_cpu(run, args.warmup, args.steps)
    tps = m / (per_block * blocks)
    sample = (f"one block (4 linears + glue) at M={m} tokens per step, torch CPU bf16 F.linear on weights "
              f"dequantized once by the oracle's formula; value = M / (block time x {blocks} blocks); "
              f"ms_per_step is the measured block time")
    line = {"metric": metric, "impl": "reference", "value": round(tps, 1), "unit": "tokens/s",
            "n_gpus": job.world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per_block * 1e3, 3), "higher_is_better": True,
            "scaling": "strong" if args.workload != "cfg1" else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": round(tps, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(tps, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg4", choices=["cfg1", "cfg2", "cfg3", "cfg4"],
                    help="cfg4: tensor-parallel video-DiT stack (default, headline); cfg1: FLUX-style stack; "
                         "cfg2: decode GEMV layer set; cfg3: packed MoE layer (expert parallel)")
    ap.add_argument("--no-nested", action="store_true", help="cfg4 line only (skip the cfg1/cfg2/cfg3 blocks)")
    ap.add_argument("--tc-tile", type=int, default=0, help="tokens per tcgen05 tile (0 = library default)")
    ap.add_argument("--gemv-ctas", type=int, default=0, help="GEMV split-K target CTAs per SM (0 = default)")
    ap.add_argument("--wbits", type=int, default=4, choices=[4, 8], help="cfg2 only: code width of the layer set")
    ap.add_argument("--gemv-impl", type=int, default=-1, choices=[-1, 0, 1, 2, 3, 4],
                    help="cfg2: decode kernel (OC_OPT_GEMV_IMPL; -1 = library default, the integer-MMA GEMV)")
    ap.add_argument("--gemv-prep", type=int, default=-1, choices=[-1, 0, 1],
                    help="cfg2: OC_OPT_GEMV_PREP (-1 = library default: the integer GEMV prepares its activations "
                         "in each CTA at M <= 2)")
    ap.add_argument("--blocks", type=int, default=0, help="override the number of DiT blocks (profiling only)")
    ap.add_argument("--moe-experts", type=int, default=0, help="cfg3: override the expert count (profiling only)")
    ap.add_argument("--moe-tokens", type=int, default=0, help="cfg3: override tokens per GPU (profiling only)")
    ap.add_argument("--moe-no-fuse", action="store_true",
                    help="cfg3: the shared expert's gate and up as two GEMMs + the silu-mul kernel too (comparison)")
    ap.add_argument("--cpu-sample-m", type=int, default=512, help="tokens of the bounded CPU sample (one block)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp-chunks", type=int, default=0,
                    help="cfg4: row chunks of the pipelined stack (0 = 1 on one GPU, 3 on several)")
    ap.add_argument("--tp-reduce", default="auto", choices=["auto", "nvls", "nccl"],
                    help="cfg4 with N > 1: all-reduce of the row-parallel outputs (own NVLS kernel, with the RMS "
                         "norm fused, or NCCL; auto = NVLS, which measured faster from 2 ranks)")
    ap.add_argument("--nvls-blocks", type=int, default=8, help="cfg4 NVLS all-reduce: CTAs per reduction (1..64)")
    ap.add_argument("--no-fused-norm", action="store_true",
                    help="cfg4 with NVLS: run the RMS norms after the all-reduces instead of inside them")
    ap.add_argument("--tc-max-ctas", type=int, default=-1,
                    help="cfg4 with N > 1: CTAs of the persistent GEMMs (0 = one per SM; -1 = SMs minus the NVLS "
                         "reduction's blocks when it runs, else one per SM)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    job = Job()
    if args.impl == "reference":
        return reference_arm(args, job)
    job.init_gpu()
    peaks = load_peaks()
    with_cpu = job.rank == 0 and job.world == 1 and not args.no_cpu_baseline
    try:
        if args.workload == "cfg4":
            line = bench_cfg4(args, job, peaks, with_cpu)
            if not args.no_nested:
                line["workloads"] = {"cfg0": bench_cfg0(args, job, peaks),
                                     "cfg1": bench_cfg1(args, job, peaks, full_line=False),
                                     "cfg2": bench_cfg2(args, job, peaks),
                                     "cfg3": bench_cfg3(args, job, peaks)}
        elif args.workload == "cfg1":
            line = bench_cfg1(args, job, peaks, full_line=True)
        elif args.workload == "cfg2":
            line = bench_cfg2(args, job, peaks)
        else:
            line = bench_cfg3(args, job, peaks)
    finally:
        job.close()
    if job.rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
