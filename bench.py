"""Benchmark of the int4 linear hot path on B200 (one JSON line on rank 0).

Default workload: a FLUX-style DiT block stack --
8 blocks of qkv 3072->9216, proj 3072->3072, fc1 3072->9216, fc2 9216->3072,
AutoGPTQ v1 int4, groupsize 32, bf16 activations N(0,1), M = 4608 tokens
(4096 image + 512 text). Random-init packed weights (seeded), synthetic
activations. Glue between linears (q slice of qkv as the attention stand-in,
residual adds, RMS norm, tanh-GELU) runs in torch and is timed with the step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload cfg1|cfg0|cfg2]

* ``value``: whole-job tokens/s (N ranks each run their own 4608-token batch:
  weak scaling, no data-path collective), device-timed with CUDA events,
  max over ranks. Inputs and weights are resident in HBM; the stack's weights
  (437 MB packed) exceed the 126 MB L2, so every step streams them from HBM.
* ``e2e``: the same step through the public module API with the input copied
  from pinned host memory and the output read back every step.
* ``roofline``: the tcgen05 GEMM launches, timed individually with CUDA events
  inside the timed steps: achieved = 2*M*K*N summed / their summed duration,
  against the measured sustained bf16 peak (MEASURED_PEAKS.json).
* ``cpu_baseline`` (rank 0, N=1): the reference CPU eager path (dequantize once,
  torch CPU bf16 ``F.linear``) restated in ``oracle/``, on a bounded sample
  (one block, extrapolated to the stack).
* ``--impl reference``: the same CPU eager path as the reference arm.
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

METRIC = "DiT-stack tokens/s (int4 GPTQ linear stack)"



# DRAM traffic measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum) for the dominant
# kernel of each workload; the commands and per-launch figures are in profiles/.
TC_TRAFFIC_BYTES_PER_LAUNCH = 103_200_000    # cfg1: mean of qkv, proj, fc1, fc2 launches
GEMV_TRAFFIC_BYTES_PER_LAUNCH = 21_852_160   # cfg2: q/k/v layer, M = 1 (algorithmic 21.8 MB)

def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d.get("hbm_gbs"), "bf16": d.get("bf16_tflops"),
                "bf16_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


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


# ----------------------------------------------------------------------------- model
def rms_norm(h: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMS norm without weight, fp32 statistics (torch's fused rms_norm)."""
    return torch.nn.functional.rms_norm(h, (h.shape[-1],), eps=eps)


class DiTStack:
    """8 FLUX-style blocks of FusedInt4Linear layers (random packed weights)."""

    def __init__(self, device, blocks: int, layers, gs: int, seed: int = 1000):
        from onecomp_runtime.layers import FusedInt4Linear
        from onecomp_runtime.testing import gptq_layer
        self.blocks = []
        for b in range(blocks):
            blk = {}
            for li, (name, K, N) in enumerate(layers):
                t = gptq_layer(K, N, gs, seed=seed * (b + 1) + li, device=device)
                blk[name] = FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t["bias"], gs)
            self.blocks.append(blk)
        self.hidden = layers[0][1]
        self.gemm_events: list | None = None

    def _lin(self, layer, x, residual=None, activation=None):
        if self.gemm_events is None:
            return layer.forward_fused(x, residual=residual, activation=activation)
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        y = layer.forward_fused(x, residual=residual, activation=activation)
        e.record()
        self.gemm_events.append((s, e, 2 * x.shape[0] * layer.in_features * layer.out_features))
        return y

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """Per block: q = qkv(h)[:, :H]; h = rms(h + proj(q)); h = rms(h + fc2(gelu(fc1(h)))).

        The residual adds and the tanh-GELU run in the GEMM epilogues (forward_fused)."""
        H = self.hidden
        for blk in self.blocks:
            qkv = self._lin(blk["qkv"], h)
            q = qkv[:, :H]                       # attention stand-in: the q slice
            h = rms_norm(self._lin(blk["proj"], q, residual=h))
            f = self._lin(blk["fc1"], h, activation="gelu_tanh")
            h = rms_norm(self._lin(blk["fc2"], f, residual=h))
        return h

    def gemm_count_per_step(self) -> int:
        return 4 * len(self.blocks)


# ----------------------------------------------------------------------------- CPU eager
def cpu_eager_block(layers, gs: int, M: int, seed: int = 1000):
    """The reference CPU eager path (oracle restatement) for one block.

    Weights are dequantized once by the oracle (as ``backend.build_eager``
    does at load time, not timed); each call runs the block's four
    ``F.linear`` in bf16 on the host cores plus the glue. Returns
    ``(run, threads)``.
    """
    from oracle import gptq
    from oracle.eager import EagerCPU
    from onecomp_runtime.testing import gptq_layer
    torch.set_num_threads(os.cpu_count() or 1)
    mods = {}
    for li, (name, K, N) in enumerate(layers):
        t = gptq_layer(K, N, gs, seed=seed + li)
        s_bits = t["scales"].view(torch.int16).numpy().view(np.uint16)
        w = gptq.dequant_gptq(t["qweight"].numpy(), s_bits, "f16", t["qzeros"].numpy(), t["g_idx"].numpy(), K, N,
                              "bf16")
        b_bits = t["bias"].view(torch.int16).numpy().view(np.uint16)
        mods[name] = EagerCPU(w, "bf16", b_bits, "f16")
    H = layers[0][1]
    x = torch.randn(M, H, dtype=torch.float32).to(torch.bfloat16)

    def run():
        qkv = mods["qkv"](x)
        h = rms_norm(x + mods["proj"](qkv[:, :H].contiguous()))
        f = torch.nn.functional.gelu(mods["fc1"](h), approximate="tanh")
        return rms_norm(h + mods["fc2"](f))

    return run, torch.get_num_threads()


def time_cpu(run, warmup: int, steps: int) -> float:
    for _ in range(warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(steps):
        run()
    return (time.perf_counter() - t0) / steps


# ----------------------------------------------------------------------------- decode (cfg2)
def bench_decode(args):
    """gptq_v2 gs128 act-order layer set (fp16 scales, bf16 activations),
    M in {1, 4, 16}, CUDA-graph replayed. ``--wbits 8``: the same shapes as 8-bit gs128 layers
    without act-order and with bf16 scales (the model dtype), as the Qwen3.6 adapter builds them.

    Reported value: packed bytes streamed per second (qweight + scales + qzeros
    + g_idx of the 5 layers, + activations) at the largest M; every M in ``per_m``.
    """
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import PackedGPTQLinear
    from onecomp_runtime.testing import CFG2_LAYERS, gptq_layer
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    _lib.require_b200(dev)
    if args.gemv_ctas:
        _lib.set_option(_lib.OPT_GEMV_CTAS, args.gemv_ctas)
    layers, nbytes = [], 0
    w8 = args.wbits == 8
    for i, (name, K, N) in enumerate(CFG2_LAYERS):
        G = (K + 127) // 128
        if w8:  # the 8-bit layers of a {4,8}-bit GPTQ checkpoint: v1 zeros, gs128, no act-order
            t = gptq_layer(K, N, 128, seed=2000 + i, v1=True, scales_range=(0.001, 0.01),
                           scales_dtype=torch.bfloat16, bias=False, device=dev, wbits=8)
            layers.append(PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], None, 128, 8,
                                           True))
            nbytes += K * N + 2 * G * N + G * N
        else:
            t = gptq_layer(K, N, 128, seed=2000 + i, v1=False, actorder=True, scales_range=(0.001, 0.01),
                           scales_dtype=torch.float16, bias=False, device=dev)  # config 2: fp16 scales
            layers.append(PackedGPTQLinear(K, N, t["qweight"], t["scales"], t["qzeros"], t["g_idx"], None, 128, 4,
                                           False))
            nbytes += K * N // 2 + 2 * G * N + G * N // 2 + 4 * K
    peaks = load_peaks()
    per_m = {}
    for M in (1, 4, 16):
        xs = [torch.randn(M, K, device=dev).to(torch.bfloat16) for _, K, _ in CFG2_LAYERS]
        act = sum(2 * M * K + 2 * M * N for _, K, N in CFG2_LAYERS)
        for _ in range(3):
            [l(x) for l, x in zip(layers, xs)]
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = [l(x) for l, x in zip(layers, xs)]
        for _ in range(args.warmup):
            g.replay()
        # time each replay (the set is ~30 us; 200 replays stream 35 GB of weights > L2)
        reps = max(args.steps, 1) * 20
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s0.record()
        for _ in range(reps):
            g.replay()
        s1.record()
        torch.cuda.synchronize()
        us = s0.elapsed_time(s1) * 1e3 / reps
        per_m[M] = {"us_per_set": round(us, 2), "GB_s": round((nbytes + act) / (us * 1e-6) / 1e9, 1),
                    "frac_hbm": round((nbytes + act) / (us * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)}
        del g, outs
    top = per_m[16]
    kind = "gptq v1 gs128 8-bit" if w8 else "gptq_v2 gs128 act-order"
    line = {"metric": f"decode GB/s ({kind} layer set, M=16)", "value": top["GB_s"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg2: q/k/v 5120->8192, o 6144->5120, gate/up 5120->17408, down 17408->5120"
                                   + (", 8-bit codes" if w8 else ""),
                       "packed_bytes_per_set": nbytes, "graph": "CUDA graph of the 5 layers, replayed"},
            "per_m": per_m,
            "roofline": {"bound": "hbm", "achieved": top["GB_s"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": top["frac_hbm"], "traffic": None if w8 else GEMV_TRAFFIC_BYTES_PER_LAUNCH,
                         "traffic_unit": "bytes per launch (q/k/v layer)",
                         "peak_source": f"{peaks['source']} hbm_gbs"}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- MoE (cfg3)
def _dist_init(dev):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not torch.distributed.is_initialized():
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    return world, int(os.environ.get("RANK", "0"))


def _timed(fn, steps, warmup, dev, world):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(steps):
        fn()
    s1.record()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ms = torch.tensor([s0.elapsed_time(s1) / steps], device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    return float(ms[0])


def bench_moe(args):
    """256 int2 experts (top-8) + int4 shared expert, T=2048 tokens per rank.

    N ranks: experts split contiguously, each rank routes its own 2048 tokens and exchanges
    rows with NCCL all_to_all (weak scaling). value = tokens/s over all ranks.
    """
    from onecomp_runtime import _lib
    from onecomp_runtime.moe import ExpertParallelMoE, PackedMoE
    from onecomp_runtime.testing import CFG3, dsv4_packed
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    world, rank = _dist_init(dev)
    _lib.require_b200(dev)
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
    if world == 1:
        moe = PackedMoE(experts, shared, k=k, device=dev)
        fn = lambda: moe(x, logits)  # noqa: E731
    else:
        loc = PackedMoE(experts, shared, k=k, device=dev)
        ep = ExpertParallelMoE(E, k, loc.expert_ffn, route=loc.route,
                               shared=loc.shared_ffn, combine=loc.combine)
        fn = lambda: ep(x, logits)  # noqa: E731
    with torch.no_grad():
        ms = _timed(fn, args.steps, args.warmup, dev, world)
    flops = 2 * T * k * 3 * H * F + 2 * T * 3 * H * F
    line = {"metric": "packed-MoE layer tokens/s (256 int2 experts top-8 + int4 shared)",
            "value": round(world * T / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg3", "tokens_per_gpu": T, "experts_per_gpu": el,
                       "parallelism": f"expert parallel x{world} (NCCL all_to_all)" if world > 1 else "1 GPU"},
            "tflops_per_gpu": round(flops / (ms / 1e3) / 1e12, 1)}
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- TP stack (cfg4)
def bench_tp(args):
    """12 video-DiT blocks (hidden 4096), M=32768 tokens, column/row tensor parallel.

    Strong scaling: the same 32768 tokens on every N; row-parallel outputs are summed with a
    chunked NCCL all-reduce that overlaps the next chunk's GEMM.
    """
    from onecomp_runtime import _lib
    from onecomp_runtime.layers import FusedInt4Linear
    from onecomp_runtime.tensor_parallel import build_tp_block
    from onecomp_runtime.testing import CFG4, CFG4_LAYERS, gptq_layer
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    world, rank = _dist_init(dev)
    _lib.require_b200(dev)
    blocks = args.blocks or CFG4["blocks"]
    M, gs, H = CFG4["M"], CFG4["gs"], CFG4["hidden"]

    def make(t, K, N):
        return FusedInt4Linear(K, N, t["qweight"], t["scales"], t["qzeros"], t.get("bias"), gs)

    stack = []
    for b in range(blocks):
        tens = {name: gptq_layer(K, N, gs, seed=4000 + 10 * b + i, device=dev)
                for i, (name, K, N) in enumerate(CFG4_LAYERS)}
        stack.append(build_tp_block(tens, CFG4_LAYERS, rank, world, gs, make))
        del tens
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn((M, H), generator=g, device=dev).to(torch.bfloat16)
    hq = H // world

    def step():
        h = x
        for blk in stack:
            qkv = blk["qkv"](h)
            h = rms_norm(h + blk["out"](qkv[:, :hq]))
            f = torch.nn.functional.gelu(blk["fc1"](h), approximate="tanh")
            h = rms_norm(h + blk["fc2"](f))
        return h

    with torch.no_grad():
        ms = _timed(step, args.steps, args.warmup, dev, world)
    flops = blocks * sum(2 * M * K * N for _, K, N in CFG4_LAYERS)
    line = {"metric": "TP video-DiT stack tokens/s (12 blocks, hidden 4096, int4 GPTQ gs32)",
            "value": round(M / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "cfg4", "tokens": M, "blocks": blocks,
                       "parallelism": f"tensor parallel x{world} (column/row, NCCL all-reduce)"},
            "tflops_total": round(flops / (ms / 1e3) / 1e12, 1)}
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="cfg1", choices=["cfg1", "cfg2", "cfg3", "cfg4"],
                    help="cfg1: DiT stack (default, headline); cfg2: decode GEMV layer set; "
                         "cfg3: packed MoE layer (expert parallel); cfg4: tensor-parallel video-DiT stack")
    ap.add_argument("--tc-tile", type=int, default=0, help="tokens per tcgen05 tile (0 = library default)")
    ap.add_argument("--gemv-ctas", type=int, default=0, help="GEMV split-K target CTAs per SM (0 = default)")
    ap.add_argument("--wbits", type=int, default=4, choices=[4, 8], help="cfg2 only: code width of the layer set")
    ap.add_argument("--blocks", type=int, default=0, help="override the number of DiT blocks (profiling only)")
    ap.add_argument("--moe-experts", type=int, default=0, help="cfg3: override the expert count (profiling only)")
    ap.add_argument("--moe-tokens", type=int, default=0, help="cfg3: override tokens per GPU (profiling only)")
    ap.add_argument("--cpu-sample-m", type=int, default=1152,
                    help="tokens of the bounded CPU-baseline sample (one block)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.workload == "cfg2":
        return bench_decode(args)
    if args.workload == "cfg3":
        return bench_moe(args)
    if args.workload == "cfg4":
        return bench_tp(args)
    from onecomp_runtime.testing import CFG1, CFG1_LAYERS
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    M, blocks, gs = CFG1["M"], (args.blocks or CFG1["blocks"]), CFG1["gs"]
    config = {"workload": "cfg1: FLUX-style DiT int4 stack, 8 blocks x (qkv 3072->9216, proj 3072->3072, "
                          "fc1 3072->9216, fc2 9216->3072), GPTQ v1 gs32, M=4608 tokens per GPU",
              "global_batch_tokens": M * world, "tokens_per_gpu": M, "blocks": blocks,
              "l2_flush": "none needed: inputs larger than L2",
              "parallelism": f"replicas x{world} (weak scaling, no collective)",
              "l2": "weights 437 MB packed per stack > 126 MB L2 (streamed every step)"}

    if args.impl == "reference":
        if rank != 0:
            return
        sample_m = args.cpu_sample_m
        run, cores = cpu_eager_block(CFG1_LAYERS, gs, sample_m)
        per_block = time_cpu(run, args.warmup, args.steps)
        tps = sample_m / (per_block * blocks)
        sample = (f"one block (4 linears + glue) at M={sample_m} tokens per step, torch CPU bf16 F.linear on "
                  "weights dequantized once by the oracle, extrapolated x8 blocks")
        line = {"metric": METRIC, "impl": "reference", "value": round(tps, 1), "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1e3 * M / tps, 3), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
                "cpu_baseline": {"value": round(tps, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(tps, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    from onecomp_runtime import _lib
    _lib.require_b200(dev)
    if args.tc_tile:
        _lib.set_option(_lib.OPT_TC_TILE, args.tc_tile)
        config["tc_tile"] = args.tc_tile
    torch.manual_seed(1234 + rank)
    stack = DiTStack(dev, blocks, CFG1_LAYERS, gs, seed=1000 + 17 * rank)
    x = torch.randn(M, CFG1["hidden"], device=dev).to(torch.bfloat16)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    with torch.no_grad():
        for _ in range(args.warmup):
            y = stack.forward(x)
        torch.cuda.synchronize(dev)
        if not torch.isfinite(y).all():
            raise RuntimeError("non-finite stack output")

        # ---- device-timed steps (inputs resident in HBM)
        clocks = ClockSampler(local)
        barrier()
        clocks.start()
        stack.gemm_events = []
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record()
        for _ in range(args.steps):
            y = stack.forward(x)
        t_end.record()
        barrier()
        clk = clocks.stop()
        ms_total = t_start.elapsed_time(t_end)
        gemm = [(s.elapsed_time(e), fl) for s, e, fl in stack.gemm_events]
        stack.gemm_events = None

        # ---- end-to-end through the module API with host buffers: every step copies its input
        # from pinned host memory and reads its result back; the copies of step i+1 / i-1 run on
        # their own streams while step i computes (double-buffered device and host tensors)
        shape = (M, CFG1["hidden"])
        x_host = [torch.empty(shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
        y_host = [torch.empty(shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
        for b in range(2):
            x_host[b].copy_(x.cpu())
        x_dev = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        main = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]
        out_ready = [torch.cuda.Event() for _ in range(2)]

        def e2e_steps(n):
            for i in range(n):
                b = i & 1
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(in_free[b])
                    x_dev[b].copy_(x_host[b], non_blocking=True)
                    in_ready[b].record(s_in)
                main.wait_event(in_ready[b])
                y = stack.forward(x_dev[b])
                in_free[b].record(main)
                out_ready[b].record(main)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(out_ready[b])
                    y_host[b].copy_(y, non_blocking=True)
                    y.record_stream(s_out)
            main.wait_stream(s_in)
            main.wait_stream(s_out)

        e2e_steps(2)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(main)
        e2e_steps(args.steps)
        e1.record(main)
        barrier()
        ms_e2e = e0.elapsed_time(e1)
        if not torch.equal(y_host[(args.steps - 1) & 1], y.cpu()):
            raise RuntimeError("end-to-end output differs from the device-timed output")

    t = torch.tensor([ms_total, ms_e2e], device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    ms_total, ms_e2e = float(t[0]), float(t[1])
    ms_step = ms_total / args.steps
    value = world * M * args.steps / (ms_total / 1e3)
    e2e_value = world * M * args.steps / (ms_e2e / 1e3)

    peaks = load_peaks()
    gemm_ms = sum(g[0] for g in gemm)
    gemm_flops = sum(g[1] for g in gemm)
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
    peak = peaks["bf16_sustained"]
    roofline = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                # DRAM read + write bytes per launch, mean over one block's four GEMM launches, from
                # one ncu capture of this workload (profiles/gptq_gemm_tc_cfg1.txt)
                "traffic": TC_TRAFFIC_BYTES_PER_LAUNCH if args.blocks == 0 else None,
                "traffic_unit": "bytes per launch",
                "kernel": "gptq_gemm_tc_kernel (tcgen05, 384-token tiles = 2 x 192 chosen by the library at M=4608)",
                "peak_source": f"{peaks['source']} bf16_tflops_sustained",
                "gemm_share_of_step": round(gemm_ms / ms_total, 4),
                "gemm_ms_per_step": round(gemm_ms / args.steps, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        run, cores = cpu_eager_block(CFG1_LAYERS, gs, args.cpu_sample_m)
        per_block = time_cpu(run, 1, 3)
        cpu = {"value": round(args.cpu_sample_m / (per_block * blocks), 1), "unit": "tokens/s", "cores": cores,
               "kind": "port",
               "sample": f"one block (4 linears + glue) at M={args.cpu_sample_m} tokens, torch CPU bf16 "
                         "F.linear on oracle-dequantized weights, extrapolated x8 blocks"}

    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random packed weights, N(0,1) activations)", "config": config,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": M * CFG1["hidden"] * 2,
                    "d2h_bytes_per_step": M * CFG1["hidden"] * 2},
            "gpu_launches": stack.gemm_count_per_step() * args.steps,
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clk}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
