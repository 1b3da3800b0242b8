"""Seeded synthetic packed layers for tests and benchmarks (like ``torch.testing``).

Generates AutoGPTQ / RTN / DSV4 tensors with the shapes and value
distributions of the benchmark configurations (there are no real checkpoints
to download): uniform 4-bit codes, zero points stored v1-shifted (``zero - 1``)
or unshifted (v2), uniform fp16 scales, N(0, 0.02^2) fp16 bias.
"""
from __future__ import annotations

import torch


def _to_int32(words: torch.Tensor) -> torch.Tensor:
    """int64 words in [0, 2^32) -> int32 with the same bit pattern."""
    return ((words + 2**31) % 2**32 - 2**31).to(torch.int32)


def pack_along_n(zeros_gn: torch.Tensor, wbits: int = 4) -> torch.Tensor:
    """int [G, N] -> qzeros int32 [G, N / (32/wbits)] (value j of a word = column pf*c + j)."""
    pf = 32 // wbits
    z = zeros_gn.to(torch.int64) & ((1 << wbits) - 1)
    acc = torch.zeros((z.shape[0], z.shape[1] // pf), dtype=torch.int64, device=z.device)
    for j in range(pf):
        acc |= z[:, j::pf] << (wbits * j)
    return _to_int32(acc)


def pack_along_k(codes_nk: torch.Tensor, wbits: int = 4) -> torch.Tensor:
    """int [N, K] -> qweight int32 [K / (32/wbits), N] (value i of a word = row pf*r + i)."""
    pf = 32 // wbits
    rows = codes_nk.t().to(torch.int64) & ((1 << wbits) - 1)
    acc = torch.zeros((rows.shape[0] // pf, rows.shape[1]), dtype=torch.int64, device=rows.device)
    for i in range(pf):
        acc |= rows[i::pf] << (wbits * i)
    return _to_int32(acc)


def gptq_layer(K: int, N: int, groupsize: int, *, seed: int = 0, v1: bool = True, actorder: bool = False,
               scales_range=(0.002, 0.02), bias: bool = True, device="cpu",
               scales_dtype=torch.float16, wbits: int = 4) -> dict:
    """Random AutoGPTQ layer (4- or 8-bit codes): ``qweight, qzeros, scales, g_idx, bias``."""
    gen_dev = torch.device(device)
    g = torch.Generator(device=gen_dev).manual_seed(int(seed))
    G = (K + groupsize - 1) // groupsize
    qmax = (1 << wbits) - 1
    qweight = torch.randint(-2**31, 2**31, (K * wbits // 32, N), generator=g, device=gen_dev, dtype=torch.int64)
    qweight = qweight.to(torch.int32)
    zero = torch.randint(1, qmax + 1, (G, N), generator=g, device=gen_dev)
    stored = (zero - 1) & qmax if v1 else zero
    qzeros = pack_along_n(stored, wbits)
    lo, hi = scales_range
    scales = (torch.rand((G, N), generator=g, device=gen_dev) * (hi - lo) + lo).to(scales_dtype)
    if actorder:
        perm = torch.randperm(K, generator=g, device=gen_dev)
        g_idx = (torch.arange(K, device=gen_dev) // groupsize)[perm].to(torch.long)
    else:
        g_idx = (torch.arange(K, device=gen_dev) // groupsize).to(torch.long)
    out = {"qweight": qweight, "qzeros": qzeros, "scales": scales, "g_idx": g_idx}
    if bias:
        out["bias"] = (torch.randn(N, generator=g, device=gen_dev) * 0.02).to(torch.float16)
    return out


def activations(M: int, K: int, *, seed: int = 0, dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=torch.device(device)).manual_seed(int(seed))
    return torch.randn((M, K), generator=g, device=device).to(dtype)


# --------------------------------------------------------------------- benchmark configs
CFG0 = dict(K=3072, N=3072, gs=32, M=256)

# FLUX-style DiT block: hidden 3072; qkv 3072->9216, proj, MLP 3072->9216->3072; M = 4096 + 512 tokens
CFG1_LAYERS = (("qkv", 3072, 9216), ("proj", 3072, 3072), ("fc1", 3072, 9216), ("fc2", 9216, 3072))
CFG1 = dict(hidden=3072, blocks=8, M=4608, gs=32)

# dense LLM decode set, gptq_v2, gs=128, act-order
CFG2_LAYERS = (("qkv", 5120, 8192), ("o", 6144, 5120), ("gate", 5120, 17408), ("up", 5120, 17408),
               ("down", 17408, 5120))
CFG2 = dict(gs=128, M=(1, 4, 16), scales_range=(0.001, 0.01))

# video-DiT tensor-parallel stack: hidden 4096; qkv 4096->12288, out 4096->4096, FFN 4096->16384->4096
CFG4_LAYERS = (("qkv", 4096, 12288), ("out", 4096, 4096), ("fc1", 4096, 16384), ("fc2", 16384, 4096))
CFG4 = dict(hidden=4096, blocks=12, M=32768, gs=32)


def entry(name: str, K: int, N: int, groupsize: int, actorder: bool = False, wbits: int = 4) -> dict:
    """A ``quant_layers_json`` manifest entry (diffusion.py contract)."""
    return {"name": name, "wbits": wbits, "groupsize": groupsize, "actorder": actorder,
            "in_features": K, "out_features": N}


# packed MoE layer: 256 experts, top-8, hidden 4096, FFN 2048; int2 DSV4 experts gs64, zeros 1.5;
# shared expert int4 gs128; T = 2048 tokens
CFG3 = dict(E=256, k=8, H=4096, F=2048, T=2048, expert_wbits=2, expert_gs=64, shared_wbits=4, shared_gs=128)


def dsv4_packed(out_f: int, in_f: int, wbits: int, groupsize: int, *, seed: int = 0, zero: float | None = 1.5,
                scales_range=(0.005, 0.05), device="cpu") -> dict:
    """Random DSV4 byte-packed layer dict (``qweight_packed``, ``scales``, ``qzeros`` [out, G] fp16)."""
    g = torch.Generator(device=torch.device(device)).manual_seed(int(seed))
    per = 8 // wbits
    ncol = (in_f + per - 1) // per
    packed = torch.randint(0, 256, (out_f, ncol), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    G = (in_f + groupsize - 1) // groupsize if groupsize > 0 else 1
    lo, hi = scales_range
    scales = (torch.rand((out_f, G), generator=g, device=device) * (hi - lo) + lo).to(torch.float16)
    if zero is None:
        zeros = (torch.rand((out_f, G), generator=g, device=device) * ((1 << wbits) - 1)).to(torch.float16)
    else:
        zeros = torch.full((out_f, G), zero, dtype=torch.float16, device=device)
    return {"qweight_packed": packed, "scales": scales, "qzeros": zeros, "wbits": wbits, "groupsize": groupsize,
            "in_features": in_f}


# --------------------------------------------------------------------- packed checkpoints
class TinyBlock(torch.nn.Module):
    """A DiT-style block (pre-norm attention-shaped and MLP linears) for loader tests."""

    def __init__(self, hidden: int, mlp: int) -> None:
        super().__init__()
        self.norm1 = torch.nn.LayerNorm(hidden)
        self.qkv = torch.nn.Linear(hidden, 3 * hidden)
        self.proj = torch.nn.Linear(hidden, hidden)
        self.norm2 = torch.nn.LayerNorm(hidden)
        self.fc1 = torch.nn.Linear(hidden, mlp)
        self.fc2 = torch.nn.Linear(mlp, hidden)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.qkv(self.norm1(x))
        x = x + self.proj(h[..., : x.shape[-1]])
        return x + self.fc2(torch.nn.functional.gelu(self.fc1(self.norm2(x)), approximate="tanh"))


class TinyDiT(torch.nn.Module):
    def __init__(self, cfg: dict) -> None:
        super().__init__()
        self.embed = torch.nn.Linear(cfg["in_channels"], cfg["hidden"])
        self.blocks = torch.nn.ModuleList(TinyBlock(cfg["hidden"], cfg["mlp"]) for _ in range(cfg["blocks"]))
        self.out = torch.nn.Linear(cfg["hidden"], cfg["in_channels"])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.embed(x)
        for b in self.blocks:
            h = b(h)
        return self.out(h)


def write_int4_checkpoint(path, cfg: dict, *, groupsize: int = 32, seed: int = 0, v1: bool = True,
                          actorder: bool = False, extra: dict | None = None) -> list[dict]:
    """Write a OneCompression packed checkpoint of ``TinyDiT(cfg)``: every block Linear as a
    random AutoGPTQ int4 layer (``qweight, scales, qzeros, g_idx, bias``), the rest as bf16
    tensors, with the ``config_json`` / ``quant_layers_json`` / ``checkpoint_format`` metadata
    the loader reads. ``extra`` adds tensors. Returns the quant-layer entries."""
    import json

    from safetensors.torch import save_file

    torch.manual_seed(seed)
    model = TinyDiT(cfg)
    tensors, entries = {}, []
    for i, blk in enumerate(model.blocks):
        for lname in ("qkv", "proj", "fc1", "fc2"):
            lin = getattr(blk, lname)
            name = f"blocks.{i}.{lname}"
            K, N = lin.in_features, lin.out_features
            t = gptq_layer(K, N, groupsize, seed=seed * 1000 + len(entries), v1=v1, actorder=actorder)
            for k, v in t.items():
                tensors[f"{name}.{k}"] = v.contiguous()
            entries.append(dict(name=name, wbits=4, groupsize=groupsize, actorder=actorder, in_features=K,
                                out_features=N))
    quant = {e["name"] for e in entries}
    for k, v in model.state_dict().items():
        if k.rsplit(".", 1)[0] not in quant:
            tensors[k] = v.to(torch.bfloat16).contiguous()
    if extra:
        tensors.update(extra)
    meta = {"config_json": json.dumps(cfg), "quant_layers_json": json.dumps(entries),
            "checkpoint_format": "gptq" if v1 else "gptq_v2"}
    save_file(tensors, str(path), metadata=meta)
    return entries
