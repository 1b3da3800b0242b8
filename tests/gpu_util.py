"""Helpers shared by the GPU parity tests (bit-pattern <-> torch conversions, reference GEMMs)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import eager, gptq

TDT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
NAME = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}

# GEMM tolerance (north star): max-abs-relative error vs the fp64-accumulated
# product of the exact dequantized weights, for bf16/fp16 outputs.
GEMM_TOL = 2e-2


def to_torch(bits: np.ndarray, name: str, device="cuda") -> torch.Tensor:
    if name == "f32":
        return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.float32)).to(device)
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(TDT[name]).to(device)


def to_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def tensors_to_np(d: dict) -> dict:
    out = {}
    for k, v in d.items():
        if v.dtype in (torch.float16, torch.bfloat16):
            out[k] = to_bits(v)
        else:
            out[k] = v.detach().cpu().numpy()
    return out


def oracle_weight(t: dict, K: int, N: int, out_name: str, v1: bool = True, wbits: int = 4) -> np.ndarray:
    """Exact dequantized weight [N, K] (bit patterns) from torch layer tensors."""
    n = tensors_to_np(t)
    s_name = NAME[t["scales"].dtype]
    return gptq.dequant_gptq(n["qweight"], n["scales"], s_name, n["qzeros"], n["g_idx"], K, N, out_name, v1=v1,
                             wbits=wbits)


def reference_output(x: torch.Tensor, w_bits: np.ndarray, w_name: str, bias: torch.Tensor | None):
    xb = to_bits(x)
    xn = NAME[x.dtype]
    b = None if bias is None else to_bits(bias)
    bn = None if bias is None else NAME[bias.dtype]
    y32, _ = eager.linear_ref(xb, xn, w_bits, w_name, b, bn)
    return y32


def max_abs_rel(y: torch.Tensor, ref: np.ndarray) -> float:
    return eager.max_abs_rel(y.detach().float().cpu().numpy(), ref)
