"""Eager linear oracle (test infrastructure only).

The reference's "eager" backend (``backend.py:246-264``) dequantizes once with
``dequant_gptq_to_fp`` into an ``nn.Linear`` of the compute dtype and then runs
``F.linear``. On CPU that is a bf16 matmul with fp32 accumulation and a single
rounding of the output.

* ``linear_ref`` is the accuracy reference the GPU kernels are held to:
  ``round(x @ W.T + b)`` with the product accumulated in float64 from the exact
  bf16/fp16 operand values (the bias is added in fp32 as well).
* ``EagerCPU`` is the reference CPU path itself (dequant once + torch CPU
  ``F.linear``), timed as the CPU baseline by ``bench.py``.
* ``max_abs_rel`` is the error metric of the parity tests:
  ``max|y - ref| / max|ref|``.
"""
from __future__ import annotations

import numpy as np

from .fp import round_to, to_f32


def linear_ref(x_bits, x_dtype, w_bits, w_dtype, bias=None, bias_dtype=None,
               out_dtype=None):
    """float64-accumulated ``x @ W.T + b`` returned as float32 (unrounded) and rounded."""
    x = to_f32(x_bits, x_dtype).astype(np.float64)
    w = to_f32(w_bits, w_dtype).astype(np.float64)
    y = x @ w.T
    if bias is not None:
        y = y + to_f32(bias, bias_dtype).astype(np.float64)
    y32 = y.astype(np.float32)
    return y32, round_to(y32, out_dtype or x_dtype)


def max_abs_rel(y: np.ndarray, ref: np.ndarray) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(ref))) if ref.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(y - ref))) if y.size else 0.0
    return float(np.max(np.abs(y - ref)) / denom)


class EagerCPU:
    """The reference eager path on host cores: one dequant, then torch CPU F.linear.

    ``weight_bits`` is the dequantized bf16/fp16 weight [N, K] (bit patterns) as
    ``dequant_gptq`` returns it; the matmul is torch's CPU ``F.linear`` in the
    compute dtype, exactly what ``backend.build_eager`` + ``nn.Linear`` run.
    """

    def __init__(self, weight_bits, dtype: str, bias=None, bias_dtype=None):
        import torch

        tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[dtype]
        self.torch = torch
        self.dtype = tdt
        self.weight = torch.from_numpy(np.ascontiguousarray(weight_bits).view(np.int16)).view(tdt)
        self.bias = None
        if bias is not None:
            self.bias = torch.from_numpy(to_f32(bias, bias_dtype)).to(tdt)

    def __call__(self, x):
        return self.torch.nn.functional.linear(x, self.weight, self.bias)
