"""Int4-packed Conv1d / ConvTranspose1d (RTN nibble codec) on B200.

Same public surface as the reference ``layers/packed_conv.py`` (DACVAE conv codecs):
``pack_int4_nibbles`` / ``unpack_int4_nibbles``, ``quantize_conv_weight``,
``PackedInt4Conv1d``, ``PackedInt4ConvTranspose1d``, ``quantize_conv_module`` and
``replace_conv_with_packed``, with the same constructor arguments, buffers
(``qweight`` uint8 nibbles, ``scales`` / ``zeros`` [rows, groups], ``cols``) and the same
pad / unpad rules for ``NormConv1d`` / ``NormConvTranspose1d`` replacements.

The layer weight is a 2-D RTN table [rows, cols] (rows = output channels for Conv1d, input
channels for ConvTranspose1d; cols = the flattened (channels / groups) x kernel_size).

* Conv1d (groups == 1, fp16/bf16 on the GPU): the table is exactly a ``PackedRTNLinear``
  weight [out, C k], so the convolution runs as ``oc_b200_im2col_1d`` (the input unfolded to
  [B T, C k]) followed by the row-packed tcgen05 GEMM in RTN mode, which multiplies the weights
  the reference's dequant produces (two roundings in the activation dtype); no cuDNN.
* Grouped Conv1d, ConvTranspose1d (whose contraction runs over the table's rows, across its
  scale groups) and fp32 inputs: the weight is dequantized on the device by
  ``oc_b200_rtn_dequant`` -- bit-exact with the reference's ``(w_int - zeros) * scales`` in the
  activation dtype (packed_conv.py:48-60) -- and handed to ``F.conv1d`` /
  ``F.conv_transpose1d``, as the reference does. Only the layer being run holds a 16-bit copy.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..quant_utils import dequant_extra_u8_to_weight


def pack_int4_nibbles(w_int: torch.Tensor) -> torch.Tensor:
    """int [rows, cols] (values 0..15) -> uint8 [rows, ceil(cols / 2)]: even column in the
    low nibble, odd column in the high nibble (a zero column pads an odd count)."""
    rows, cols = w_int.shape
    v = w_int.to(torch.uint8) & 0x0F
    if cols % 2:
        v = torch.cat([v, torch.zeros(rows, 1, dtype=torch.uint8, device=v.device)], dim=1)
    return (v[:, 0::2] | (v[:, 1::2] << 4)).contiguous()


def unpack_int4_nibbles(packed: torch.Tensor, cols: int) -> torch.Tensor:
    """uint8 [rows, ceil(cols / 2)] -> int16 [rows, cols] (inverse of ``pack_int4_nibbles``)."""
    rows = packed.shape[0]
    both = torch.stack([(packed & 0x0F).to(torch.int16), ((packed >> 4) & 0x0F).to(torch.int16)], dim=-1)
    return both.reshape(rows, -1)[:, :cols]


def _dequant_weight(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, cols: int,
                    dtype: torch.dtype) -> torch.Tensor:
    """[rows, cols] weight in ``dtype`` (device kernel, bit-exact with the reference)."""
    return dequant_extra_u8_to_weight(qweight, scales, zeros, cols, qweight.shape[0], dtype)


def quantize_conv_weight(weight: torch.Tensor, groupsize: int = -1):
    """RTN 4-bit quantization of a 2-D (flattened) conv weight, as the reference's encoder
    (packed_conv.py:63-90): per row and group (``groupsize`` columns when it divides the
    column count, else the whole row) scale = max((max - min) / 15, 1e-8), zero =
    round(-min / scale), q = clamp(round(w / scale) + zero, 0, 15); an all-zero group uses
    min = -1, max = 1. Returns ``(qweight_u8, scales_fp16, zeros_fp16, cols)``."""
    if weight.dim() != 2:
        raise ValueError("flatten weight to 2-D before quantization")
    rows, cols = weight.shape
    groups = cols // groupsize if groupsize > 0 and cols % groupsize == 0 else 1
    w = weight.float().reshape(rows, groups, cols // groups)
    hi = w.amax(dim=-1, keepdim=True)
    lo = w.amin(dim=-1, keepdim=True)
    empty = (hi == 0) & (lo == 0)
    hi = torch.where(empty, torch.ones_like(hi), hi)
    lo = torch.where(empty, -torch.ones_like(lo), lo)
    scale = ((hi - lo) / 15).clamp(min=1e-8)
    zero = torch.round(-lo / scale)
    q = torch.clamp(torch.round(w / scale) + zero, 0, 15).to(torch.int32).reshape(rows, cols)
    scales = scale.squeeze(-1).to(torch.float16).reshape(rows, groups)
    zeros = zero.squeeze(-1).to(torch.float16).reshape(rows, groups)
    return pack_int4_nibbles(q), scales, zeros, cols


def _conv1d_pad(x: torch.Tensor, kernel_size: int, stride: int, dilation: int, pad_mode: str,
                causal: bool) -> torch.Tensor:
    """NormConv1d padding: enough on the right to complete the last frame, ``padding_total``
    split left / right (all on the left when causal); ``pad_mode == "none"`` pads nothing."""
    if pad_mode == "none":
        return x
    eff = (kernel_size - 1) * dilation + 1
    total = eff - stride
    frames = (x.shape[-1] - eff + total) / stride + 1
    extra = (math.ceil(frames) - 1) * stride + (kernel_size - total) - x.shape[-1]
    if causal:
        return F.pad(x, (total, extra))
    right = extra // 2
    return F.pad(x, (total - right, right + extra))


def _convtranspose1d_unpad(x: torch.Tensor, kernel_size: int, stride: int, pad_mode: str,
                           causal: bool) -> torch.Tensor:
    """NormConvTranspose1d trimming of ``kernel_size - stride`` samples (all from the right
    when causal)."""
    if pad_mode == "none":
        return x
    total = kernel_size - stride
    n = x.shape[-1]
    if causal:
        return x[..., :n - total]
    right = total // 2
    return x[..., total - right:n - right]


class _PackedConvBase(nn.Module):
    def _init_packed(self, rows: int, ck: int, qweight, scales, zeros, cols, bias):
        if qweight is None:
            qweight = torch.zeros(rows, (ck + 1) // 2, dtype=torch.uint8)
            scales = torch.zeros(rows, 1, dtype=torch.float16)
            zeros = torch.zeros(rows, 1, dtype=torch.float16)
            cols = ck
        self.register_buffer("qweight", qweight.contiguous())
        self.register_buffer("scales", scales.contiguous())
        self.register_buffer("zeros", zeros.contiguous())
        self.cols = int(cols)
        if bias is not None:
            self.register_parameter("bias", nn.Parameter(bias.detach(), requires_grad=False))
        else:
            self.bias = None

    def _bias(self, dtype):
        return self.bias.to(dtype) if self.bias is not None else None


class PackedInt4Conv1d(_PackedConvBase):
    """``NormConv1d``-compatible int4 Conv1d: weight [out, in / groups, k] stored as an RTN
    nibble table [out, (in / groups) * k]; padding as NormConv1d."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1, padding: int = 0,
                 dilation: int = 1, groups: int = 1, qweight: torch.Tensor | None = None,
                 scales: torch.Tensor | None = None, zeros: torch.Tensor | None = None, cols: int | None = None,
                 bias: torch.Tensor | None = None, causal: bool = False, pad_mode: str = "auto"):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.dilation = dilation
        self.groups = groups
        self.causal = causal
        self.pad_mode = pad_mode
        self._init_packed(out_channels, (in_channels // groups) * kernel_size, qweight, scales, zeros, cols, bias)

    def _materialize(self, dtype: torch.dtype) -> torch.Tensor:
        w = _dequant_weight(self.qweight, self.scales, self.zeros, self.cols, dtype)
        return w.reshape(self.out_channels, self.in_channels // self.groups, self.kernel_size)

    def _gemm_linear(self):
        """The same nibble table seen as an RTN linear [out, (in / groups) k] (shared buffers, not a
        submodule, so ``state_dict`` is unchanged), or None when the row-packed GEMM cannot take it."""
        from .packed_linear import PackedRTNLinear
        lin = self.__dict__.get("_lin")
        if lin is None or lin.qweight_u8 is not self.qweight or lin.scales is not self.scales:
            lin = PackedRTNLinear(self.cols, self.out_channels, self.qweight, self.scales, self.zeros, None)
            self.__dict__["_lin"] = lin
        return lin if lin._rows_handle() is not None else None

    def _forward_gemm(self, x: torch.Tensor, lin) -> torch.Tensor:
        """Conv1d as im2col (``oc_b200_im2col_1d``) + the row-packed tcgen05 GEMM in RTN mode, which
        multiplies exactly the weights ``_materialize`` produces; output [B, out, T] like F.conv1d."""
        from .. import _lib
        unbatched = x.dim() == 2
        xb = x.unsqueeze(0) if unbatched else x
        if xb.stride(-1) != 1:
            xb = xb.contiguous()
        B, C, L = xb.shape
        span = self.dilation * (self.kernel_size - 1) + 1
        T = (L + 2 * self.padding - span) // self.stride + 1
        if T <= 0:
            raise RuntimeError(f"PackedInt4Conv1d: input length {L} is shorter than the kernel span {span}")
        k_run = lin.__dict__["_k_run"]
        a = torch.empty((B * T, k_run), dtype=x.dtype, device=x.device)
        _lib.call("oc_b200_im2col_1d", xb.data_ptr(), xb.stride(0), xb.stride(1), B, C, L, self.kernel_size,
                  self.stride, self.dilation, self.padding, T, k_run, a.data_ptr(), a.stride(0),
                  _lib.stream_of(x.device))
        y = torch.empty((B * T, self.out_channels), dtype=x.dtype, device=x.device)
        if B * T:
            lin._rows_handle().gemm(a, y, bias=self._bias(x.dtype))
        y = y.view(B, T, self.out_channels).permute(0, 2, 1).contiguous()
        return y[0] if unbatched else y

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = _conv1d_pad(x, self.kernel_size, self.stride, self.dilation, self.pad_mode, self.causal)
        if x.is_cuda and x.dtype in (torch.float16, torch.bfloat16) and self.groups == 1:
            lin = self._gemm_linear()
            if lin is not None:
                return self._forward_gemm(x, lin)
        return F.conv1d(x, self._materialize(x.dtype), self._bias(x.dtype), self.stride, self.padding,
                        self.dilation, self.groups)

    def _apply(self, fn, recurse=True):
        self.__dict__["_lin"] = None
        return super()._apply(fn, recurse=recurse)


class PackedInt4ConvTranspose1d(_PackedConvBase):
    """``NormConvTranspose1d``-compatible int4 ConvTranspose1d: weight [in, out / groups, k]
    stored as an RTN nibble table [in, (out / groups) * k]; trimming as NormConvTranspose1d."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, stride: int = 1, padding: int = 0,
                 output_padding: int = 0, dilation: int = 1, groups: int = 1, qweight: torch.Tensor | None = None,
                 scales: torch.Tensor | None = None, zeros: torch.Tensor | None = None, cols: int | None = None,
                 bias: torch.Tensor | None = None, causal: bool = False, pad_mode: str = "auto"):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding
        self.output_padding = output_padding
        self.dilation = dilation
        self.groups = groups
        self.causal = causal
        self.pad_mode = pad_mode
        self._init_packed(in_channels, (out_channels // groups) * kernel_size, qweight, scales, zeros, cols, bias)

    def _materialize(self, dtype: torch.dtype) -> torch.Tensor:
        w = _dequant_weight(self.qweight, self.scales, self.zeros, self.cols, dtype)
        return w.reshape(self.in_channels, self.out_channels // self.groups, self.kernel_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = F.conv_transpose1d(x, self._materialize(x.dtype), self._bias(x.dtype), self.stride, self.padding,
                               self.output_padding, self.groups, self.dilation)
        return _convtranspose1d_unpad(y, self.kernel_size, self.stride, self.pad_mode, self.causal)


def _first(v):
    return v[0] if isinstance(v, tuple) else v


def quantize_conv_module(mod: nn.Module, groupsize: int = 32):
    """Packed replacement of a Conv1d / ConvTranspose1d (or NormConv wrapper exposing the
    same attributes) -- remove weight_norm first, as with the reference (packed_conv.py:227)."""
    weight = mod.weight.detach()
    bias = mod.bias.detach() if mod.bias is not None else None
    q, s, z, cols = quantize_conv_weight(weight.reshape(weight.shape[0], -1), groupsize=groupsize)
    common = dict(in_channels=mod.in_channels, out_channels=mod.out_channels, kernel_size=_first(mod.kernel_size),
                  stride=_first(mod.stride), padding=_first(mod.padding), dilation=_first(mod.dilation),
                  groups=mod.groups, qweight=q, scales=s, zeros=z, cols=cols, bias=bias,
                  causal=getattr(mod, "causal", False), pad_mode=getattr(mod, "pad_mode", "none"))
    if isinstance(mod, nn.ConvTranspose1d):
        return PackedInt4ConvTranspose1d(output_padding=_first(mod.output_padding), **common)
    return PackedInt4Conv1d(**common)


def replace_conv_with_packed(model: nn.Module, *, groupsize: int = 32,
                             cast_remaining_to: torch.dtype | None = torch.float16) -> dict:
    """Swap every (Norm)Conv1d / (Norm)ConvTranspose1d of ``model`` for its packed form and
    cast the remaining floating parameters and buffers to ``cast_remaining_to``; returns
    ``{"replaced", "bytes_before", "bytes_after", "ratio"}`` as the reference does
    (packed_conv.py:267-339)."""
    targets = ("NormConv1d", "NormConvTranspose1d", "Conv1d", "ConvTranspose1d")
    found = [(name, m) for name, m in model.named_modules()
             if type(m).__name__ in targets and hasattr(m, "kernel_size")]
    replaced = bytes_before = bytes_after = 0
    for name, mod in found:
        try:
            from torch.nn.utils import remove_weight_norm
            remove_weight_norm(mod)
        except (ValueError, AttributeError):
            pass
        bytes_before += sum(p.numel() * p.element_size() for p in mod.parameters(recurse=False))
        packed = quantize_conv_module(mod, groupsize=groupsize)
        bytes_after += sum(b.numel() * b.element_size() for b in packed.buffers(recurse=False))
        bytes_after += sum(p.numel() * p.element_size() for p in packed.parameters(recurse=False))
        parent_name, _, child = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child, packed)
        replaced += 1
    if cast_remaining_to is not None:
        for mod in model.modules():
            if isinstance(mod, (PackedInt4Conv1d, PackedInt4ConvTranspose1d)):
                continue
            for pname, p in list(mod._parameters.items()):
                if p is not None and p.dtype.is_floating_point and p.dtype != cast_remaining_to:
                    mod._parameters[pname] = nn.Parameter(p.data.to(cast_remaining_to), requires_grad=p.requires_grad)
            for bname, b in list(mod._buffers.items()):
                if b is not None and b.dtype.is_floating_point and b.dtype != cast_remaining_to:
                    mod._buffers[bname] = b.to(cast_remaining_to)
        for mod in model.modules():
            if isinstance(mod, nn.LSTM):
                mod.flatten_parameters()
    return {"replaced": replaced, "bytes_before": bytes_before, "bytes_after": bytes_after,
            "ratio": bytes_after / bytes_before if bytes_before else 0.0}
