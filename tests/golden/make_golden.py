"""Generate golden vectors by running the reference ``onecomp_runtime`` on CPU.

Run in a container that has the reference checked out (read-only is fine)::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference

Every case draws seeded inputs with numpy, feeds them to the reference's own
functions (``quant_utils.dequant_gptq_to_fp``, ``quant_utils.dequant_extra_u8_to_weight``,
``layers.dsv4_packed_linear.dequant_dsv4_packed``, ``backend.build_eager`` +
``nn.Linear``, ``layers.packed_linear.PackedEmbedding``, ``layers.packed_conv``) and stores inputs and outputs (bf16/fp16 as uint16 bit patterns)
in ``tests/golden/<case>.npz``. The tests load these fixtures; nothing at test
time imports the reference.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _bits(t):
    import torch
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def _tdt(name):
    import torch
    return {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[name]


def _pack_k(codes_nk: np.ndarray, wbits: int) -> np.ndarray:
    pf = 32 // wbits
    rows = codes_nk.T.astype(np.int64)
    out = np.zeros((rows.shape[0] // pf, rows.shape[1]), dtype=np.int64)
    for i in range(pf):
        out |= (rows[i::pf] & ((1 << wbits) - 1)) << (i * wbits)
    return out.astype(np.uint32).view(np.int32)


def _pack_n(z_gn: np.ndarray, wbits: int) -> np.ndarray:
    pf = 32 // wbits
    g, n = z_gn.shape
    out = np.zeros((g, n // pf), dtype=np.int64)
    for j in range(pf):
        out |= (z_gn[:, j::pf].astype(np.int64) & ((1 << wbits) - 1)) << (j * wbits)
    return out.astype(np.uint32).view(np.int32)


def gptq_case(name, *, K, N, gs, wbits=4, v1=True, actorder=False, scales_dtype="f16",
              out_dtypes=("bf16", "f16"), M=0, bias=True, seed=0, g_idx_mode="default"):
    import torch
    from onecomp_runtime import backend, quant_utils

    rng = np.random.default_rng(seed)
    qmax = (1 << wbits) - 1
    G = (K + gs - 1) // gs
    codes = rng.integers(0, qmax + 1, size=(N, K))
    zero = rng.integers(1, qmax + 1, size=(G, N))
    stored = (zero - 1) & qmax if v1 else zero
    qweight = _pack_k(codes, wbits)
    qzeros = _pack_n(stored, wbits)
    s32 = rng.uniform(0.002, 0.02, size=(G, N)).astype(np.float32)
    scales_t = torch.from_numpy(s32).to(_tdt(scales_dtype))
    if actorder:
        g_idx = (np.arange(K) // gs)[rng.permutation(K)].astype(np.int64)
    elif g_idx_mode == "irregular":
        g_idx = np.sort(rng.integers(0, G, size=K)).astype(np.int64)
        g_idx[:G] = np.arange(G)
        g_idx = np.sort(g_idx)
    else:
        g_idx = (np.arange(K) // gs).astype(np.int64)
    data = dict(qweight=qweight, qzeros=qzeros, scales=_bits(scales_t), g_idx=g_idx,
                meta=json.dumps(dict(K=K, N=N, gs=gs, wbits=wbits, v1=v1,
                                     scales_dtype=scales_dtype, M=M, bias=bias,
                                     out_dtypes=list(out_dtypes), actorder=actorder)))
    for od in out_dtypes:
        w = quant_utils.dequant_gptq_to_fp(
            torch.from_numpy(qweight), scales_t, torch.from_numpy(qzeros),
            torch.from_numpy(g_idx), K, N, _tdt(od), v1=v1, wbits=wbits)
        data[f"w_{od}"] = _bits(w)
    if M:
        x32 = rng.standard_normal((M, K)).astype(np.float32)
        b32 = (rng.standard_normal(N) * 0.02).astype(np.float32)
        for od in out_dtypes:
            dt = _tdt(od)
            st = {"qweight": torch.from_numpy(qweight), "scales": scales_t,
                  "qzeros": torch.from_numpy(qzeros), "g_idx": torch.from_numpy(g_idx)}
            if bias:
                st["bias"] = torch.from_numpy(b32).to(torch.float16)
            entry = dict(name="l", wbits=wbits, groupsize=gs, actorder=actorder,
                         in_features=K, out_features=N,
                         checkpoint_format="gptq" if v1 else "gptq_v2")
            if wbits == 4:
                lin = backend.build_eager(entry, st, dt, torch.device("cpu"))
            else:
                # the reference's build_eager dequantizes with the default wbits=4
                # (backend.py:253-257); its PackedGPTQLinear passes wbits through
                from onecomp_runtime.layers.packed_gptq_linear import PackedGPTQLinear
                lin = PackedGPTQLinear(K, N, st["qweight"], st["scales"], st["qzeros"], st["g_idx"],
                                       st.get("bias"), gs, wbits, v1)
            x = torch.from_numpy(x32).to(dt)
            with torch.no_grad():
                y = lin(x)
            data[f"x_{od}"] = _bits(x)
            data[f"y_{od}"] = _bits(y)
        if bias:
            data["bias_f16"] = _bits(torch.from_numpy(b32).to(torch.float16))
    np.savez_compressed(HERE / f"{name}.npz", **data)
    print("wrote", name)


def rtn_case(name, *, out_f, in_f, ncols, groups, zeros_dtype, scales_dtype, seed, M=0):
    import torch
    from onecomp_runtime import quant_utils
    from onecomp_runtime.layers.packed_linear import PackedRTNLinear

    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, size=(out_f, ncols), dtype=np.uint8)
    s32 = rng.uniform(0.002, 0.05, size=(out_f, groups)).astype(np.float32)
    if zeros_dtype == "f32":
        z32 = rng.uniform(0.0, 15.0, size=(out_f, groups)).astype(np.float32)
    else:
        z32 = rng.integers(0, 16, size=(out_f, groups)).astype(np.float32) + 0.5 * rng.integers(0, 2, size=(out_f, groups))
    s_t = torch.from_numpy(s32).to(_tdt(scales_dtype))
    z_t = torch.from_numpy(z32.astype(np.float32)).to(_tdt(zeros_dtype))
    data = dict(qweight_u8=q, scales=_bits(s_t), zeros=_bits(z_t),
                meta=json.dumps(dict(out_f=out_f, in_f=in_f, groups=groups,
                                     zeros_dtype=zeros_dtype, scales_dtype=scales_dtype, M=M)))
    for od in ("bf16", "f16"):
        w = quant_utils.dequant_extra_u8_to_weight(torch.from_numpy(q), s_t, z_t, in_f, out_f, _tdt(od))
        data[f"w_{od}"] = _bits(w)
    if M:
        x32 = rng.standard_normal((M, in_f)).astype(np.float32)
        b32 = (rng.standard_normal(out_f) * 0.02).astype(np.float32)
        for od in ("bf16", "f16"):
            dt = _tdt(od)
            lin = PackedRTNLinear(in_f, out_f, torch.from_numpy(q), s_t, z_t,
                                  bias=torch.from_numpy(b32))
            x = torch.from_numpy(x32).to(dt)
            with torch.no_grad():
                y = lin(x)
            data[f"x_{od}"] = _bits(x)
            data[f"y_{od}"] = _bits(y)
        data["bias_f32"] = b32
    np.savez_compressed(HERE / f"{name}.npz", **data)
    print("wrote", name)


def dsv4_case(name, *, out_f, in_f, wbits, gs, layout, seed, zeros="const"):
    import torch
    from onecomp_runtime.layers.dsv4_packed_linear import dequant_dsv4_packed

    rng = np.random.default_rng(seed)
    per = 8 // wbits
    ncol = (in_f + per - 1) // per
    packed = rng.integers(0, 256, size=(out_f, ncol), dtype=np.uint8)
    G = (in_f + gs - 1) // gs if gs > 0 else 1
    s32 = rng.uniform(0.005, 0.05, size=(out_f, G)).astype(np.float32)
    if zeros == "const":
        z32 = np.full((out_f, G), 1.5, dtype=np.float32)
    else:
        z32 = rng.uniform(0.0, (1 << wbits) - 1, size=(out_f, G)).astype(np.float32)
    if layout == "go":
        s32, z32 = np.ascontiguousarray(s32.T), np.ascontiguousarray(z32.T)
    s_t = torch.from_numpy(s32).to(torch.float16)
    z_t = torch.from_numpy(z32).to(torch.float16)
    p = {"qweight_packed": torch.from_numpy(packed), "scales": s_t, "qzeros": z_t,
         "wbits": wbits, "groupsize": gs, "in_features": in_f}
    data = dict(qweight_packed=packed, scales=_bits(s_t), qzeros=_bits(z_t),
                meta=json.dumps(dict(out_f=out_f, in_f=in_f, wbits=wbits, gs=gs, layout=layout)))
    for od in ("bf16", "f16"):
        data[f"w_{od}"] = _bits(dequant_dsv4_packed(p, dtype=_tdt(od)))
    np.savez_compressed(HERE / f"{name}.npz", **data)
    print("wrote", name)


def embedding_case(name, *, vocab, dim, groups, scales_dtype, zeros_dtype, ids_shape, seed):
    import torch
    from onecomp_runtime.layers.packed_linear import PackedEmbedding

    rng = np.random.default_rng(seed)
    q = rng.integers(0, 256, size=(vocab, (dim + 1) // 2), dtype=np.uint8)
    s32 = rng.uniform(0.002, 0.05, size=(vocab, groups)).astype(np.float32)
    z32 = (rng.integers(0, 16, size=(vocab, groups)) + 0.5 * rng.integers(0, 2, size=(vocab, groups))).astype(np.float32)
    ids = rng.integers(-vocab, vocab, size=ids_shape).astype(np.int64)
    s_t = torch.from_numpy(s32).to(_tdt(scales_dtype))
    z_t = torch.from_numpy(z32).to(_tdt(zeros_dtype))
    emb = PackedEmbedding(vocab, dim, torch.from_numpy(q), s_t, z_t)
    with torch.no_grad():
        y = emb(torch.from_numpy(ids))
    np.savez_compressed(HERE / f"{name}.npz", qweight_u8=q, scales=_bits(s_t), zeros=_bits(z_t), ids=ids,
                        y=_bits(y), meta=json.dumps(dict(vocab=vocab, dim=dim, groups=groups,
                                                         scales_dtype=scales_dtype, zeros_dtype=zeros_dtype,
                                                         out_dtype={torch.float16: "f16", torch.bfloat16: "bf16",
                                                                    torch.float32: "f32"}[y.dtype])))
    print("wrote", name)


def conv_case(name, *, transpose, cin, cout, k, stride, dilation, groups, groupsize, causal, pad_mode, L, seed):
    import torch
    from onecomp_runtime.layers import packed_conv as pc

    rng = np.random.default_rng(seed)
    wshape = (cin, cout // groups, k) if transpose else (cout, cin // groups, k)
    w32 = (rng.standard_normal(wshape) * 0.1).astype(np.float32)
    w32.reshape(w32.shape[0], -1)[0, :] = 0.0          # an all-zero quantization group
    b32 = (rng.standard_normal(cout) * 0.05).astype(np.float32)
    q, s, z, cols = pc.quantize_conv_weight(torch.from_numpy(w32).reshape(w32.shape[0], -1), groupsize=groupsize)
    common = dict(kernel_size=k, stride=stride, dilation=dilation, groups=groups, qweight=q, scales=s, zeros=z,
                  cols=cols, bias=torch.from_numpy(b32), causal=causal, pad_mode=pad_mode)
    mod = (pc.PackedInt4ConvTranspose1d(cin, cout, **common) if transpose else pc.PackedInt4Conv1d(cin, cout, **common))
    x32 = rng.standard_normal((2, cin, L)).astype(np.float32)
    data = dict(weight_f32=w32, bias_f32=b32, qweight=q.numpy(), scales=_bits(s), zeros=_bits(z), x_f32=x32,
                meta=json.dumps(dict(transpose=transpose, cin=cin, cout=cout, k=k, stride=stride, dilation=dilation,
                                     groups=groups, groupsize=groupsize, causal=causal, pad_mode=pad_mode, cols=cols)))
    for od in ("bf16", "f16"):
        data[f"w_{od}"] = _bits(pc._dequant_weight(q, s, z, cols, _tdt(od)))
    x = torch.from_numpy(x32).to(torch.bfloat16)
    with torch.no_grad():
        data["y_bf16"] = _bits(mod(x))
    np.savez_compressed(HERE / f"{name}.npz", **data)
    print("wrote", name)


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ONECOMP_REFERENCE", "")
    if not ref:
        raise SystemExit("usage: make_golden.py <path-to-reference-checkout>")
    sys.path.insert(0, ref)
    import torch
    torch.manual_seed(0)

    gptq_case("gptq_v1_gs32", K=256, N=128, gs=32, M=5, seed=1)
    gptq_case("gptq_v2_gs128_actorder", K=512, N=64, gs=128, v1=False, actorder=True, M=3, seed=2)
    gptq_case("gptq_v1_gs128_bf16scales", K=384, N=64, gs=128, scales_dtype="bf16", M=4, seed=3)
    gptq_case("gptq_v1_gs26_odd", K=520, N=64, gs=26, M=7, seed=4)
    gptq_case("gptq_v1_gs64_8bit", K=128, N=64, gs=64, wbits=8, seed=5)
    gptq_case("gptq_v2_irregular_gidx", K=256, N=32, gs=32, v1=False, g_idx_mode="irregular", M=2, seed=6)
    gptq_case("gptq_v1_gs32_m17", K=192, N=72, gs=32, M=17, bias=False, seed=7)
    gptq_case("gptq_v1_gs32_8bit_m5", K=512, N=128, gs=32, wbits=8, M=5, seed=8)
    gptq_case("gptq_v2_gs128_8bit_bf16", K=640, N=256, gs=128, wbits=8, v1=False, scales_dtype="bf16", M=2,
              seed=9)
    rtn_case("rtn_grouped", out_f=48, in_f=202, ncols=104, groups=2, zeros_dtype="f32",
             scales_dtype="f16", seed=10, M=3)
    rtn_case("rtn_perrow", out_f=40, in_f=96, ncols=48, groups=1, zeros_dtype="f16",
             scales_dtype="f32", seed=11, M=2)
    rtn_case("rtn_gs32_bf16", out_f=64, in_f=256, ncols=128, groups=8, zeros_dtype="bf16",
             scales_dtype="bf16", seed=12, M=9)
    dsv4_case("dsv4_int2_gs64", out_f=64, in_f=256, wbits=2, gs=64, layout="og", seed=20)
    dsv4_case("dsv4_int4_gs128_go", out_f=48, in_f=256, wbits=4, gs=128, layout="go", seed=21,
              zeros="rand")
    dsv4_case("dsv4_int2_perrow", out_f=32, in_f=100, wbits=2, gs=0, layout="og", seed=22,
              zeros="rand")
    dsv4_case("dsv4_int4_ragged", out_f=40, in_f=200, wbits=4, gs=64, layout="og", seed=23,
              zeros="rand")
    embedding_case("rtn_embedding_f16", vocab=300, dim=192, groups=6, scales_dtype="f16", zeros_dtype="f16",
                   ids_shape=(3, 5), seed=30)
    embedding_case("rtn_embedding_bf16_perrow", vocab=50, dim=70, groups=1, scales_dtype="bf16",
                   zeros_dtype="f32", ids_shape=(9,), seed=31)
    embedding_case("rtn_embedding_f32", vocab=64, dim=96, groups=4, scales_dtype="f32", zeros_dtype="f16",
                   ids_shape=(2, 7), seed=32)
    conv_case("conv1d_int4", transpose=False, cin=12, cout=16, k=5, stride=2, dilation=1, groups=1, groupsize=20,
              causal=False, pad_mode="auto", L=33, seed=40)
    conv_case("conv1d_int4_causal_grouped", transpose=False, cin=8, cout=12, k=7, stride=1, dilation=2, groups=2,
              groupsize=4, causal=True, pad_mode="auto", L=40, seed=41)
    conv_case("convtr1d_int4", transpose=True, cin=16, cout=8, k=8, stride=4, dilation=1, groups=1, groupsize=32,
              causal=False, pad_mode="auto", L=11, seed=42)


if __name__ == "__main__":
    main()
