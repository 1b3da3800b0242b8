"""Shared pytest setup: markers, import paths and fixture loaders."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "onecompression-runtime_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running test")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        data = {k: z[k] for k in z.files}
    data["meta"] = json.loads(str(data["meta"]))
    return data


GPTQ_CASES = [
    "gptq_v1_gs32",
    "gptq_v2_gs128_actorder",
    "gptq_v1_gs128_bf16scales",
    "gptq_v1_gs26_odd",
    "gptq_v1_gs64_8bit",
    "gptq_v2_irregular_gidx",
    "gptq_v1_gs32_m17",
    "gptq_v1_gs32_8bit_m5",
    "gptq_v2_gs128_8bit_bf16",
]
RTN_CASES = ["rtn_grouped", "rtn_perrow", "rtn_gs32_bf16"]
DSV4_CASES = ["dsv4_int2_gs64", "dsv4_int4_gs128_go", "dsv4_int2_perrow", "dsv4_int4_ragged"]
EMB_CASES = ["rtn_embedding_f16", "rtn_embedding_bf16_perrow", "rtn_embedding_f32"]
CONV_CASES = ["conv1d_int4", "conv1d_int4_causal_grouped", "convtr1d_int4"]


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100, got sm_{major}{minor}")
    return torch.device("cuda:0")
