"""Build the sm_100a C-ABI library ``liboc_b200.so`` in-tree.

    python onecompression-runtime_b200/build.py [--verbose]

The library is a single CUDA translation unit (``csrc/oc_b200.cu``) compiled by
nvcc for ``sm_100a`` only and placed next to the Python package
(``onecomp_runtime/liboc_b200.so``), where ``onecomp_runtime._lib`` loads it.
No torch headers are involved: the Python layer binds the plain C ABI.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "onecomp_runtime" / "liboc_b200.so"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "oc_b200.h"]


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE}", str(CSRC / "oc_b200.cu"), "-o", str(OUT) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(force=True, verbose="--verbose" in sys.argv)
    print(OUT)
