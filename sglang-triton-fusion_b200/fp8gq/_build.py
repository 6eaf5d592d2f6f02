"""Build libfp8gq.so (the C ABI in include/fp8gq.h) in-tree with nvcc for
sm_100a.  Run ``python -m fp8gq._build`` (with ``sglang-triton-fusion_b200``
on sys.path) or call :func:`build`."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_DIR = PKG_DIR.parent / "csrc"
REPO_DIR = PKG_DIR.parent.parent
LIB_PATH = PKG_DIR / "libfp8gq.so"
SOURCES = ["fp8gq_api.cu"]
HEADERS = ["fp8gq_device.cuh", "gemv_row.cuh", "gemm_tm.cuh", "quant_only.cuh", "swiglu_writer.cuh", "chain.cuh",
           "add_rmsnorm.cuh", "stack.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin/ on PATH)")
    return cand


def _inputs():
    files = [SRC_DIR / s for s in SOURCES] + [SRC_DIR / h for h in HEADERS]
    files.append(REPO_DIR / "include" / "fp8gq.h")
    return files


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(f.stat().st_mtime <= t for f in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> Path:
    """Compile libfp8gq.so next to this file unless it is already current."""
    if not force and up_to_date():
        return LIB_PATH
    cmd = [nvcc_path(), *NVCC_FLAGS, *(extra_flags or []),
           "-I", str(REPO_DIR / "include"),
           "-o", str(LIB_PATH) + ".tmp", *[str(SRC_DIR / s) for s in SOURCES]]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None))
