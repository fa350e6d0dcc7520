"""Build the sm_100a shared library ``libtilemix_b200.so`` in-tree with nvcc.

The library is a plain C-ABI shared object (see ``include/tilemix_b200.h``):
no PyTorch headers, the CUDA runtime linked statically, so it loads on hosts
without a GPU driver (the symbols can be inspected there; launching needs a
B200). Run ``python -m tilemix_b200.build`` or call :func:`build`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "libtilemix_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["attn_api.cu", "attn_fwd_general.cu", "attn_fwd_paired.cu", "quant.cu", "precision_map.cu",
           "attn_noalloc.cu", "prefill.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
    "-cudart", "static",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists() and shutil.which(cand) is None:
        raise RuntimeError("nvcc not found; the sm_100a kernels need the CUDA toolkit")
    return cand


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every CUDA source into ``tilemix_b200/libtilemix_b200.so``."""
    if not force and not _stale():
        return LIB_PATH
    srcs = [str(CSRC / s) for s in SOURCES]
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-shared", "-o", str(tmp), *srcs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
