"""Build the sm_100a C-ABI library in-tree (kernel_optim_b200/libkopt.so).

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the CUDA 12.9 toolchain is
installed. The library links the CUDA runtime statically and has no torch dependency; Python binds
it with ctypes (kernel_optim_b200/_lib.py).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libkopt.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["decode_attn.cu", "gemv.cu", "prefill_attn.cu"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/*.cu into libkopt.so if any source or header is newer than it."""
    deps = [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if not force and not _stale(LIB, deps):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-cudart", "static",
        "-I", str(INCLUDE), "-o", str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
