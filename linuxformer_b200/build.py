"""Build the CUDA library in-tree: nvcc for sm_100a straight into linuxformer_b200/_build/.

    python -m linuxformer_b200.build

The library is a plain shared object with the C ABI of include/lxb.h; Python reaches it through
ctypes (linuxformer_b200/_lib.py), as the reference reaches its megakernel
(lx/lx/mk_build.py:40-57), but it is built ahead of time, not at first use.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
OUT = PKG / "_build"
LIB = OUT / "liblxb.so"
SOURCES = [PKG / "csrc" / "decode.cu", PKG / "csrc" / "prefill.cu", PKG / "csrc" / "text.cu"]
HEADERS = [PKG / "csrc" / "lxb_math.h", PKG / "csrc" / "lxb_plan.h", PKG / "csrc" / "lxb_prefill.h",
           ROOT / "include" / "lxb.h"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
              "-fmad=false", "-Xcompiler", "-fPIC", "-shared", f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (Path(c).exists() or c == "nvcc"):
            return c
    return "nvcc"


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    OUT.mkdir(exist_ok=True)
    tmp = OUT / f"liblxb.{os.getpid()}.so"
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc failed:\n{r.stderr}")
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
