"""Build the Kitty B200 CUDA library in-tree.

    python kitty-kv_b200/build.py            # -> kitty-kv_b200/kitty/libkitty_b200.so

Compiles every ``csrc/*.cu`` for sm_100a only (no PTX for other targets) with
IEEE float32 division and square root (no --use_fast_math: the quantisers must
round exactly like the reference) and links one shared library exporting the
C ABI declared in ``include/kitty_b200.h``.  Objects go to ``_build/``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD = PKG_ROOT / "_build"
LIB = PKG_ROOT / "kitty" / "libkitty_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-I", str(REPO_ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin directory on PATH")


def build(verbose: bool = False, extra: list | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + [REPO_ROOT / "include" / "kitty_b200.h"]
    newest_header = max(h.stat().st_mtime for h in headers)
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
            continue
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *(extra or []), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if (not LIB.exists()) or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv, extra=[a for a in sys.argv[1:] if a != "-q"])
    print(LIB)
