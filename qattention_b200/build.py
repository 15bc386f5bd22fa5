"""Build the in-tree C-ABI library ``libqattn_b200.so`` for sm_100a with nvcc.

Each ``csrc/*.cu`` file is compiled to an object (``_build/``) and linked into
one shared library next to this file, so that the library travels with the
source tree. Rebuilds only what changed (by mtime of the source and headers).
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libqattn_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _headers() -> list[Path]:
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr_mtime = max((p.stat().st_mtime for p in _headers()), default=0.0)
    objs, cmds = [], []
    for src in sorted(CSRC.glob("*.cu")):
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if obj.exists() and not ptxas_info and obj.stat().st_mtime > max(src.stat().st_mtime, hdr_mtime):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
    # the translation units are independent: compile them side by side
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as pool:
        for r in pool.map(lambda c: subprocess.run(c, check=True), cmds):
            pass
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
