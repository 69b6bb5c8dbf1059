"""Build ``libsarbon_sparse.so`` (the C ABI in ``include/sarbon_sparse.h``) for sm_100a.

The library is built in-tree next to this file so that it travels with the source
tree; object files go to ``sarbon_b200/_build``.  Usage::

    python -m sarbon_b200.build_lib          # or: from sarbon_b200.build_lib import build
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libsarbon_sparse.so"
SOURCES = ["sb_engine.cu", "sb_gate.cu", "sb_conv_tc.cu", "sb_conv_simt.cu", "sb_noalloc.cu", "sb_cells.cu", "sb_boxes.cu",
           "sb_prep.cu", "sb_deform.cu", "sb_gemm.cu", "sb_detops.cu", "sb_attn.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{PKG.parent / 'include'}"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _compile(src: str, extra) -> Path:
    out = OBJ / (Path(src).stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", str(CSRC / src), "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)
    return out


def build(force: bool = False, extra=(), verbose: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library."""
    srcs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "sarbon_sparse.h"]
    if LIB.exists() and not force:
        newest = max(p.stat().st_mtime for p in srcs)
        if LIB.stat().st_mtime > newest:
            return LIB
    OBJ.mkdir(exist_ok=True)
    with ThreadPoolExecutor(len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, list(extra)), SOURCES))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "--cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
