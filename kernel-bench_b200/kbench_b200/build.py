"""Build ``libkb_solver.so`` (all CUDA kernels + the C ABI) in-tree with nvcc for sm_100a.

    python kernel-bench_b200/kbench_b200/build.py [--verbose]

The shared library lands next to this file (``kbench_b200/libkb_solver.so``); the Python layer
loads it with ctypes and fails loudly when it is missing.  ``-Xptxas -v`` output (registers,
spills, shared memory per kernel) is written to ``_build/ptxas.txt`` for inspection.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libkb_solver.so"
SOURCES = ["kb_misc.cu", "kb_estep.cu", "kb_params.cu", "kb_dts.cu", "kb_wave_fwd.cu", "kb_wave_bwd.cu", "kb_engine.cu", "kb_tangent.cu", "kb_hvp.cu", "kb_builder.cu", "kb_sched.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + [INCLUDE / "kb_solver.h"]
    if LIB.exists() and not force:
        lib_mtime = LIB.stat().st_mtime
        if all(d.stat().st_mtime <= lib_mtime for d in deps):
            return LIB
    build_dir = REPO / "_build"
    build_dir.mkdir(exist_ok=True)
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-Xptxas", "-v", f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(LIB) + ".tmp", *map(str, srcs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    (build_dir / "ptxas.txt").write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    os.replace(str(LIB) + ".tmp", LIB)
    if verbose:
        print(res.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
