"""Build the sm_100a C-ABI library libgptq_b200.so in-tree.

    python mlx-gptq-mxfp_b200/build.py [--force] [-v]

Compiles every csrc/*.cu with nvcc for sm_100a only and links them into
mlx_gptq_b200/_lib/libgptq_b200.so. Objects go to _build/ (git-ignored); a
source is recompiled when it or any csrc header is newer than its object.
-fmad=false keeps every float expression rounded per operation, like the
reference's torch ops; intended fused multiply-adds are explicit fmaf().
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT_DIR = os.path.join(HERE, "mlx_gptq_b200", "_lib")
LIB = os.path.join(OUT_DIR, "libgptq_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(OUT_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.inc")) + [
        os.path.join(INCLUDE, "gptq_b200.h")]
    newest_header = max(os.path.getmtime(h) for h in headers)
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if (not force and os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
                and os.path.getmtime(obj) >= newest_header):
            continue
        cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args()
    print(build(a.force or a.ptxas_info, a.verbose, ["-Xptxas", "-v"] if a.ptxas_info else None))
