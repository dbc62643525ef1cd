"""Build liboz_b200.so (sm_100a) in-tree with nvcc.

    python -m ozaki_triton_b200.csrc.build      # or build() from Python

The translation units are compiled for sm_100a only (in parallel) and
linked with the CUDA runtime static, so the .so loads without a CUDA toolkit
on the library path.  No GPU is needed to build.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "liboz_b200.so")
UNITS = ["oz_api.cu", "oz_split.cu", "oz_gemm.cu", "oz_peer.cu"]
SOURCES = UNITS + ["oz_common.cuh", "oz_log2_table.h", "oz_tile_table.h"]
BUILD_DIR = os.path.join(PKG, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(HERE, f) for f in SOURCES] + [os.path.join(ROOT, "include", "ozaki_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = nvcc_path()
    common = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-I", os.path.join(ROOT, "include")]
    if verbose:
        common.append("-Xptxas=-v")
    procs, objs = [], []
    for unit in UNITS:
        obj = os.path.join(BUILD_DIR, unit.replace(".cu", ".o"))
        cmd = [nvcc, *common, "-c", os.path.join(HERE, unit), "-o", obj]
        print("[ozaki_b200] nvcc", unit, flush=True)
        procs.append((unit, subprocess.Popen(cmd)))
        objs.append(obj)
    failed = [u for u, pr in procs if pr.wait() != 0]
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    link = [nvcc, *ARCH, "-shared", "-cudart", "static", *objs, "-o", LIB + ".tmp"]
    subprocess.run(link, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
