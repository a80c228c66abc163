"""Build liblvb.so (the sm_100a kernels + the C ABI) in-tree with nvcc.

    python lava.jl_b200/build.py [--force] [--verbose]

Output: lava.jl_b200/lib/liblvb.so. The library links the CUDA runtime statically and
resolves the one driver call it needs (cuTensorMapEncodeTiled) through the runtime's
driver entry point, so it loads on a machine without a GPU or libcuda (the CPU tests check
its exported symbols there) and needs nothing but the driver on a B200 box.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
LIBDIR = HERE / "lib"
LIB = LIBDIR / "liblvb.so"
SOURCES = ["abi.cu", "gemm_sm100.cu", "gemv_sm100.cu", "attn_sm100.cu", "attn_decode_sm100.cu",
           "selftest.cu", "comm.cu"]
HEADERS = ["sm100.cuh", "epilogue.cuh", "lvb_internal.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _inputs():
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [REPO / "include" / "lvb.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_v else []

    def compile_one(s):
        obj = objdir / (Path(s).stem + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-I", str(REPO / "include"), "-c", str(CSRC / s),
               "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        return s, obj, subprocess.run(cmd, capture_output=True, text=True)

    # The translation units are independent: compile them side by side (nvcc is
    # single-threaded per file).
    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    objs = []
    for s, obj, r in results:
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"nvcc failed on {s}")
        if verbose or ptxas_v:
            sys.stderr.write(r.stderr)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print registers/spills per kernel")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))
