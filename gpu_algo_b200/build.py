"""Build recipe for libbfknn.so (sm_100a only), in-tree.

    python -m gpu_algo_b200.build            # incremental
    python -m gpu_algo_b200.build --force    # rebuild everything

The CUDA runtime is linked statically and the driver entry points are
resolved at run time, so the library loads on a machine without a GPU
driver (symbol checks) and needs nothing but the NVIDIA driver on a B200.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libbfknn.so")
SOURCES = ["bfknn.cu", "direct.cu", "merge.cu", "tc.cu", "noalloc.cu", "scan.cu"]
HEADERS = ["common.cuh", "internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE,
]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "bfknn.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _newer(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lpthread", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose, ptxas_info=a.ptxas_info))
    return 0


if __name__ == "__main__":
    sys.exit(main())
