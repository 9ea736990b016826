"""Compile the reference's own CUDA kernels into ``oracle/_ref/`` (TEST INFRASTRUCTURE).

The reference (hantaoyu-theory/gpu_algo, ``bf/``) keeps its kernels as CUDA C
source strings inside Python modules and JIT-compiles them through CuPy.
CuPy is not installed here, so this recipe:

1. imports the reference modules from the reference checkout with a stub
   ``cupy`` module (the strings are module constants; nothing else runs);
2. substitutes the template constants exactly as ``compile_kernel`` does
   (bf/fp32.py:200-209) for a few (K, D, BLOCK[, QPB]) instances;
3. appends a small host launcher of ours that launches the kernel with the
   runner's own grid / block / dynamic shared memory (bf/fp32.py:255-271,
   bf/fp32_heap.py:150-166);
4. compiles each instance with nvcc for sm_100a into
   ``oracle/_ref/ref_<instance>.so`` (git-ignored; it travels to the GPU box).

Only the GPU-side oracle pin (tests marked ``gpu``) loads these libraries,
to check the C oracle against the reference's real kernels.  Generated
sources stay under ``oracle/_ref/``; nothing of the reference is committed.

    python oracle/build_ref.py --ref /path/to/reference
    GPU_ALGO_REFERENCE=/path/to/reference python oracle/build_ref.py
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# where the reference checkout is: --ref, or this environment variable
REF_ENV = "GPU_ALGO_REFERENCE"


def reference_dir() -> str | None:
    """The reference checkout named by the environment, if any."""
    return os.environ.get(REF_ENV) or None

# (instance name, module, source constant, kernel name, K, D, block) -- block as the
# reference runner would choose it (bf/fp32.py:212-221) for these shapes.
INSTANCES = [
    ("bf_fp32_k10_d128", "bf.fp32", "_BF32_SRC", "bf_fp32", 10, 128),
    ("bf_fp32_k1_d128", "bf.fp32", "_BF32_SRC", "bf_fp32", 1, 128),
    ("bf_fp32_k100_d128", "bf.fp32", "_BF32_SRC", "bf_fp32", 100, 128),
    ("bf_fp32_smallk_k32_d128", "bf.fp32", "_BF32_SMALLK_SRC", "bf_fp32_smallk", 32, 128),
    ("bf_fp32_heap_k10_d128", "bf.fp32_heap", "_BF32_HEAP_SRC", "bf_fp32_heap", 10, 128),
    ("bf_fp32_k10_d96", "bf.fp32", "_BF32_SRC", "bf_fp32", 10, 96),
]

LAUNCHER = r"""
// ---- host launcher (not from the reference): the runner's launch shape ----
#include <cuda_runtime.h>
extern "C" __attribute__((visibility("default")))
int ref_launch(const float* Q, const float* X, int* out_ids, float* out_dists,
               int n, int m, void* stream) {
  const int smem = (D_VAL + 2 * BLOCK * K_VAL) * 4;
  cudaError_t e = cudaFuncSetAttribute(%(kernel)s, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  %(kernel)s<<<n, BLOCK, smem, (cudaStream_t)stream>>>(Q, X, out_ids, out_dists, m);
  return (int)cudaGetLastError();
}
extern "C" __attribute__((visibility("default"))) int ref_block() { return BLOCK; }
"""


def _choose_block(k: int, d: int) -> int:
    # the reference's heuristic, bf/fp32.py:212-221 (needed before import, for naming)
    limit = 47 * 1024
    reg_cap = max(32, 65536 // max(64, d + k + 10))
    for b in [128, 64, 32, 256, 512]:
        if b > reg_cap:
            continue
        if (d + 2 * b * k) * 4 < limit:
            return b
    return 32


def load_reference_sources(ref: str) -> dict:
    """Import the reference's bf modules with a stub cupy; return their kernel strings."""
    stub = types.ModuleType("cupy")
    stub.ndarray = object
    saved = {k: sys.modules.get(k) for k in ("cupy", "bf", "bf.fp32", "bf.fp32_heap")}
    sys.modules["cupy"] = stub
    sys.path.insert(0, ref)
    try:
        for k in ("bf", "bf.fp32", "bf.fp32_heap"):
            sys.modules.pop(k, None)
        mods = {name: importlib.import_module(name) for name in ("bf.fp32", "bf.fp32_heap")}
        return {(mod, const): getattr(mods[mod], const)
                for _, mod, const, _, _, _ in INSTANCES}
    finally:
        sys.path.remove(ref)
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def build(ref: str, force: bool = False) -> list[str]:
    if not os.path.isdir(os.path.join(ref, "bf")):
        raise FileNotFoundError(f"reference checkout not found at {ref}")
    os.makedirs(OUT, exist_ok=True)
    srcs = load_reference_sources(ref)
    built = []
    manifest = {}
    for inst, mod, const, kname, k, d in INSTANCES:
        block = _choose_block(k, d)
        code = srcs[(mod, const)]
        for key, val in (("K", k), ("D", d), ("BLOCK", block)):
            code = code.replace(f"__{key}__", str(val))
        code += LAUNCHER % {"kernel": kname}
        cu = os.path.join(OUT, f"ref_{inst}.cu")
        so = os.path.join(OUT, f"ref_{inst}.so")
        with open(cu, "w") as f:
            f.write(code)
        if force or not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(cu):
            cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared",
                   "-Xcompiler", "-fPIC", "-cudart", "static", cu, "-o", so]
            subprocess.run(cmd, check=True)
        manifest[inst] = {"kernel": kname, "k": k, "d": d, "block": block,
                          "shared_mem": (d + 2 * block * k) * 4, "module": mod}
        built.append(so)
    with open(os.path.join(OUT, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return built


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--ref", default=reference_dir(),
                    help=f"reference checkout (default: ${REF_ENV})")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    if not a.ref:
        ap.error(f"name the reference checkout with --ref or ${REF_ENV}")
    for p in build(a.ref, a.force):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
