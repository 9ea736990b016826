"""Drop-in for bf/fp32.py: the BF-FP32 runner and the helpers the other
runners import (compile_kernel, choose_block, tms, kernel_attrs).

Reference: bf/fp32.py:196-289.  Differences, by design:
* there is no JIT -- the kernels are compiled ahead of time for sm_100a into
  ``libbfknn.so``; ``compile_kernel`` returns a handle to the precompiled
  engine instead of a ``cupy.RawKernel`` (bf/fp32.py:200-209);
* results are exact top-k sorted by (distance, index); ``run_*`` also return
  the distances under ``"dists"`` (the reference leaves them on the device);
* inputs are torch CUDA tensors or any ``__cuda_array_interface__`` array
  (CuPy arrays are wrapped without a copy).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import engine as _engine

_KERN_CACHE: dict = {}
_KERNEL_SRC_VERSION = 1

# reference kernel name -> engine it maps to ("auto" picks per shape)
_NAME_TO_ENGINE = {
    "bf_fp32": "auto",
    "bf_fp32_smallk": "auto",
    "bf_fp32_heap": "auto",
    "bf_fp32_tiled_partial": "auto",
    "bf_fp32_tiled_merge": "auto",
    "bf_fp32_qgroup_partial": "auto",
    "bf_fp32_qgroup_merge": "auto",
    "bf_fp32_q2": "auto",
}


class CompiledKernel:
    """Handle to a precompiled engine; stands in for ``cupy.RawKernel``."""

    def __init__(self, name: str, subs: dict):
        self.name = name
        self.subs = dict(subs)
        self.engine = _NAME_TO_ENGINE.get(name, "auto")

    @property
    def attributes(self) -> dict:
        k = int(self.subs.get("K", 10))
        d = int(self.subs.get("D", 128))
        eng = "direct" if self.engine == "auto" else self.engine
        return _engine.kernel_attrs(eng, d, k)


def compile_kernel(src: str, name: str, subs: dict) -> CompiledKernel:
    """Return the precompiled engine for (name, subs); cached like the reference."""
    key = (_KERNEL_SRC_VERSION, name, tuple(sorted(subs.items())))
    kern = _KERN_CACHE.get(key)
    if kern is None:
        kern = CompiledKernel(name, subs)
        _KERN_CACHE[key] = kern
    return kern


def choose_block(k: int, d: int) -> int:
    """The reference's block heuristic (bf/fp32.py:212-221), kept for callers that
    report it; the B200 engines choose their own launch shapes."""
    limit = 47 * 1024
    reg_cap = max(32, 65536 // max(64, d + k + 10))
    for b in [128, 64, 32, 256, 512]:
        if b > reg_cap:
            continue
        if (d + 2 * b * k) * 4 < limit:
            return b
    return 32


def tms(fn, warmup: int = 10, reps: int = 20) -> float:
    """Mean milliseconds per call, CUDA events on the current stream
    (bf/fp32.py:224-235 times on the null stream the same way)."""
    for _ in range(warmup):
        fn()
    torch.cuda.current_stream().synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(reps):
        fn()
    ev1.record()
    ev1.synchronize()
    return float(ev0.elapsed_time(ev1)) / reps


def kernel_attrs(kern: CompiledKernel) -> dict:
    """Kernel attributes (bf/fp32.py:238-249) from cudaFuncGetAttributes."""
    attrs = dict(kern.attributes)
    keys = [
        "num_regs",
        "shared_size_bytes",
        "local_size_bytes",
        "const_size_bytes",
        "max_threads_per_block",
        "binary_version",
        "ptx_version",
    ]
    return {key: int(attrs[key]) for key in keys if key in attrs}


def _make_runner(Q_gpu, X_gpu, k: int, engine: str = "auto", slices: int = 0):
    Q = _engine.as_device_f32(Q_gpu, "Q_gpu")
    X = _engine.as_device_f32(X_gpu, "X_gpu")
    n, d = Q.shape
    m = X.shape[0]
    out_ids = torch.zeros((n, k), dtype=torch.int32, device=Q.device)
    out_dists = torch.zeros((n, k), dtype=torch.float32, device=Q.device)
    opts = _engine._lib.make_opts(engine, slices)
    with torch.cuda.device(Q.device):
        ws = _engine.workspace(_engine.workspace_size(n, m, d, k, opts), Q.device)

    def fn():
        _engine.search(Q, X, k, engine=engine, slices=slices, out=(out_dists, out_ids), ws=ws)

    return Q, X, fn, out_ids, out_dists


def _engine_attrs(Q, X, k, engine: str, slices: int, label: str) -> tuple[int, int, dict]:
    stats = _engine.last_stats(Q, X, k, engine=engine, slices=slices)
    used = stats["engine"]
    attrs = _engine.kernel_attrs(used, Q.shape[1], k)
    block = int(attrs.pop("block_threads"))
    smem = int(attrs.pop("dynamic_smem_bytes"))
    attrs = {key: int(v) for key, v in attrs.items()}
    attrs["kernel_variant"] = used
    attrs["reference_variant"] = label
    return block, smem, attrs


def _merge_report(Q, X, k, engine: str, slices: int, label: str) -> tuple[int, dict]:
    """(merge_shared_mem_bytes, merge_kernel_attrs) of the merge the search really ran.

    The SIMT engine merges its database slices with the kernel of ``bfk_merge``; the
    tensor-core engine and a one-slice search run no merge, which is reported as 0
    bytes and an attribute dict that says so."""
    stats = _engine.last_stats(Q, X, k, engine=engine, slices=slices)
    lists = int(stats["slices"])
    if stats["engine"] != "direct" or lists <= 1:
        return 0, {"kernel_variant": "none", "reference_variant": label,
                   "note": f"the {stats['engine']} engine ran no merge for this search"}
    attrs = _engine.merge_attrs(lists, k)
    smem = int(attrs.pop("dynamic_smem_bytes"))
    attrs.pop("block_threads")
    attrs = {key: int(v) for key, v in attrs.items()}
    attrs["kernel_variant"] = f"merge of {lists} lists"
    attrs["reference_variant"] = label
    return smem, attrs


def build_bf_fp32_runner(Q_gpu, X_gpu, k: int):
    """(fn, out_ids, out_dists, block, shared_mem, attrs) as bf/fp32.py:252-275."""
    Q, X, fn, out_ids, out_dists = _make_runner(Q_gpu, X_gpu, k)
    fn()
    label = "smallk_sorted" if k in {2, 4, 8, 16, 32} else "generic_heap"
    block, smem, attrs = _engine_attrs(Q, X, k, "auto", 0, label)
    return fn, out_ids, out_dists, block, smem, attrs


def _finish(fn, out_ids, out_dists, reps: int) -> tuple[float, np.ndarray, np.ndarray]:
    ms = tms(fn, reps=reps)
    torch.cuda.current_stream().synchronize()
    fn()
    return ms, out_ids.cpu().numpy(), out_dists.cpu().numpy()


def run_bf_fp32(Q_gpu, X_gpu, k: int, reps: int = 10) -> dict:
    """bf/fp32.py:278-289: time the search, return host ids (+ dists)."""
    fn, out_ids, out_dists, block, shared_mem, attrs = build_bf_fp32_runner(Q_gpu, X_gpu, k)
    ms, ids, dists = _finish(fn, out_ids, out_dists, reps)
    return {
        "ids": ids,
        "dists": dists,
        "ms": ms,
        "block": block,
        "shared_mem_bytes": shared_mem,
        "kernel_attrs": attrs,
    }
