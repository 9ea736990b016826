"""gpu_algo_b200 -- exact brute-force k-NN on NVIDIA B200 (sm_100a).

A drop-in for the reference's ``bf`` package (hantaoyu-theory/gpu_algo):
``gpu_algo_b200.bf.fp32.run_bf_fp32`` and friends keep the reference's call
surface, and run hand-written sm_100a CUDA through the C ABI in
``include/bfknn.h`` (``libbfknn.so``, loaded with ctypes).

    from gpu_algo_b200 import search
    dists, ids = search(Q, X, k)          # torch CUDA float32 in, device out
"""
from .engine import search, merge, kernel_attrs, last_stats  # noqa: F401

__all__ = ["search", "merge", "kernel_attrs", "last_stats"]
