"""Drop-in replacement for the reference's ``bf`` package (hantaoyu-theory/gpu_algo).

Same modules and entry points as bf/fp32.py, bf/fp32_heap.py, bf/fp32_tiled.py,
bf/fp32_qgroup.py and bf/fp32_q2.py; every runner executes the B200 engine in
``libbfknn.so``.  ``install()`` registers this package under the name ``bf`` so
the reference's own bench CLIs (``python -m bf.bench_fp32 ...``) import it.
"""
import sys


def install() -> None:
    """Make ``import bf`` / ``import bf.fp32`` resolve to this package."""
    from . import fp32, fp32_heap, fp32_tiled, fp32_qgroup, fp32_q2  # noqa: F401
    pkg = sys.modules[__name__]
    sys.modules["bf"] = pkg
    for name in ("fp32", "fp32_heap", "fp32_tiled", "fp32_qgroup", "fp32_q2"):
        sys.modules[f"bf.{name}"] = sys.modules[f"{__name__}.{name}"]
