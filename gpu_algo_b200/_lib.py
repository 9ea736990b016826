"""ctypes binding to ``libbfknn.so`` (the C ABI declared in include/bfknn.h).

The library is built in-tree by ``gpu_algo_b200.build``.  There is no CPU or
Python fallback: if the shared library is missing or a call fails, an
exception is raised.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbfknn.so")

ENGINE_AUTO = 0
ENGINE_DIRECT = 1
ENGINE_TC_F16 = 2
ENGINES = {"auto": ENGINE_AUTO, "direct": ENGINE_DIRECT, "tc_f16": ENGINE_TC_F16}
ENGINE_NAMES = {v: k for k, v in ENGINES.items()}

STATUS = {
    0: "BFK_OK",
    1: "BFK_ERR_INVALID_ARGUMENT",
    2: "BFK_ERR_UNSUPPORTED",
    3: "BFK_ERR_WORKSPACE",
    4: "BFK_ERR_CUDA",
    5: "BFK_ERR_DEVICE_TIMEOUT",
    6: "BFK_ERR_NO_DEVICE",
}

# every entry point include/bfknn.h declares
EXPORTS = (
    "bfk_version",
    "bfk_status_string",
    "bfk_last_error",
    "bfk_workspace_size",
    "bfk_search",
    "bfk_merge",
    "bfk_merge_strided",
    "bfk_kernel_attrs",
    "bfk_merge_attrs",
    "bfk_filter_values_workspace",
    "bfk_filter_values",
    "bfk_search_stats",
    "bfk_plan_info",
    "bfk_search_noalloc",
    "bfk_prepared_size",
    "bfk_prepare",
    "bfk_search_prepared",
)


LEVEL_HOOK = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                              ctypes.c_void_p)


class Opts(ctypes.Structure):
    _fields_ = [("engine", ctypes.c_int32), ("slices", ctypes.c_int32),
                ("max_candidates", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("shards", ctypes.c_int32), ("reserved", ctypes.c_int32 * 3), ("level_hook", LEVEL_HOOK),
                ("hook_user", ctypes.c_void_p), ("plan_rows", ctypes.c_int64)]


class Attrs(ctypes.Structure):
    _fields_ = [("num_regs", ctypes.c_int32), ("shared_size_bytes", ctypes.c_int32),
                ("dynamic_smem_bytes", ctypes.c_int32), ("local_size_bytes", ctypes.c_int32),
                ("const_size_bytes", ctypes.c_int32), ("max_threads_per_block", ctypes.c_int32),
                ("binary_version", ctypes.c_int32), ("ptx_version", ctypes.c_int32),
                ("block_threads", ctypes.c_int32), ("reserved", ctypes.c_int32 * 7)]


class Stats(ctypes.Structure):
    _fields_ = [("engine_used", ctypes.c_int32), ("fallback_queries", ctypes.c_int32),
                ("candidates", ctypes.c_int64), ("max_query_candidates", ctypes.c_int32),
                ("slices", ctypes.c_int32), ("survivors", ctypes.c_int64),
                ("device_error", ctypes.c_int32), ("kernel_launches", ctypes.c_int32),
                ("timed_calls", ctypes.c_int32), ("main_kernel_ms", ctypes.c_float),
                ("cta_pair", ctypes.c_int32), ("reserved", ctypes.c_int32 * 1)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("engine", ctypes.c_int32), ("cta_pair", ctypes.c_int32),
                ("levels", ctypes.c_int32), ("q_tiles", ctypes.c_int32),
                ("cand_cap", ctypes.c_int32), ("reserved0", ctypes.c_int32),
                ("level_tiles", ctypes.c_int64 * 6), ("level_slices", ctypes.c_int32 * 6)]


class BfkError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        msg = f"{what}: {STATUS.get(status, status)} ({status_string(status)})"
        if status == 4:
            try:
                msg += f" [{load().bfk_last_error().decode()}]"
            except Exception:  # pragma: no cover
                pass
        super().__init__(msg)


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the in-tree library; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m gpu_algo_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        i32, i64, u64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p
        i32p = ctypes.POINTER(i32)
        lib.bfk_version.restype = i32
        lib.bfk_version.argtypes = [i32p, i32p]
        lib.bfk_status_string.restype = ctypes.c_char_p
        lib.bfk_status_string.argtypes = [i32]
        lib.bfk_last_error.restype = ctypes.c_char_p
        lib.bfk_last_error.argtypes = []
        lib.bfk_workspace_size.restype = i32
        lib.bfk_workspace_size.argtypes = [i64, i64, i32, i32, ctypes.POINTER(Opts),
                                           ctypes.POINTER(u64)]
        lib.bfk_search.restype = i32
        lib.bfk_search.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, vp, u64,
                                   ctypes.POINTER(Opts), vp]
        lib.bfk_merge.restype = i32
        lib.bfk_merge.argtypes = [vp, vp, i64, i32, i32, vp, vp, vp]
        lib.bfk_merge_strided.restype = i32
        lib.bfk_merge_strided.argtypes = [vp, vp, i64, i32, i64, i32, vp, vp, vp]
        lib.bfk_kernel_attrs.restype = i32
        lib.bfk_kernel_attrs.argtypes = [i32, i32, i32, ctypes.POINTER(Attrs)]
        lib.bfk_merge_attrs.restype = i32
        lib.bfk_merge_attrs.argtypes = [i32, i32, ctypes.POINTER(Attrs)]
        lib.bfk_filter_values_workspace.restype = i32
        lib.bfk_filter_values_workspace.argtypes = [i64, i64, i32, ctypes.POINTER(u64)]
        lib.bfk_filter_values.restype = i32
        lib.bfk_filter_values.argtypes = [vp, i64, vp, i64, i32, vp, vp, i32p, vp, u64, vp]
        lib.bfk_prepared_size.restype = i32
        lib.bfk_prepared_size.argtypes = [i64, i32, ctypes.POINTER(u64)]
        lib.bfk_prepare.restype = i32
        lib.bfk_prepare.argtypes = [vp, i64, i32, vp, u64, vp]
        lib.bfk_search_prepared.restype = i32
        lib.bfk_search_prepared.argtypes = [vp, i64, vp, vp, i64, i32, i32, i64, vp, vp, vp, u64,
                                            ctypes.POINTER(Opts), vp]
        lib.bfk_search_noalloc.restype = i32
        lib.bfk_search_noalloc.argtypes = [vp, i64, vp, i64, i32, i32, i64, vp, vp, vp]
        lib.bfk_search_stats.restype = i32
        lib.bfk_search_stats.argtypes = [vp, i64, i64, i32, i32, ctypes.POINTER(Opts), vp,
                                         ctypes.POINTER(Stats)]
        lib.bfk_plan_info.restype = i32
        lib.bfk_plan_info.argtypes = [i64, i64, i32, i32, ctypes.POINTER(Opts),
                                      ctypes.POINTER(PlanInfo)]
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().bfk_status_string(status).decode()
    except Exception:  # pragma: no cover - only while the library is unavailable
        return "?"


def check(status: int, what: str) -> None:
    if status != 0:
        raise BfkError(status, what)


FLAG_TIME_MAIN = 1
FLAG_CTA_PAIR = 2
FLAG_PREPARED = 4
FLAG_SINGLE_CTA = 8


def make_opts(engine: str | int = "auto", slices: int = 0, max_candidates: int = 0,
              flags: int = 0) -> Opts:
    o = Opts()
    o.engine = ENGINES[engine] if isinstance(engine, str) else int(engine)
    o.slices = int(slices)
    o.max_candidates = int(max_candidates)
    o.flags = int(flags)
    return o


def version() -> tuple[int, int]:
    a, b = ctypes.c_int32(), ctypes.c_int32()
    check(load().bfk_version(ctypes.byref(a), ctypes.byref(b)), "bfk_version")
    return a.value, b.value
