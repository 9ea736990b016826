"""Device-side search API over torch CUDA tensors (PyTorch is only the buffer).

``search(Q, X, k)`` is the call every ``bf`` runner makes: Q (n, d) and X
(m, d) float32 CUDA tensors (or any object with ``__cuda_array_interface__``,
e.g. a CuPy array, wrapped without a copy) -> (dists (n, k) float32,
ids (n, k) int32) on the same device, sorted ascending by (distance, index).
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from . import _lib

_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def as_device_f32(a, name: str) -> torch.Tensor:
    """Zero-copy view of a CUDA float32 array as a contiguous torch tensor."""
    if not isinstance(a, torch.Tensor):
        if hasattr(a, "__cuda_array_interface__"):
            a = torch.as_tensor(a, device="cuda")
        else:
            raise TypeError(f"{name} must be a CUDA array (torch tensor or __cuda_array_interface__)")
    if not a.is_cuda:
        raise TypeError(f"{name} must live on a CUDA device")
    if a.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {a.dtype}")
    if a.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(a.shape)}")
    return a.contiguous()


def workspace(nbytes: int, device: torch.device, stream: torch.cuda.Stream | None = None
              ) -> torch.Tensor:
    """A cached, grow-only device workspace (one per device and stream)."""
    dev = device.index if device.index is not None else torch.cuda.current_device()
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    key = (dev, s.cuda_stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=f"cuda:{dev}")
            _ws_cache[key] = buf
        return buf


def workspace_size(n: int, m: int, d: int, k: int, opts: _lib.Opts) -> int:
    nb = ctypes.c_uint64()
    _lib.check(_lib.load().bfk_workspace_size(n, m, d, k, ctypes.byref(opts), ctypes.byref(nb)),
               "bfk_workspace_size")
    return int(nb.value)


class _DeviceArray:
    """A raw device float32 vector exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def _pair_flags(cta_pair) -> int:
    """cta_pair: True forces CTA pairs, False single CTAs, None the engine's default."""
    if cta_pair is None:
        return 0
    return _lib.FLAG_CTA_PAIR if cta_pair else _lib.FLAG_SINGLE_CTA


def search(Q, X, k: int, *, engine: str = "auto", slices: int = 0, max_candidates: int = 0,
           id_offset: int = 0, out: tuple[torch.Tensor, torch.Tensor] | None = None,
           ws: torch.Tensor | None = None, time_main: bool = False, cta_pair: bool | None = None,
           bound_hook=None, plan_rows: int = 0, shards: int = 0, prepared=None):
    """Exact k-NN on the GPU.  Returns (dists, ids) device tensors.

    ``bound_hook(t)``, if given, is called by the tensor-core engine after each
    filter level with ``t``, a float32 CUDA tensor of per-query bounds that it
    may lower in place (a sharded search takes the minimum over shards): (n,)
    values, or (2n,) when ``shards`` > 1 (the number of shards in that minimum;
    see ``bfk_level_hook_t``).  ``plan_rows`` makes shards of one search plan
    the same levels.  ``prepared`` (a ``PreparedRows`` of this X) skips the
    conversion of the rows.
    """
    Q = as_device_f32(Q, "Q")
    X = as_device_f32(X, "X")
    n, d = Q.shape
    m = X.shape[0]
    if X.shape[1] != d:
        raise ValueError(f"Q has d={d} but X has d={X.shape[1]}")
    if Q.device != X.device:
        raise ValueError("Q and X must be on the same device")
    k = int(k)
    if k <= 0:
        raise ValueError("k must be positive")
    lib = _lib.load()
    opts = _lib.make_opts(engine, slices, max_candidates,
                          (_lib.FLAG_TIME_MAIN if time_main else 0) |
                          _pair_flags(cta_pair))
    opts.plan_rows = int(plan_rows)
    opts.shards = int(shards)
    if prepared is not None:
        if prepared.shape != (m, d) or prepared.buffer.device != X.device:
            raise ValueError(f"prepared rows are {prepared.shape} on {prepared.buffer.device}, "
                             f"X is {(m, d)} on {X.device}")
        opts.flags |= _lib.FLAG_PREPARED
    hook_error = []
    if bound_hook is not None:
        def _hook(ptr, count, user, stream_ptr):
            try:
                bound_hook(torch.as_tensor(_DeviceArray(ptr, count), device=Q.device))
            except BaseException as exc:  # re-raised after the search returns
                hook_error.append(exc)
        c_hook = _lib.LEVEL_HOOK(_hook)
        opts.level_hook = c_hook
    with torch.cuda.device(Q.device):
        stream = torch.cuda.current_stream()
        if out is None:
            dists = torch.empty((n, k), dtype=torch.float32, device=Q.device)
            ids = torch.empty((n, k), dtype=torch.int32, device=Q.device)
        else:
            dists, ids = out
        nbytes = workspace_size(n, m, d, k, opts)
        if ws is None:
            ws = workspace(nbytes, Q.device, stream)
        elif ws.numel() < nbytes:
            raise ValueError(f"workspace needs {nbytes} bytes, got {ws.numel()}")
        if prepared is None:
            st = lib.bfk_search(Q.data_ptr(), n, X.data_ptr() if m else None, m, d, k,
                                int(id_offset), dists.data_ptr(), ids.data_ptr(), ws.data_ptr(),
                                ws.numel(), ctypes.byref(opts),
                                ctypes.c_void_p(stream.cuda_stream))
        else:
            st = lib.bfk_search_prepared(Q.data_ptr(), n, X.data_ptr() if m else None,
                                         prepared.buffer.data_ptr(), m, d, k, int(id_offset),
                                         dists.data_ptr(), ids.data_ptr(), ws.data_ptr(),
                                         ws.numel(), ctypes.byref(opts),
                                         ctypes.c_void_p(stream.cuda_stream))
        if hook_error:
            raise hook_error[0]
        _lib.check(st, "bfk_search")
    return dists, ids


class PreparedRows:
    """The tensor-core engine's form of one database X (``bfk_prepare``): f16 rows in
    64-row groups scaled by powers of two, ||x||^2 and the group scales.  A search with
    ``prepared=`` skips that conversion; it still reads X for the exact re-rank.

    ``save(path)`` writes the buffer's bytes (a 512-byte header that records m and d,
    then the arrays); ``load(path, device)`` reads them back.  The library rejects a
    buffer made for another (m, d).
    """

    def __init__(self, buffer: torch.Tensor, shape: tuple[int, int]):
        self.buffer = buffer
        self.shape = (int(shape[0]), int(shape[1]))

    @staticmethod
    def nbytes(m: int, d: int) -> int:
        nb = ctypes.c_uint64()
        _lib.check(_lib.load().bfk_prepared_size(int(m), int(d), ctypes.byref(nb)),
                   "bfk_prepared_size")
        return int(nb.value)

    @classmethod
    def prepare(cls, X) -> "PreparedRows":
        X = as_device_f32(X, "X")
        m, d = X.shape
        with torch.cuda.device(X.device):
            stream = torch.cuda.current_stream()
            nb = cls.nbytes(m, d)
            buf = torch.empty(nb, dtype=torch.uint8, device=X.device)
            _lib.check(_lib.load().bfk_prepare(X.data_ptr() if m else None, m, d,
                                               buf.data_ptr(), nb,
                                               ctypes.c_void_p(stream.cuda_stream)),
                       "bfk_prepare")
        return cls(buf, (m, d))

    def save(self, path) -> None:
        header = np.array([self.shape[0], self.shape[1]], dtype=np.int64)
        with open(path, "wb") as f:
            f.write(b"BFKROWS1")
            f.write(header.tobytes())
            f.write(self.buffer.cpu().numpy().tobytes())

    @classmethod
    def load(cls, path, device) -> "PreparedRows":
        with open(path, "rb") as f:
            if f.read(8) != b"BFKROWS1":
                raise ValueError(f"{path} is not a prepared-rows file")
            m, d = (int(v) for v in np.frombuffer(f.read(16), dtype=np.int64))
            data = np.frombuffer(f.read(), dtype=np.uint8)
        if data.size != cls.nbytes(m, d):
            raise ValueError(f"{path}: {data.size} bytes, expected {cls.nbytes(m, d)}")
        return cls(torch.from_numpy(data.copy()).to(device), (m, d))


def last_stats(Q, X, k: int, *, engine: str = "auto", slices: int = 0,
               max_candidates: int = 0, plan_rows: int = 0, shards: int = 0,
               prepared: bool = False, cta_pair: bool | None = None) -> dict:
    """Statistics of the last search of this shape on the current stream's workspace
    (pass the search's own engine options)."""
    Q = as_device_f32(Q, "Q")
    X = as_device_f32(X, "X")
    n, d = Q.shape
    m = X.shape[0]
    opts = _lib.make_opts(engine, slices, max_candidates, _pair_flags(cta_pair))
    opts.plan_rows = int(plan_rows)
    opts.shards = int(shards)
    if prepared:
        opts.flags |= _lib.FLAG_PREPARED
    with torch.cuda.device(Q.device):
        stream = torch.cuda.current_stream()
        ws = workspace(workspace_size(n, m, d, k, opts), Q.device, stream)
        s = _lib.Stats()
        _lib.check(_lib.load().bfk_search_stats(ws.data_ptr(), n, m, d, k, ctypes.byref(opts),
                                                ctypes.c_void_p(stream.cuda_stream),
                                                ctypes.byref(s)), "bfk_search_stats")
    return {
        "engine": _lib.ENGINE_NAMES.get(s.engine_used, s.engine_used),
        "fallback_queries": s.fallback_queries,
        "candidates": s.candidates,
        "max_query_candidates": s.max_query_candidates,
        "slices": s.slices,
        "survivors": s.survivors,
        "device_error": s.device_error,
        "kernel_launches": s.kernel_launches,
        "timed_calls": s.timed_calls,
        "main_kernel_ms": s.main_kernel_ms,
        "cta_pair": bool(s.cta_pair),
    }


def plan_info(n: int, m: int, d: int, k: int, *, engine: str = "auto", slices: int = 0,
              max_candidates: int = 0, plan_rows: int = 0, shards: int = 0,
              prepared: bool = False, cta_pair: bool | None = None) -> dict:
    """The plan a search of this shape would run (computed on the host, no GPU): the
    engine, and for the tensor-core engine its levels (tiles and slices of each), its
    CTA-pair choice and candidate pool."""
    opts = _lib.make_opts(engine, slices, max_candidates, _pair_flags(cta_pair))
    opts.plan_rows = int(plan_rows)
    opts.shards = int(shards)
    if prepared:
        opts.flags |= _lib.FLAG_PREPARED
    info = _lib.PlanInfo()
    _lib.check(_lib.load().bfk_plan_info(int(n), int(m), int(d), int(k), ctypes.byref(opts),
                                         ctypes.byref(info)), "bfk_plan_info")
    lv = info.levels
    return {"engine": _lib.ENGINE_NAMES.get(info.engine, info.engine),
            "cta_pair": bool(info.cta_pair), "levels": lv, "q_tiles": info.q_tiles,
            "cand_cap": info.cand_cap, "level_tiles": list(info.level_tiles[:lv]),
            "level_slices": list(info.level_slices[:lv])}


def merge(cand_d: torch.Tensor, cand_i: torch.Tensor, k: int):
    """Merge (lists, n, k) sorted candidate lists into the k best per query."""
    if cand_d.dim() != 3 or cand_d.shape != cand_i.shape:
        raise ValueError("candidates must be (lists, n, k) distance/index pairs")
    if cand_d.dtype != torch.float32 or cand_i.dtype != torch.int32:
        raise TypeError("candidates must be float32 distances and int32 indices")
    lists, n, kk = cand_d.shape
    if kk != k:
        raise ValueError("list length must equal k")
    cand_d = cand_d.contiguous()
    cand_i = cand_i.contiguous()
    with torch.cuda.device(cand_d.device):
        stream = torch.cuda.current_stream()
        out_d = torch.empty((n, k), dtype=torch.float32, device=cand_d.device)
        out_i = torch.empty((n, k), dtype=torch.int32, device=cand_d.device)
        _lib.check(_lib.load().bfk_merge(cand_d.data_ptr(), cand_i.data_ptr(), n, lists, k,
                                         out_d.data_ptr(), out_i.data_ptr(),
                                         ctypes.c_void_p(stream.cuda_stream)), "bfk_merge")
    return out_d, out_i


def _attrs_dict(a: "_lib.Attrs") -> dict:
    return {
        "num_regs": a.num_regs,
        "shared_size_bytes": a.shared_size_bytes + a.dynamic_smem_bytes,
        "local_size_bytes": a.local_size_bytes,
        "const_size_bytes": a.const_size_bytes,
        "max_threads_per_block": a.max_threads_per_block,
        "binary_version": a.binary_version,
        "ptx_version": a.ptx_version,
        "block_threads": a.block_threads,
        "dynamic_smem_bytes": a.dynamic_smem_bytes,
    }


def merge_packed(blocks: torch.Tensor, k: int):
    """Merge gathered (lists, 2, n, k) int32 blocks -- list l's distance bits in
    [l, 0], its ids in [l, 1] -- into the k best per query, read in place."""
    if blocks.dim() != 4 or blocks.shape[1] != 2 or blocks.dtype != torch.int32:
        raise ValueError("blocks must be (lists, 2, n, k) int32")
    lists, _, n, kk = blocks.shape
    if kk != k:
        raise ValueError("list length must equal k")
    blocks = blocks.contiguous()
    with torch.cuda.device(blocks.device):
        stream = torch.cuda.current_stream()
        out_d = torch.empty((n, k), dtype=torch.float32, device=blocks.device)
        out_i = torch.empty((n, k), dtype=torch.int32, device=blocks.device)
        base = blocks.data_ptr()
        _lib.check(_lib.load().bfk_merge_strided(base, base + 4 * n * k, n, lists, 2 * n * k, k,
                                                 out_d.data_ptr(), out_i.data_ptr(),
                                                 ctypes.c_void_p(stream.cuda_stream)),
                   "bfk_merge_strided")
    return out_d, out_i


def kernel_attrs(engine: str, d: int, k: int) -> dict:
    """Attributes of the main kernel an engine launches for (d, k)."""
    a = _lib.Attrs()
    _lib.check(_lib.load().bfk_kernel_attrs(_lib.ENGINES[engine], d, k, ctypes.byref(a)),
               "bfk_kernel_attrs")
    return _attrs_dict(a)


def merge_attrs(lists: int, k: int) -> dict:
    """Attributes of the kernel ``merge`` launches for ``lists`` lists of k."""
    a = _lib.Attrs()
    _lib.check(_lib.load().bfk_merge_attrs(int(lists), int(k), ctypes.byref(a)),
               "bfk_merge_attrs")
    return _attrs_dict(a)


def filter_values(Q, X) -> tuple[torch.Tensor, torch.Tensor, bool]:
    """The tensor-core filter's value of every (query, row) pair (``bfk_filter_values``).

    Returns (v (n, m), qinfo (n, 2) = (||q||^2 in FP32, margin), exact_only), v as the
    filter computes ||x||^2 - 2 q.x, NaN where it reported none.  Test infrastructure
    for the engine's error margin: every pair must satisfy
    |(||q||^2 + v) - D| <= margin, D the reference distance."""
    Q = as_device_f32(Q, "Q")
    X = as_device_f32(X, "X")
    n, d = Q.shape
    m = X.shape[0]
    if X.shape[1] != d:
        raise ValueError(f"Q has d={d} but X has d={X.shape[1]}")
    lib = _lib.load()
    nb = ctypes.c_uint64()
    _lib.check(lib.bfk_filter_values_workspace(n, m, d, ctypes.byref(nb)),
               "bfk_filter_values_workspace")
    with torch.cuda.device(Q.device):
        stream = torch.cuda.current_stream()
        ws = torch.empty(int(nb.value), dtype=torch.uint8, device=Q.device)
        v = torch.empty((n, m), dtype=torch.float32, device=Q.device)
        qinfo = torch.empty((n, 2), dtype=torch.float32, device=Q.device)
        eo = ctypes.c_int32()
        _lib.check(lib.bfk_filter_values(Q.data_ptr(), n, X.data_ptr(), m, d, v.data_ptr(),
                                         qinfo.data_ptr(), ctypes.byref(eo), ws.data_ptr(),
                                         ws.numel(), ctypes.c_void_p(stream.cuda_stream)),
                   "bfk_filter_values")
    return v, qinfo, bool(eo.value)
