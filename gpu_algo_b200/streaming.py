"""Out-of-core search: a database in host memory, larger than the GPU's, streamed
through it in row chunks.

The reference's tiled runner splits the database into row tiles and merges their
partial lists (bf/fp32_tiled.py:182-239); here the tiles live in host memory and
cross PCIe while the previous tile is searched:

* two device buffers of `chunk_rows` rows; the copy of chunk c+1 (on its own
  stream, from pinned memory) overlaps the search of chunk c;
* every chunk is an ordinary exact search with `id_offset` = its first row, and
  the running top-k is merged with it (`bfk_merge`);
* the running k-th distance bounds the final one, so it is handed to the next
  chunk's filter levels through the engine's level hook: later chunks keep only
  rows that can still enter the top k.

    python -m gpu_algo_b200.streaming --rows 20000000 --d 128 --queries 10000 --k 100
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np
import torch

from . import engine

PAD_DIST = np.float32(3.402823e38)


def _bound_from_running(run_d: torch.Tensor, qn2_low: torch.Tensor, k: int) -> torch.Tensor:
    """Per query, an upper bound on (k-th distance - ||q||^2) from the running lists:
    their k-th distance D is a real row's exact distance, so the final k-th is <= D.
    ||q||^2 is taken from below (qn2_low) and the difference rounded up, so the bound
    holds for the engine's FP32 ||q||^2 too.  +inf while the list holds padding."""
    dk = run_d[:, k - 1].double()
    b = dk - qn2_low
    b = b + b.abs() * 2.0 ** -22 + 1e-30  # above the float32 rounding of the difference
    b = torch.where(dk >= float(PAD_DIST), torch.full_like(b, float("inf")), b)
    return b.float()


def streamed_search(Q, X_host: torch.Tensor, k: int, *, chunk_rows: int = 1 << 21,
                    engine_name: str = "auto", share_bound: bool = True):
    """Exact k-NN of Q (device, (n, d) float32) against X_host ((m, d) float32 in host
    memory, pinned for overlap).  Returns device (dists, ids), sorted by (distance, index)."""
    Q = engine.as_device_f32(Q, "Q")
    if not isinstance(X_host, torch.Tensor) or X_host.is_cuda or X_host.dtype != torch.float32:
        raise TypeError("X_host must be a float32 torch tensor in host memory")
    if X_host.dim() != 2 or X_host.shape[1] != Q.shape[1]:
        raise ValueError(f"X_host must be (m, {Q.shape[1]}), got {tuple(X_host.shape)}")
    X_host = X_host.contiguous()
    n, d = Q.shape
    m = X_host.shape[0]
    k = int(k)
    if k <= 0:
        raise ValueError("k must be positive")
    dev = Q.device
    run_d = torch.full((n, k), float(PAD_DIST), dtype=torch.float32, device=dev)
    run_i = torch.full((n, k), -1, dtype=torch.int32, device=dev)
    if m == 0 or n == 0:
        return run_d, run_i
    chunk_rows = max(1, min(int(chunk_rows), m))
    # ||q||^2 from below: the FP32 sum of d squares rounds by less than (d + 2) 2^-24
    qn2 = Q.double().pow(2).sum(1)
    qn2_low = qn2 * (1.0 - (d + 2) * 2.0 ** -23)
    with torch.cuda.device(dev):
        compute = torch.cuda.current_stream()
        copier = torch.cuda.Stream()
        bufs = [torch.empty((chunk_rows, d), dtype=torch.float32, device=dev) for _ in range(2)]
        copied = [torch.cuda.Event() for _ in range(2)]
        used = [None, None]
        chunks = [(r0, min(r0 + chunk_rows, m)) for r0 in range(0, m, chunk_rows)]

        def issue_copy(c):
            b = c % 2
            r0, r1 = chunks[c]
            with torch.cuda.stream(copier):
                if used[b] is not None:
                    copier.wait_event(used[b])  # the search of chunk c-2 is done with it
                bufs[b][: r1 - r0].copy_(X_host[r0:r1], non_blocking=True)
                copied[b].record(copier)

        issue_copy(0)
        for c, (r0, r1) in enumerate(chunks):
            if c + 1 < len(chunks):
                issue_copy(c + 1)
            b = c % 2
            compute.wait_event(copied[b])
            hook = None
            if share_bound and c > 0:
                bound = _bound_from_running(run_d, qn2_low, k)

                def hook(t, bound=bound):
                    torch.minimum(t, bound, out=t)
            d_, i_ = engine.search(Q, bufs[b][: r1 - r0], k, engine=engine_name, id_offset=r0,
                                   bound_hook=hook)
            ev = torch.cuda.Event()
            ev.record(compute)
            used[b] = ev
            run_d, run_i = engine.merge(torch.stack([run_d, d_]), torch.stack([run_i, i_]), k)
    return run_d, run_i


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Measure the out-of-core search (synthetic "
                                             "normal data in pinned host memory).")
    ap.add_argument("--rows", type=int, default=20_000_000)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--queries", type=int, default=10_000)
    ap.add_argument("--k", type=int, default=100)
    ap.add_argument("--chunk-rows", type=int, default=1 << 21)
    ap.add_argument("--repeats", type=int, default=2)
    a = ap.parse_args(argv)
    from . import data
    X = torch.from_numpy(data.generate("normal", 12, a.d, 0, a.rows)).pin_memory()
    Q = torch.from_numpy(data.generate("normal", 13, a.d, 0, a.queries)).cuda()
    streamed_search(Q, X[: min(a.rows, a.chunk_rows * 2)], a.k, chunk_rows=a.chunk_rows)  # warm-up
    times = []
    for _ in range(a.repeats):
        torch.cuda.synchronize()
        t = time.perf_counter()
        streamed_search(Q, X, a.k, chunk_rows=a.chunk_rows)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t)
    best = min(times)
    print(json.dumps({"rows": a.rows, "d": a.d, "queries": a.queries, "k": a.k,
                      "chunk_rows": a.chunk_rows, "seconds": best,
                      "queries_per_second": a.queries / best,
                      "host_to_device_GBps": a.rows * a.d * 4 / best / 1e9}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
