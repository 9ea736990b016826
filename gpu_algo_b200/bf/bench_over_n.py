#!/usr/bin/env python3
"""Variant study over the query count n, writing the reference's result payload.

The reference publishes its only numbers as JSON files written by
bf/bench_fp32_variant_repeat_over_n.py, and its plot script
bf/plot_fp32_variant_repeat_over_n.py reads them (``meta`` m/d/k/trials; per row
variant, n, mean_queries_per_second, std_queries_per_second).  This study takes
the same command-line flags with the same defaults and writes a payload with the
same keys (``meta``, ``results``, ``failures``), so that plot script reads its
output unchanged:

    python -m gpu_algo_b200.bf.bench_over_n --m 1000000 --d 8 --k 1 \\
        --n-values 1000,16000,128000 --out-json over_n.json

Everything else is this package's own:
* data: NumPy PCG64 seeded with ``--seed``, rows then queries from one stream
  (the reference draws from CuPy's generator, which is not installed here);
  ``clustered`` queries are noisy copies of shared centres;
* every variant name runs this package's runner of that name, and all of them
  return the same exact, sorted top-k;
* throughput per (variant, n) is n over the mean trial time; its spread is the
  mean time's spread carried through q = n / t to first order, which is the
  quantity the published files report;
* each row also carries the search's roofline, max(2 n m d / tensor peak,
  m d 4 / HBM bandwidth) at the measured peaks of MEASURED_PEAKS.json when the
  working directory or the repository holds one (else fixed fallback figures),
  and the mean time's fraction of it; the plot script ignores these keys.
"""
from __future__ import annotations

import argparse
import itertools
import json
import os
import statistics
import sys
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

VARIANT_NAMES = ("baseline", "heap", "q2", "q4", "q8", "q16", "q32", "q64", "q128")
QGROUP_SIZES = {f"q{g}": g for g in (4, 8, 16, 32, 64, 128)}

# (flag, type, default, help): the reference study's flags and defaults
_FLAGS = (
    ("--m", int, 1_000_000, "database rows"),
    ("--d", int, 8, "dimensions"),
    ("--n-values", str, "1000,2000,4000,8000,16000", "query counts, comma separated"),
    ("--k", int, 1, "neighbours per query"),
    ("--variants", str, ",".join(VARIANT_NAMES), "runner names, comma separated"),
    ("--trials", int, 20, "timed trials per (variant, n)"),
    ("--reps", int, 5, "searches per trial (the runner's reps)"),
    ("--seed", int, 42, "PCG64 seed of the data"),
    ("--cluster-size", int, 16, "clustered queries: queries per centre"),
    ("--cluster-noise", float, 0.05, "clustered queries: noise scale around a centre"),
    ("--out-json", str, "bf_fp32_variant_repeat_over_n_d8_k1.json", "where to write the payload"),
)


# used when no MEASURED_PEAKS.json is found: an HBM copy rate and a dense bf16 GEMM rate
# measured earlier on B200s
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_peaks(paths=None) -> dict:
    """The measured HBM (GB/s) and dense bf16 (TFLOP/s) peaks, from the first
    MEASURED_PEAKS.json among `paths` (default: the working directory, then the
    repository root), else FALLBACK_PEAKS."""
    if paths is None:
        root = Path(__file__).resolve().parents[2]
        paths = [Path("MEASURED_PEAKS.json"), root / "MEASURED_PEAKS.json"]
    for p in paths:
        if os.path.exists(p):
            with open(p, encoding="utf-8") as f:
                j = json.load(f)
            return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
                    "source": "measured"}
    return dict(FALLBACK_PEAKS)


def roofline(n: int, m: int, d: int, peaks: dict) -> tuple[float, str]:
    """(ms, bound) of one search of n queries over m rows of d dimensions: the longer of
    the algorithmic flops at the tensor peak and the FP32 rows at HBM bandwidth."""
    t_flops = 2.0 * n * m * d / (peaks["bf16_tflops"] * 1e12)
    t_bytes = 4.0 * m * d / (peaks["hbm_gbs"] * 1e9)
    return (max(t_flops, t_bytes) * 1e3, "tensor" if t_flops >= t_bytes else "hbm")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(
        description="Exact k-NN runner variants timed over a range of query counts; writes the "
                    "reference's over-n JSON payload.")
    for flag, typ, default, text in _FLAGS:
        ap.add_argument(flag, type=typ, default=default, help=f"{text} (default {default})")
    ap.add_argument("--query-mode", default="gaussian", choices=("gaussian", "clustered"),
                    help="query distribution (default gaussian)")
    ap.add_argument("--skip-failures", action="store_true",
                    help="record a failing (variant, n) in 'failures' and go on")
    return ap


def _split(raw: str, what: str, convert) -> list:
    items = [convert(tok) for tok in (t.strip() for t in raw.split(",")) if tok]
    if not items:
        raise ValueError(f"{what}: the list is empty")
    return items


def n_values_of(raw: str) -> list[int]:
    return _split(raw, "--n-values", int)


def variants_of(raw: str) -> list[str]:
    names = _split(raw, "--variants", str)
    unknown = sorted(set(names) - set(VARIANT_NAMES))
    if unknown:
        raise ValueError(f"--variants: no runner named {', '.join(unknown)} "
                         f"(choose from {', '.join(VARIANT_NAMES)})")
    return names


def runner_for(variant: str):
    """The package runner behind a variant name: f(Q, X, k, reps) -> result dict."""
    from . import fp32, fp32_heap, fp32_q2, fp32_qgroup
    if variant == "baseline":
        return lambda Q, X, k, reps: fp32.run_bf_fp32(Q, X, k, reps=reps)
    if variant == "heap":
        return lambda Q, X, k, reps: fp32_heap.run_bf_fp32_heap(Q, X, k, reps=reps)
    if variant == "q2":
        return lambda Q, X, k, reps: fp32_q2.run_bf_fp32_q2(Q, X, k, reps=reps)
    g = QGROUP_SIZES[variant]
    return lambda Q, X, k, reps: fp32_qgroup.run_bf_fp32_qgroup(Q, X, k, qpb=g, reps=reps)


def synthetic_data(seed: int, m: int, d: int, n_max: int, query_mode: str = "gaussian",
                   cluster_size: int = 16, cluster_noise: float = 0.05):
    """(X (m, d), Q (n_max, d)) float32: standard normal rows, then the queries."""
    gen = np.random.default_rng(np.random.PCG64(seed))
    X = gen.standard_normal((m, d), dtype=np.float32)
    if query_mode == "gaussian":
        return X, gen.standard_normal((n_max, d), dtype=np.float32)
    if query_mode != "clustered":
        raise ValueError(f"query mode {query_mode!r} is neither gaussian nor clustered")
    if cluster_size <= 0:
        raise ValueError("cluster size must be at least 1")
    centres = gen.standard_normal((-(-n_max // cluster_size), d), dtype=np.float32)
    owner = np.repeat(np.arange(centres.shape[0]), cluster_size)[:n_max]
    jitter = gen.standard_normal((n_max, d), dtype=np.float32) * np.float32(cluster_noise)
    return X, np.ascontiguousarray(centres[owner] + jitter)


@dataclass
class Cell:
    """The timed trials of one (variant, n)."""
    variant: str
    n: int
    trial_ms: list[float] = field(default_factory=list)
    block: int = 0

    def summary(self, args, peaks: dict | None = None) -> dict:
        """The payload row: the reference's keys, then the roofline keys."""
        mean_ms = statistics.fmean(self.trial_ms)
        sd_ms = statistics.pstdev(self.trial_ms)
        qps = self.n / (mean_ms / 1e3)
        # q = n / t, so dq = q * dt / t to first order
        sd_qps = qps * sd_ms / mean_ms if mean_ms > 0 else 0.0
        peaks = peaks or load_peaks()
        roof_ms, bound = roofline(self.n, args.m, args.d, peaks)
        return dict(variant=self.variant, distribution=args.query_mode, m=args.m, d=args.d,
                    n=self.n, k=args.k, trials=args.trials, reps=args.reps,
                    trial_query_ms=list(self.trial_ms), mean_query_ms=mean_ms,
                    std_query_ms=sd_ms, mean_queries_per_second=qps,
                    std_queries_per_second=sd_qps, block=int(self.block),
                    roofline_ms=roof_ms, roofline_bound=bound,
                    roofline_fraction=roof_ms / mean_ms if mean_ms > 0 else None,
                    roofline_peaks=peaks["source"])


def payload(args, n_values: list[int], variants: list[str], rows: list[dict],
            failures: list[dict]) -> dict:
    meta = {key: getattr(args, key) for key in
            ("m", "d", "k", "seed", "trials", "reps", "query_mode", "cluster_size",
             "cluster_noise")}
    meta.update(skip_failures=bool(args.skip_failures), n_values=list(n_values),
                variants=list(variants))
    return {"meta": meta, "results": rows, "failures": failures}


def run_study(args, log=print) -> dict:
    import torch
    n_values = n_values_of(args.n_values)
    variants = variants_of(args.variants)
    X, Q = synthetic_data(args.seed, args.m, args.d, max(n_values), args.query_mode,
                          args.cluster_size, args.cluster_noise)
    Xd = torch.from_numpy(X).cuda()
    Qd = torch.from_numpy(Q).cuda()
    rows, failures = [], []
    peaks = load_peaks()
    log(f"# over-n study: m={args.m} d={args.d} k={args.k} trials={args.trials} "
        f"reps={args.reps} queries={args.query_mode}")
    log(f"# {'variant':>8} {'n':>8} {'ms':>10} {'+-':>8} {'queries/s':>12} {'+-':>10}")
    for variant, n in itertools.product(variants, n_values):
        run = runner_for(variant)
        cell = Cell(variant, n)
        try:
            for _ in range(args.trials):
                res = run(Qd[:n], Xd, args.k, args.reps)
                cell.trial_ms.append(float(res["ms"]))
                cell.block = int(res["block"])
        except Exception as exc:  # noqa: BLE001 -- recorded, or re-raised below
            if not args.skip_failures:
                raise
            failures.append({"variant": variant, "n": n, "k": args.k,
                             "error": f"{type(exc).__name__}: {exc}"})
            log(f"  {variant:>8} {n:>8} failed: {exc}")
            continue
        row = cell.summary(args, peaks)
        rows.append(row)
        log(f"  {variant:>8} {n:>8} {row['mean_query_ms']:10.4f} {row['std_query_ms']:8.4f} "
            f"{row['mean_queries_per_second']:12.0f} {row['std_queries_per_second']:10.0f}")
    return payload(args, n_values, variants, rows, failures)


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    out = run_study(args)
    Path(args.out_json).write_text(json.dumps(out, indent=2) + "\n", encoding="ascii")
    print(f"# payload: {args.out_json}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
