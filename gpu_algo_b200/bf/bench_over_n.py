#!/usr/bin/env python3
"""Drop-in for bf/bench_fp32_variant_repeat_over_n.py: the repeated variant study
over n at fixed k, writing the same JSON payload (``meta`` / ``results`` /
``failures``, bf/bench_fp32_variant_repeat_over_n.py:165-184), so the reference's
plot scripts read its output unchanged.

    python -m gpu_algo_b200.bf.bench_over_n --m 1000000 --d 8 --k 1 \\
        --n-values 1000,16000,128000 --out-json over_n.json

The arguments and their defaults are the reference's.  Two differences:
* the data comes from NumPy's PCG64 seeded with ``--seed`` (the reference draws
  from CuPy's generator, which is not available here), Gaussian rows and queries
  as in the reference, or clustered queries built the same way;
* every variant runs this package's runner of the same name; they return the
  same exact sorted results (the engine is chosen per shape).
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import numpy as np

VARIANT_NAMES = ("baseline", "heap", "q2", "q4", "q8", "q16", "q32", "q64", "q128")


def variants_table():
    """Variant name -> runner(Q, X, k, reps), as in the reference's VARIANTS."""
    from .fp32 import run_bf_fp32
    from .fp32_heap import run_bf_fp32_heap
    from .fp32_q2 import run_bf_fp32_q2
    from .fp32_qgroup import run_bf_fp32_qgroup
    table = {
        "baseline": lambda Q, X, k, reps: run_bf_fp32(Q, X, k, reps=reps),
        "heap": lambda Q, X, k, reps: run_bf_fp32_heap(Q, X, k, reps=reps),
        "q2": lambda Q, X, k, reps: run_bf_fp32_q2(Q, X, k, reps=reps),
    }
    for g in (4, 8, 16, 32, 64, 128):
        table[f"q{g}"] = (lambda qpb: lambda Q, X, k, reps: run_bf_fp32_qgroup(Q, X, k, qpb=qpb,
                                                                               reps=reps))(g)
    return table


def parse_csv_ints(raw: str) -> list[int]:
    values = [int(part.strip()) for part in raw.split(",") if part.strip()]
    if not values:
        raise ValueError("Need at least one integer value")
    return values


def parse_variants(raw: str) -> list[str]:
    values = [part.strip() for part in raw.split(",") if part.strip()]
    if not values:
        raise ValueError("Need at least one variant")
    bad = [v for v in values if v not in VARIANT_NAMES]
    if bad:
        raise ValueError(f"Unknown variants: {bad}")
    return values


def mean_std(values: list[float]) -> tuple[float, float]:
    mean = sum(values) / len(values)
    var = sum((v - mean) ** 2 for v in values) / len(values)
    return mean, math.sqrt(var)


def make_data(seed: int, m: int, d: int, max_n: int, mode: str, cluster_size: int,
              cluster_noise: float) -> tuple[np.ndarray, np.ndarray]:
    """Rows, then queries, from one PCG64 stream (the reference's order)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    X = rng.standard_normal((m, d), dtype=np.float32)
    if mode == "gaussian":
        Q = rng.standard_normal((max_n, d), dtype=np.float32)
    elif mode == "clustered":
        if cluster_size <= 0:
            raise ValueError("cluster_size must be positive")
        groups = (max_n + cluster_size - 1) // cluster_size
        centers = rng.standard_normal((groups, d), dtype=np.float32)
        noise = rng.standard_normal((max_n, d), dtype=np.float32) * np.float32(cluster_noise)
        Q = centers[np.arange(max_n) // cluster_size] + noise
    else:
        raise ValueError(f"Unknown query mode: {mode}")
    return X, Q


def result_row(variant: str, args, n: int, trial_ms: list[float], block: int) -> dict:
    """One ``results`` entry, with the reference's keys and formulas."""
    mean_ms, std_ms = mean_std(trial_ms)
    mean_qps = n / (mean_ms * 1e-3)
    std_qps = 0.0 if mean_ms == 0 else (n * std_ms) / ((mean_ms ** 2) * 1e-3)
    return {
        "variant": variant,
        "distribution": args.query_mode,
        "m": args.m,
        "d": args.d,
        "n": n,
        "k": args.k,
        "trials": args.trials,
        "reps": args.reps,
        "trial_query_ms": trial_ms,
        "mean_query_ms": mean_ms,
        "std_query_ms": std_ms,
        "mean_queries_per_second": mean_qps,
        "std_queries_per_second": std_qps,
        "block": int(block),
    }


def make_payload(args, n_values: list[int], variants: list[str], rows: list[dict],
                 failures: list[dict]) -> dict:
    return {
        "meta": {
            "m": args.m,
            "d": args.d,
            "k": args.k,
            "seed": args.seed,
            "trials": args.trials,
            "reps": args.reps,
            "skip_failures": bool(args.skip_failures),
            "query_mode": args.query_mode,
            "cluster_size": args.cluster_size,
            "cluster_noise": args.cluster_noise,
            "n_values": n_values,
            "variants": variants,
        },
        "results": rows,
        "failures": failures,
    }


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="Repeated BF-FP32 variant study over n at fixed k.")
    ap.add_argument("--m", type=int, default=1_000_000)
    ap.add_argument("--d", type=int, default=8)
    ap.add_argument("--n-values", type=str, default="1000,2000,4000,8000,16000")
    ap.add_argument("--k", type=int, default=1)
    ap.add_argument("--variants", type=str, default=",".join(VARIANT_NAMES))
    ap.add_argument("--trials", type=int, default=20)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--query-mode", type=str, default="gaussian", choices=["gaussian", "clustered"])
    ap.add_argument("--cluster-size", type=int, default=16)
    ap.add_argument("--cluster-noise", type=float, default=0.05)
    ap.add_argument("--skip-failures", action="store_true")
    ap.add_argument("--out-json", type=str, default="bf_fp32_variant_repeat_over_n_d8_k1.json")
    return ap


def main(argv=None) -> None:
    import torch
    args = build_parser().parse_args(argv)
    n_values = parse_csv_ints(args.n_values)
    variants = parse_variants(args.variants)
    table = variants_table()
    X, Q = make_data(args.seed, args.m, args.d, max(n_values), args.query_mode,
                     args.cluster_size, args.cluster_noise)
    X_gpu = torch.from_numpy(X).cuda()
    Q_full = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    rows: list[dict] = []
    failures: list[dict] = []
    print(f"BF-FP32 repeated variant study over n | m={args.m:,} d={args.d} k={args.k} "
          f"n_values={n_values} variants={variants} trials={args.trials}")
    for variant in variants:
        print(f"\n[{variant}]")
        runner = table[variant]
        for n in n_values:
            Q_gpu = Q_full[:n]
            trial_ms = []
            last = None
            try:
                for _ in range(args.trials):
                    last = runner(Q_gpu, X_gpu, args.k, args.reps)
                    trial_ms.append(float(last["ms"]))
            except Exception as exc:  # recorded like the reference's --skip-failures
                msg = f"{type(exc).__name__}: {exc}"
                if not args.skip_failures:
                    raise
                failures.append({"variant": variant, "n": n, "k": args.k, "error": msg})
                print(f"  n={n:>6}  FAILED  {msg}")
                continue
            row = result_row(variant, args, n, trial_ms, last["block"])
            rows.append(row)
            print(f"  n={n:>6}  mean={row['mean_query_ms']:9.3f} ms  "
                  f"std={row['std_query_ms']:7.3f} ms  "
                  f"qps={row['mean_queries_per_second']:9.0f} +/- "
                  f"{row['std_queries_per_second']:7.0f}  block={row['block']}")
    out_path = Path(args.out_json)
    out_path.write_text(json.dumps(make_payload(args, n_values, variants, rows, failures),
                                   indent=2) + "\n", encoding="ascii")
    print(f"\nWrote {out_path}")


if __name__ == "__main__":
    main()
