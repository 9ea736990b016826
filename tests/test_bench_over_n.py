"""The over-n study CLI writes the reference's JSON payload (no GPU needed).

The key sets are those of bf/bench_fp32_variant_repeat_over_n.py:141-184 and of
its published result files (bf/5090_results/bf_fp32_variant_repeat_over_n_d8_k1_full.json);
bf/plot_fp32_variant_repeat_over_n.py:47-83 reads meta m/d/k/trials and, per row,
variant, n, mean_queries_per_second and std_queries_per_second.
"""
import json

import numpy as np
import pytest

from gpu_algo_b200.bf import bench_over_n as b

RESULT_KEYS = {"variant", "distribution", "m", "d", "n", "k", "trials", "reps", "trial_query_ms",
               "mean_query_ms", "std_query_ms", "mean_queries_per_second",
               "std_queries_per_second", "block"}
META_KEYS = {"m", "d", "k", "seed", "trials", "reps", "skip_failures", "query_mode",
             "cluster_size", "cluster_noise", "n_values", "variants"}


def test_payload_keys_and_formulas():
    args = b.build_parser().parse_args(["--n-values", "1000,2000", "--trials", "3"])
    row = b.result_row("q16", args, 1000, [2.0, 2.0, 4.0], 128)
    assert set(row) == RESULT_KEYS
    mean = 8.0 / 3
    std = float(np.std([2.0, 2.0, 4.0]))
    assert row["mean_query_ms"] == pytest.approx(mean)
    assert row["mean_queries_per_second"] == pytest.approx(1000 / (mean * 1e-3))
    assert row["std_queries_per_second"] == pytest.approx(1000 * std / (mean ** 2 * 1e-3))
    payload = b.make_payload(args, [1000, 2000], ["q16"], [row], [])
    assert set(payload) == {"meta", "results", "failures"}
    assert set(payload["meta"]) == META_KEYS
    json.dumps(payload)  # serialisable as written


def test_arguments_and_data_match_the_reference_defaults():
    args = b.build_parser().parse_args([])
    assert (args.m, args.d, args.k, args.trials, args.reps, args.seed) == (1_000_000, 8, 1, 20, 5, 42)
    assert b.parse_variants(args.variants) == list(b.VARIANT_NAMES)
    with pytest.raises(ValueError):
        b.parse_variants("q3")
    X, Q = b.make_data(42, 100, 8, 40, "clustered", 16, 0.05)
    assert X.shape == (100, 8) and Q.shape == (40, 8) and Q.dtype == np.float32
    # clustered queries: members of a group lie close to their shared centre
    assert np.abs(Q[0] - Q[1]).max() < 1.0
