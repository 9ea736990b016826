"""The over-n study CLI writes the reference's JSON payload (no GPU needed).

The key sets are those of the reference's published result files
(bf/5090_results/bf_fp32_variant_repeat_over_n_d8_k1_full.json, written by
bf/bench_fp32_variant_repeat_over_n.py); bf/plot_fp32_variant_repeat_over_n.py:47-83
reads meta m/d/k/trials and, per row, variant, n, mean_queries_per_second and
std_queries_per_second.
"""
import json

import numpy as np
import pytest

from gpu_algo_b200.bf import bench_over_n as b

REFERENCE_RESULT_KEYS = {"variant", "distribution", "m", "d", "n", "k", "trials", "reps",
                         "trial_query_ms", "mean_query_ms", "std_query_ms",
                         "mean_queries_per_second", "std_queries_per_second", "block"}
RESULT_KEYS = REFERENCE_RESULT_KEYS | {"roofline_ms", "roofline_bound", "roofline_fraction",
                                       "roofline_peaks"}
META_KEYS = {"m", "d", "k", "seed", "trials", "reps", "skip_failures", "query_mode",
             "cluster_size", "cluster_noise", "n_values", "variants"}


def test_payload_keys_and_statistics():
    args = b.build_parser().parse_args(["--n-values", "1000,2000", "--trials", "3"])
    row = b.Cell("q16", 1000, [2.0, 2.0, 4.0], 128).summary(args)
    assert set(row) == RESULT_KEYS
    mean = 8.0 / 3
    sd = float(np.std([2.0, 2.0, 4.0]))
    assert row["mean_query_ms"] == pytest.approx(mean)
    assert row["std_query_ms"] == pytest.approx(sd)
    assert row["mean_queries_per_second"] == pytest.approx(1000 / (mean * 1e-3))
    # the spread of n / t carried to first order from the spread of t
    assert row["std_queries_per_second"] == pytest.approx(1000 * sd / (mean ** 2 * 1e-3))
    out = b.payload(args, [1000, 2000], ["q16"], [row], [])
    assert REFERENCE_RESULT_KEYS <= set(row)  # the keys the reference's plot script reads
    assert set(out) == {"meta", "results", "failures"}
    assert set(out["meta"]) == META_KEYS
    assert out["meta"]["n_values"] == [1000, 2000] and out["meta"]["skip_failures"] is False
    json.dumps(out)  # serialisable as written


def test_flags_defaults_and_data():
    args = b.build_parser().parse_args([])
    assert (args.m, args.d, args.k, args.trials, args.reps, args.seed) == (1_000_000, 8, 1, 20, 5, 42)
    assert args.n_values == "1000,2000,4000,8000,16000" and args.query_mode == "gaussian"
    assert (args.cluster_size, args.cluster_noise) == (16, 0.05)
    assert args.out_json == "bf_fp32_variant_repeat_over_n_d8_k1.json"
    assert b.variants_of(args.variants) == list(b.VARIANT_NAMES)
    assert b.n_values_of(" 5, 7 ,") == [5, 7]
    for bad in ("q3", ""):
        with pytest.raises(ValueError):
            b.variants_of(bad)
    X, Q = b.synthetic_data(42, 100, 8, 40, "clustered", 16, 0.05)
    assert X.shape == (100, 8) and Q.shape == (40, 8) and Q.dtype == np.float32
    # clustered queries: members of a group lie close to their shared centre
    assert np.abs(Q[0] - Q[1]).max() < 1.0
    X2, Q2 = b.synthetic_data(42, 100, 8, 40)
    np.testing.assert_array_equal(X, X2)  # rows come first from the same stream
    with pytest.raises(ValueError):
        b.synthetic_data(42, 10, 8, 4, "uniform")


def test_roofline_fields(tmp_path):
    """Each row's roofline: the 1M x d=8 published shape is HBM-bound for a few hundred
    queries (the rows' 32 MB), tensor-bound above; peaks come from a MEASURED_PEAKS.json
    when one is found, else the fallback figures."""
    peaks = {"hbm_gbs": 8000.0, "bf16_tflops": 1000.0, "source": "measured"}
    ms, bound = b.roofline(100, 1_000_000, 8, peaks)
    assert bound == "hbm" and ms == pytest.approx(4 * 1_000_000 * 8 / 8e12 * 1e3)
    ms, bound = b.roofline(128_000, 1_000_000, 8, peaks)
    assert bound == "tensor" and ms == pytest.approx(2 * 128_000 * 1_000_000 * 8 / 1e15 * 1e3)
    args = b.build_parser().parse_args([])
    row = b.Cell("q16", 128_000, [0.4096], 128).summary(args, peaks)
    assert row["roofline_bound"] == "tensor" and row["roofline_peaks"] == "measured"
    assert row["roofline_fraction"] == pytest.approx(row["roofline_ms"] / 0.4096)
    p = tmp_path / "MEASURED_PEAKS.json"
    p.write_text(json.dumps({"hbm_gbs": 6000.0, "bf16_tflops": 1500.0}))
    assert b.load_peaks([p]) == {"hbm_gbs": 6000.0, "bf16_tflops": 1500.0, "source": "measured"}
    assert b.load_peaks([tmp_path / "absent.json"]) == b.FALLBACK_PEAKS


@pytest.mark.gpu
def test_study_runs_on_the_gpu(tmp_path):
    out = tmp_path / "over_n.json"
    assert b.main(["--m", "20000", "--d", "8", "--n-values", "100,300", "--variants",
                   "baseline,q16", "--trials", "2", "--reps", "1", "--out-json", str(out)]) == 0
    got = json.loads(out.read_text(encoding="ascii"))
    assert [(r["variant"], r["n"]) for r in got["results"]] == [
        ("baseline", 100), ("baseline", 300), ("q16", 100), ("q16", 300)]
    assert all(set(r) == RESULT_KEYS and r["mean_queries_per_second"] > 0
               for r in got["results"])
    assert got["failures"] == []
