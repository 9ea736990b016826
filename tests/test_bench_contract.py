"""bench.py's reference arm on CPU: one JSON line with the keys the driver reads, on
rank 0 only; the other ranks exit 0 without work."""
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
        "--workload", "plumbing", "--steps", "2", "--warmup", "1", "--cpu-sample", "8"]


def _run(rank: str):
    env = dict(os.environ, RANK=rank)
    return subprocess.run(ARGS, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    p = _run("0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    j = json.loads(lines[0])
    assert j["impl"] == "reference"
    assert j["metric"] == "queries/sec, exact FP32 k-NN" and j["unit"] == "queries/s"
    assert j["value"] > 0 and j["ms_per_step"] > 0 and j["higher_is_better"] is True
    assert (j["steps"], j["warmup"], j["n_gpus"]) == (2, 1, 1)
    # the same config dict the repository arm prints for this run
    assert j["config"] == {"workload": "plumbing", "N": 65_536, "Q": 1_024, "d": 128, "k": 10,
                           "parallelism": "rowshard1", "rows_prepared_once": False,
                           "l2": "inputs fit in L2 (database 0.034 GB): 256 MB written before "
                                 "each timed step, which is timed alone"}
    cb = j["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == j["value"]
    assert "8 queries" in cb["sample"]
    assert j["e2e"] == {"value": j["value"], "unit": "queries/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_no_work():
    p = _run("1")
    assert p.returncode == 0 and p.stdout.strip() == ""


def test_clock_sampler_reads_clocks_and_active_reasons(tmp_path, monkeypatch):
    """The clock record comes from `nvidia-smi --query-gpu ... -lms`; a stand-in script
    prints three samples, one with sw_power_cap active."""
    fake = tmp_path / "nvidia-smi"
    fake.write_text(
        "#!/bin/sh\n"
        "echo '0, 1800, 1965, 700.5, 0x4, Not Active, Not Active, Not Active, Active'\n"
        "echo '0, 1900, 1965, 710.0, 0x0, Not Active, Not Active, Not Active, Not Active'\n"
        "echo '0, 1850, 1965, 705.0, 0x0, Not Active, Not Active, Not Active, Not Active'\n"
        "exec sleep 30\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    import bench  # the repository root is on sys.path (conftest)
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.5)
    assert s.stop() == {"sm_mhz": 1850.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                        "samples": 3}


def test_clock_sampler_has_a_sample_for_a_short_timed_region(tmp_path, monkeypatch):
    """start() returns only once the first sample is in, so a timed region shorter than
    the sampling interval still has one."""
    fake = tmp_path / "nvidia-smi"
    fake.write_text(
        "#!/bin/sh\n"
        "sleep 0.3\n"
        "echo '0, 1965, 1965, 650.0, 0x0, Not Active, Not Active, Not Active, Not Active'\n"
        "exec sleep 30\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    import bench
    s = bench.ClockSampler(0)
    s.start()
    assert s.stop() == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 1}


def test_roofline_bound_follows_the_workload():
    """Tensor-bound for the 10M-row tensor-core filter at Q = 10k; HBM-bound for a 128-query
    filter over 12.5M rows (f16 rows read once) and for the SIMT scan (FP32 rows)."""
    import bench
    peaks = {"bf16_tflops": 1649.3, "hbm_gbs": 6554.6, "source": "measured"}
    r = bench.roofline_of("tc_f16", 10_000, 10_000_000, 128, 25.0, peaks)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert abs(r["achieved"] - 2 * 10_000 * 10_000_000 * 128 / 25e-3 / 1e12) < 1e-6
    r = bench.roofline_of("tc_f16", 128, 12_500_000, 96, 0.87, peaks)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert abs(r["achieved"] - 12_500_000 * 96 * 2 / 0.87e-3 / 1e9) < 1e-6
    r = bench.roofline_of("direct", 1, 12_500_000, 96, 1.0, peaks)
    assert r["bound"] == "hbm" and abs(r["frac"] - 4.8 / 6.5546) < 1e-3
    assert bench.roofline_of("direct", 1, 10, 8, 0.0, peaks)["achieved"] is None
