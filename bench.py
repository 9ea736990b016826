#!/usr/bin/env python3
"""Exact FP32 brute-force k-NN benchmark: queries/sec and fraction of roofline.

    python bench.py [--gpus N --steps K --warmup W] [--workload unit-10m]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --impl reference      # the CPU baseline arm

A step is one exact k-NN search of the whole query batch against the whole
database: on N GPUs the database is row-sharded, each rank searches its shard
(sharing per-query distance bounds with the other ranks after every filter level,
one all-reduce of 2n floats), one NCCL all-gather moves the per-shard (n, k)
lists and the merge kernel produces the result on every rank.  `value` is queries/sec of the whole job
(the query batch / the max over ranks of the device-timed step).  Inputs are
synthetic (seeded, the workload's shapes and distributions), resident in HBM
when timing starts.  When a GPU's inputs are larger than L2 the steps run back to
back; when L2 could hold them, a 256 MB buffer is written before every step and
each step is timed alone.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from gpu_algo_b200 import data  # noqa: E402
from gpu_algo_b200.sharded import shard_range  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
DEFAULT_WORKLOAD = "unit-10m"
# published queries/sec for a workload's exact shape (other hardware): the reference's best
# run at 1M rows, d=8, k=1, 128k queries, on an RTX 5090 (the q16 query-group variant,
# bf/5090_results/bf_fp32_variant_repeat_over_n_d8_k1_full.json:1772)
PUBLISHED_QPS = {("published-d8", 1_000_000, 128_000, 8, 1): 607_025.0}
# DRAM bytes read per database row by one main-filter launch, keyed by (workload, queries,
# d, k): ncu dram__bytes_read.sum of the launch over all rows of a 3,000,000-row sample
# (1.213 GB / 3M rows), CTA pairs.  Its writes are the candidate appends, 8 bytes each
# (0.323 GB for the sample's 35.8M candidates, 9.0 B each with write granularity).
TRAFFIC_READ_PER_ROW = {("unit-10m", 10_000, 128, 100): 404}
TRAFFIC_WRITE_PER_CANDIDATE = 9.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(data.WORKLOADS))
    ap.add_argument("--k", type=int, default=None, help="default: the workload's first k")
    ap.add_argument("--rows", type=int, default=None, help="override the database size")
    ap.add_argument("--queries", type=int, default=None, help="override the query count")
    ap.add_argument("--engine", default="auto", choices=["auto", "direct", "tc_f16"])
    ap.add_argument("--cta-pair", action="store_true",
                    help="TC engine: force CTA pairs (tcgen05.mma.cta_group::2)")
    ap.add_argument("--single-cta", action="store_true",
                    help="TC engine: no CTA pairs (by default the engine picks)")
    ap.add_argument("--prepared", action="store_true",
                    help="index use: the rows' TC form is prepared once, outside the timed "
                         "steps (bfk_prepare); the default step converts them every time")
    ap.add_argument("--cpu-sample", type=int, default=32,
                    help="queries in the bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--phases", action="store_true",
                    help="after the timed steps, time one more step phase by phase (CUDA "
                         "events at each phase boundary; the max over ranks is reported)")
    return ap.parse_args(argv)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.err = None
        self.lines = []
        self.reader = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line)

    def start(self):
        """Starts sampling every 100 ms and returns once the first sample is in (up to
        2 s), so that a timed region shorter than the interval still has the sample
        taken as it begins, under the warm-up's load."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception as e:  # nvidia-smi missing
            self.err = str(e)
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        t_end = time.monotonic() + 2.0
        while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
            time.sleep(0.005)

    def stop(self) -> dict:
        if self.proc is None:
            return {"unavailable": self.err or "nvidia-smi not started"}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            self.proc.wait()
        self.reader.join(timeout=5)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"unavailable": "no samples"}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax),
                "reasons": sorted(reasons), "samples": len(sm)}


def roofline_of(engine_name: str, queries: int, rows: int, d: int, main_ms: float,
                peaks: dict) -> dict:
    """The dominant kernel's roofline for one launch on one GPU.

    Its algorithmic work is 2*Q*N_shard*d flops and the rows it must read: f16 for the
    tensor-core filter, FP32 for the SIMT engines.  Its bound is whichever of the two takes
    longer at the measured peaks; the SIMT engines stream the database and are taken as
    HBM-bound.  `achieved` is that work over the launch's CUDA-event time."""
    flops = 2.0 * queries * rows * d
    tc = engine_name == "tc_f16"
    kbytes = float(rows * d * (2 if tc else 4))
    t_tensor = flops / (peaks["bf16_tflops"] * 1e12)
    t_hbm = kbytes / (peaks["hbm_gbs"] * 1e9)
    bound = "tensor" if tc and t_tensor >= t_hbm else "hbm"
    main_s = main_ms / 1e3 if main_ms > 0 else None
    if bound == "tensor":
        achieved = flops / main_s / 1e12 if main_s else None
        peak, unit, peak_kind = peaks["bf16_tflops"], "TFLOP/s", "dense bf16 (burst)"
        algorithmic = "2*Q*N_shard*d flops per launch"
    else:
        achieved = kbytes / main_s / 1e9 if main_s else None
        peak, unit, peak_kind = peaks["hbm_gbs"], "GB/s", "HBM copy"
        algorithmic = (f"N_shard*d*{2 if tc else 4} bytes per launch "
                       f"({'f16' if tc else 'FP32'} rows read once)")
    return {"bound": bound, "kernel": engine_name, "achieved": achieved, "peak": peak,
            "unit": unit, "frac": (achieved / peak) if achieved else None,
            "peak_source": f"{peaks['source']} {peak_kind}", "main_kernel_ms": main_ms,
            "algorithmic": algorithmic, "flops_per_launch": flops, "bytes_per_launch": kbytes}


def gen_workload(name, rank, world, rows, queries):
    w = data.WORKLOADS[name]
    N = rows or w["N"]
    Qn = queries or w["Q"]
    cs = w["db_seed"] if w["kind"] == "mixture" else None
    r0, r1 = shard_range(N, rank, world)
    X = data.generate(w["kind"], w["db_seed"], w["d"], r0, r1, centre_seed=cs)
    Q = data.generate(w["kind"], w["q_seed"], w["d"], 0, Qn, centre_seed=cs)
    return w, N, Qn, r0, r1, X, Q


def cpu_baseline(X, Q, k, sample, steps=1):
    """The NumPy/OpenBLAS restatement timed on this host (the CPU baseline).

    BLAS runs on every core this process may use, whatever OMP_NUM_THREADS the
    launcher set (torch.distributed.run sets it to 1); returns the per-step times
    and the BLAS thread count in effect."""
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import numpy_knn
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    times = []
    with threadpool_limits(limits=cores, user_api="blas"):
        blas = [p["num_threads"] for p in threadpool_info() if p.get("user_api") == "blas"]
        threads = max(blas) if blas else 1
        for s in range(steps):
            q0 = (s * sample) % max(1, Q.shape[0] - sample + 1)
            t = time.perf_counter()
            numpy_knn(Q[q0:q0 + sample], X, k)
            times.append(time.perf_counter() - t)
    return times, threads


L2_BYTES = 126 * 1024 * 1024        # B200 L2
L2_FLUSH_BYTES = 256 * 1024 * 1024  # written before each timed step when the inputs fit in L2


def l2_resident(N, Qn, d, world=1) -> bool:
    """Whether one GPU's inputs (its rows and the queries, in FP32) could sit in L2."""
    return (-(-N // world) + Qn) * d * 4 <= 2 * L2_BYTES


def bench_config(a, N, Qn, d, k):
    """The workload description both arms print (the same dict for the same run)."""
    if l2_resident(N, Qn, d, a.gpus):
        l2 = (f"inputs fit in L2 (database {N * d * 4 / 1e9:.3f} GB): {L2_FLUSH_BYTES >> 20} MB "
              "written before each timed step, which is timed alone")
    else:
        l2 = f"inputs larger than L2 (database {N * d * 4 / 1e9:.2f} GB), no flush"
    return {"workload": a.workload, "N": N, "Q": Qn, "d": d, "k": k,
            "parallelism": f"rowshard{a.gpus}", "rows_prepared_once": bool(a.prepared),
            "l2": l2}


def run_reference(a):
    """--impl reference: the reference path has no CPU implementation of its own,
    so the arm times the oracle's NumPy restatement of it on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    w, N, Qn, r0, r1, X, Q = gen_workload(a.workload, 0, 1, a.rows, a.queries)
    k = a.k or w["ks"][0]
    sample = min(a.cpu_sample, Qn)
    cpu_baseline(X, Q, k, sample, steps=a.warmup)
    times, cores = cpu_baseline(X, Q, k, sample, steps=a.steps)
    ms = 1e3 * sum(times) / len(times)
    qps = sample / (ms / 1e3)
    line = {
        "impl": "reference",
        "metric": "queries/sec, exact FP32 k-NN",
        "value": qps, "unit": "queries/s", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(a, N, Qn, w["d"], k),
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{sample} queries per step against the full {N}-row database "
                                   "(NumPy/OpenBLAS blocked GEMM + argpartition)"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    a = parse_args(argv)
    if a.impl == "reference":
        return run_reference(a)

    import torch
    import torch.distributed as dist
    from gpu_algo_b200 import engine
    from gpu_algo_b200.sharded import sharded_search

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.gpus != world and world > 1:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=device)

    w, N, Qn, r0, r1, X, Q = gen_workload(a.workload, rank, world, a.rows, a.queries)
    k = a.k or w["ks"][0]
    d = w["d"]
    Xd = torch.from_numpy(X).to(device)
    Qd = torch.from_numpy(Q).to(device)
    torch.cuda.synchronize()

    # inputs that L2 could hold are evicted before every timed step
    flush = (torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)
             if l2_resident(N, Qn, d, world) else None)

    # every rank plans its sampling levels for the largest shard
    plan_rows = shard_range(N, 0, world)[1] - shard_range(N, 0, world)[0]

    prepared = engine.PreparedRows.prepare(Xd) if a.prepared else None

    cta_pair = True if a.cta_pair else (False if a.single_cta else None)

    def step(time_main=False, Q_=None, on_phase=None):
        return sharded_search(Qd if Q_ is None else Q_, Xd, k, r0, plan_rows=plan_rows,
                              engine=a.engine, time_main=time_main, cta_pair=cta_pair,
                              prepared=prepared, on_phase=on_phase)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    # the stats calls pass the search's own plan options (same workspace size)
    stat_opts = dict(engine=a.engine, plan_rows=plan_rows if world > 1 else 0,
                     shards=world if world > 1 else 0, prepared=a.prepared, cta_pair=cta_pair)
    engine.last_stats(Qd, Xd, k, **stat_opts)  # clear timing records
    # the sampler starts first: its start waits for the first sample, for a time that
    # differs between ranks, and the barrier after it lines the ranks up again so that
    # no rank's timed steps wait on a rank still starting its sampler
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    if flush is None:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(a.steps):
            step(time_main=True)
        ev1.record()
        torch.cuda.synchronize()
        t_ms = ev0.elapsed_time(ev1) / a.steps
    else:
        # the inputs fit in L2: each step is timed alone, after a write of a buffer
        # larger than L2 has evicted them
        evs = []
        for _ in range(a.steps):
            flush.zero_()
            e_a = torch.cuda.Event(enable_timing=True)
            e_b = torch.cuda.Event(enable_timing=True)
            e_a.record()
            step(time_main=True)
            e_b.record()
            evs.append((e_a, e_b))
        torch.cuda.synchronize()
        t_ms = sum(x.elapsed_time(y) for x, y in evs) / a.steps
    barrier()
    clocks = sampler.stop()
    stats = engine.last_stats(Qd, Xd, k, **stat_opts)
    main_ms = stats["main_kernel_ms"] / max(1, stats["timed_calls"])
    tt = torch.tensor([t_ms, main_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    t_max, main_max = float(tt[0]), float(tt[1])
    value = Qn / (t_max / 1e3)

    phases = None
    if a.phases:
        marks = []

        def mark(name):
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            marks.append((name, ev))

        barrier()
        step(on_phase=mark)
        torch.cuda.synchronize()
        spans = [(f"{marks[i - 1][0]} -> {marks[i][0]}", marks[i - 1][1].elapsed_time(marks[i][1]))
                 for i in range(1, len(marks))]
        tp = torch.tensor([ms for _, ms in spans], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tp, op=dist.ReduceOp.MAX)
        phases = {name: round(float(ms), 4) for (name, _), ms in zip(spans, tp.tolist())}

    # end to end through the public API with host buffers: queries H2D from pinned
    # memory, search, (dists, ids) D2H into pinned memory, every step
    e2e = None
    if not a.no_e2e:
        Qh = torch.from_numpy(Q).pin_memory()
        Qd2 = torch.empty_like(Qd)
        out_d = torch.empty((Qn, k), dtype=torch.float32).pin_memory()
        out_i = torch.empty((Qn, k), dtype=torch.int32).pin_memory()

        def e2e_step():
            Qd2.copy_(Qh, non_blocking=True)
            dd, ii = step(Q_=Qd2)
            out_d.copy_(dd, non_blocking=True)
            out_i.copy_(ii, non_blocking=True)

        for _ in range(max(1, a.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        te = torch.tensor([e0.elapsed_time(e1) / a.steps], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": Qn / (float(te[0]) / 1e3), "unit": "queries/s",
               "h2d_bytes_per_step": Qn * d * 4, "d2h_bytes_per_step": Qn * k * 8,
               "note": "database resident in HBM (an index); queries uploaded and results "
                       "downloaded every step"}

    peaks = load_peaks()
    m_shard = r1 - r0
    # DRAM bytes of one main-filter launch, from an ncu capture of a smaller case of the
    # same workload: the reads scale with the rows (the f16 rows, fetched again by some of
    # the query tiles), the writes with the candidates the launch appended
    traffic = None
    per_row = TRAFFIC_READ_PER_ROW.get((a.workload, Qn, d, k))
    if per_row is not None and stats["engine"] == "tc_f16":
        traffic = per_row * m_shard + TRAFFIC_WRITE_PER_CANDIDATE * stats["candidates"]
    roofline = roofline_of(stats["engine"], Qn, m_shard, d, main_max, peaks)
    roofline.update({
        "traffic": traffic,
        "traffic_source": (f"ncu dram__bytes of a 3M-row sample: {per_row} B read per row x "
                           f"{m_shard} rows + {TRAFFIC_WRITE_PER_CANDIDATE} B written per "
                           f"candidate x {stats['candidates']}") if traffic else None,
        "db_bytes_per_launch": m_shard * d * 4,
    })
    launches = stats["kernel_launches"] + (1 if world > 1 else 0)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        sample = min(a.cpu_sample, Qn)
        times, cores = cpu_baseline(X, Q, k, sample, steps=1)
        cpu = {"value": sample / times[0], "unit": "queries/s", "cores": cores, "kind": "port",
               "sample": f"{sample} queries against the full {N}-row database "
                         "(NumPy/OpenBLAS blocked GEMM + argpartition, all host threads)"}

    if rank == 0:
        line = {
            "metric": "queries/sec, exact FP32 k-NN",
            "value": value,
            "unit": "queries/s",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": t_max,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": (value / PUBLISHED_QPS[(a.workload, N, Qn, d, k)]
                            if (a.workload, N, Qn, d, k) in PUBLISHED_QPS else None),
            "dtype": "f32",
            "data": "synthetic",
            "config": bench_config(a, N, Qn, d, k),
            "engine": stats["engine"],
            "cta_pair": stats["cta_pair"],
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches * a.steps,
            "clocks": clocks,
            "phases_ms_max_over_ranks": phases,
            "search_stats": {kk: stats[kk] for kk in ("candidates", "max_query_candidates",
                                                       "survivors", "fallback_queries", "slices")},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
