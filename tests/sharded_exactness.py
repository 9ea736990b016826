"""Exactness of a row-sharded multi-GPU search at full size, checked against the oracle.

Run with one process per GPU (not collected by pytest; it needs N GPUs):

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        tests/sharded_exactness.py --workload stream-100m --queries 1,16,128 --sample 4

Every rank generates its own shard of the workload's rows (the same seeded chunks
bench.py uses), runs the sharded search for each query count, and then checks a
sample of queries exactly: each rank runs the C oracle (the reference's arithmetic,
bf/fp32.py:74-82) on its own shard for the sampled queries, the per-shard lists are
all-gathered and merged by the oracle's merge, and rank 0 compares the result with
the engine's merged lists bit for bit (distances and ids).  Rank 0 prints one JSON
line per query count.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from gpu_algo_b200 import data  # noqa: E402
from gpu_algo_b200.sharded import shard_range, sharded_search  # noqa: E402
from oracle import oracle_knn, oracle_merge  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--workload", default="stream-100m", choices=sorted(data.WORKLOADS))
    ap.add_argument("--rows", type=int, default=None)
    ap.add_argument("--queries", default=None, help="query counts, comma separated")
    ap.add_argument("--k", type=int, default=None)
    ap.add_argument("--sample", type=int, default=4, help="queries checked per query count")
    a = ap.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    try:
        w = data.WORKLOADS[a.workload]
        N = a.rows or w["N"]
        k = a.k or w["ks"][0]
        counts = [int(v) for v in (a.queries or str(w["Q"])).split(",")]
        cs = w["db_seed"] if w["kind"] == "mixture" else None
        r0, r1 = shard_range(N, rank, world)
        X = data.generate(w["kind"], w["db_seed"], w["d"], r0, r1, centre_seed=cs)
        Xd = torch.from_numpy(X).to(device)
        plan_rows = shard_range(N, 0, world)[1]
        for n in counts:
            Q = data.generate(w["kind"], w["q_seed"], w["d"], 0, n, centre_seed=cs)
            d_, i_ = sharded_search(torch.from_numpy(Q).to(device), Xd, k, r0,
                                    plan_rows=plan_rows)
            torch.cuda.synchronize()
            idx = np.unique(np.linspace(0, n - 1, min(a.sample, n)).astype(np.int64))
            od, oi = oracle_knn(Q[idx], X, k, id_offset=r0)
            part_d = torch.from_numpy(od).to(device)
            part_i = torch.from_numpy(oi).to(device)
            all_d = [torch.empty_like(part_d) for _ in range(world)]
            all_i = [torch.empty_like(part_i) for _ in range(world)]
            dist.all_gather(all_d, part_d)
            dist.all_gather(all_i, part_i)
            if rank == 0:
                ed, ei = oracle_merge(np.stack([t.cpu().numpy() for t in all_d]),
                                      np.stack([t.cpu().numpy() for t in all_i]), k)
                got_d = d_.cpu().numpy()[idx]
                got_i = i_.cpu().numpy()[idx]
                print(json.dumps({"workload": a.workload, "N": N, "Q": n, "k": k,
                                  "ranks": world, "checked_queries": idx.tolist(),
                                  "ids_equal": bool(np.array_equal(got_i, ei)),
                                  "dists_equal": bool(np.array_equal(got_d, ed))}),
                      flush=True)
            dist.barrier(device_ids=[local])
    finally:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
