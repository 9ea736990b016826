"""Sharded search with shared bounds, as 2 and 3 ranks on one GPU (B200 only).

Every rank runs the tensor-core engine on its own row shard of cuda:0 and
all-reduces its level bounds with the other ranks through gloo after every
filter level (the same hook the NCCL path uses); the ranks' lists are then
gathered on the host and merged.  The merged lists must equal the oracle's
exact top-k of the whole database: the shared bounds (the minimum of the
shards' k-th values and the maximum of their ceil(k / shards)-th values) may
only drop rows that cannot be in the global top-k.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_ROWS, N_QUERIES, DIM = 60_013, 300, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, k, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from gpu_algo_b200 import data, engine
        from gpu_algo_b200.sharded import make_local_search, shard_range, sharded_search
        r0, r1 = shard_range(N_ROWS, rank, world)
        X = torch.from_numpy(data.generate("mixture", 2, DIM, r0, r1, centre_seed=2)).cuda()
        Q = torch.from_numpy(data.generate("mixture", 3, DIM, 0, N_QUERIES, centre_seed=2)).cuda()
        calls = []
        plan_rows = shard_range(N_ROWS, 0, world)[1]  # the largest shard is the first
        phases = []
        inner = make_local_search(plan_rows=plan_rows, engine="tc_f16", on_phase=phases.append)

        def local(Qt, Xt, kk, off):
            d_, i_ = inner(Qt, Xt, kk, off)
            st = engine.last_stats(Qt, Xt, kk, engine="tc_f16", plan_rows=plan_rows,
                                   shards=world)
            calls.append(st)
            torch.cuda.synchronize()
            return d_.cpu(), i_.cpu()  # gloo gathers host tensors

        def merge(blocks, kk):
            from gpu_algo_b200.sharded import unpack_lists
            all_d, all_i = unpack_lists(blocks)
            from oracle import oracle_merge
            d_, i_ = oracle_merge(all_d.numpy(), all_i.numpy(), kk)
            return torch.from_numpy(d_), torch.from_numpy(i_)

        d_, i_ = sharded_search(Q, X, k, r0, local_search=local, merge_fn=merge)
        # every filter level shares its bounds, and reports before and after doing so
        levels = len(phases) // 2
        assert levels >= 2 and phases == [f"level {i} {w}" for i in range(levels)
                                          for w in ("filtered", "shared")], phases
        np.savez(os.path.join(outdir, f"r{rank}.npz"), d=d_.numpy(), i=i_.numpy(),
                 survivors=calls[0]["survivors"], err=calls[0]["device_error"])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,k", [(2, 10), (2, 100), (3, 100)])
def test_shared_bounds_over_ranks_exact(tmp_path, world, k):
    from gpu_algo_b200 import data
    from oracle import oracle_knn
    mp.start_processes(_rank_main, args=(world, _free_port(), k, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    X = data.generate("mixture", 2, DIM, 0, N_ROWS, centre_seed=2)
    Q = data.generate("mixture", 3, DIM, 0, N_QUERIES, centre_seed=2)
    ed, ei = oracle_knn(Q, X, k)
    survivors = 0
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        assert int(z["err"]) == 0
        np.testing.assert_array_equal(z["i"], ei, err_msg=f"rank {r} ids")
        np.testing.assert_array_equal(z["d"], ed, err_msg=f"rank {r} dists")
        survivors += int(z["survivors"])
    # the shards re-rank about k rows per query between them, not k each
    assert survivors < 2 * k * N_QUERIES
