"""The row-sharded multi-GPU orchestration, run as 2 or 3 gloo ranks on CPU.

The per-shard search and the merge are CPU stand-ins from the oracle; what is
under test is the host logic of gpu_algo_b200.sharded: shard ranges, the
global row offsets, the all-gather layout, the merge call, and the size
exchange that rejects an empty shard on every rank.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from gpu_algo_b200 import data
        from gpu_algo_b200.sharded import shard_range, sharded_search
        from oracle import oracle_knn, oracle_merge
        N, k = 20_011, 13
        r0, r1 = shard_range(N, rank, world)
        X = data.generate("normal", 0, 24, r0, r1)
        Q = data.generate("normal", 1, 24, 0, 37)

        def local(Qt, Xt, kk, off):
            d_, i_ = oracle_knn(Qt.numpy(), Xt.numpy(), kk, id_offset=off)
            return torch.from_numpy(d_), torch.from_numpy(i_)

        def merge(blocks, kk):
            from gpu_algo_b200.sharded import unpack_lists
            all_d, all_i = unpack_lists(blocks)
            d_, i_ = oracle_merge(all_d.numpy(), all_i.numpy(), kk)
            return torch.from_numpy(d_), torch.from_numpy(i_)

        phases = []
        d_, i_ = sharded_search(torch.from_numpy(Q), torch.from_numpy(X), k, r0,
                                local_search=local, merge_fn=merge, on_phase=phases.append)
        assert phases == ["start", "searched", "gathered", "merged"], phases
        np.savez(os.path.join(outdir, f"r{rank}.npz"), d=d_.numpy(), i=i_.numpy(), r0=r0, r1=r1)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_search_matches_single_shard(tmp_path, world):
    from gpu_algo_b200 import data
    from oracle import oracle_knn
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    X = data.generate("normal", 0, 24, 0, 20_011)
    Q = data.generate("normal", 1, 24, 0, 37)
    ed, ei = oracle_knn(Q, X, 13)
    spans = []
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        np.testing.assert_array_equal(z["i"], ei)
        np.testing.assert_array_equal(z["d"], ed)
        spans.append((int(z["r0"]), int(z["r1"])))
    assert spans[0][0] == 0 and spans[-1][1] == 20_011
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def _empty_shard_main(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # a rank left waiting in the size exchange ends with an error, not a hang
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from gpu_algo_b200.sharded import make_local_search
        rows = 0 if rank == world - 1 else 5000
        X = torch.zeros((rows, 16), dtype=torch.float32)
        Q = torch.zeros((3, 16), dtype=torch.float32)
        local = make_local_search()  # plan_rows looked up from the shards
        try:
            local(Q, X, 4, 0)
            outcome = "searched"
        except ValueError as e:
            outcome = str(e)
        with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
            f.write(outcome)
    finally:
        dist.destroy_process_group()


def test_empty_shard_is_rejected_on_every_rank(tmp_path):
    """The size exchange that finds the largest shard finds the smallest too, so every
    rank raises before any search (and its bound all-reduces) starts."""
    world = 3
    mp.start_processes(_empty_shard_main, args=(world, _free_port(), str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        assert "at least one row" in (tmp_path / f"r{r}.txt").read_text()


def test_shard_range_balanced():
    from gpu_algo_b200.sharded import shard_range
    for total in (0, 1, 7, 100_000_000):
        for world in (1, 2, 4, 8):
            sizes = [shard_range(total, r, world) for r in range(world)]
            assert sizes[0][0] == 0 and sizes[-1][1] == total
            lens = [b - a for a, b in sizes]
            assert max(lens) - min(lens) <= 1


def test_pack_and_unpack_lists_round_trip():
    from gpu_algo_b200.sharded import pack_lists, unpack_lists
    g = np.random.default_rng(0)
    d_ = [torch.from_numpy(g.standard_normal((5, 3)).astype(np.float32)) for _ in range(2)]
    i_ = [torch.from_numpy(g.integers(-1, 100, (5, 3)).astype(np.int32)) for _ in range(2)]
    blocks = torch.stack([pack_lists(a, b) for a, b in zip(d_, i_)]).view(2, 2, 5, 3)
    all_d, all_i = unpack_lists(blocks)
    assert torch.equal(all_d, torch.stack(d_)) and torch.equal(all_i, torch.stack(i_))
