"""Row-sharded multi-GPU search: one process per GPU, NCCL over NVLink.

The database is split by rows across the ranks of a process group; every
rank searches its own shard (global row index = shard start + local row),
one all-gather moves each rank's (n, k) sorted (distance, index) lists, packed
into one block, to every rank, and the on-device merge kernel
(``bfk_merge_strided``) reduces the world * k candidates per query to the
final k, reading the gathered blocks in place.  The reference has no
multi-GPU path; this is the exchange step its split-N partial/merge design
(bf/fp32_tiled.py:182-239) implies once the tiles live on different GPUs.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_range(total_rows: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [begin, end) of `rank`: contiguous, sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, rem = divmod(total_rows, world)
    begin = rank * base + min(rank, rem)
    return begin, begin + base + (1 if rank < rem else 0)


def pack_lists(d_: torch.Tensor, i_: torch.Tensor) -> torch.Tensor:
    """One rank's (n, k) distances and ids as one int32 block [distance bits | ids]."""
    return torch.cat((d_.contiguous().view(torch.int32).view(-1), i_.contiguous().view(-1)))


def gather_lists(d_: torch.Tensor, i_: torch.Tensor, group=None) -> torch.Tensor:
    """One all-gather of every rank's packed (distance, index) block: (world, 2, n, k)
    int32 on every rank, rank r's distance bits in [r, 0] and its ids in [r, 1]."""
    world = dist.get_world_size(group)
    n, k = d_.shape
    send = pack_lists(d_, i_)
    recv = torch.empty((world * send.numel(),), dtype=torch.int32, device=d_.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    return recv.view(world, 2, n, k)


def unpack_lists(blocks: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(world, 2, n, k) packed blocks -> (world, n, k) distances and ids (copies)."""
    return blocks[:, 0].contiguous().view(torch.float32), blocks[:, 1].contiguous()


def make_local_search(group=None, plan_rows: int = 0, on_phase: Callable | None = None,
                      **search_kwargs) -> Callable:
    """The per-shard search of `sharded_search` with the CUDA engine.

    Every rank must use the same `plan_rows` (the largest shard's row count);
    0 looks it up with an all-reduce on the first call, which also finds the
    smallest shard, so that every rank raises if one shard is empty.  With more
    than one rank, the engine's level hook all-reduces (MIN) each query's bounds
    over `group` after every filter level; `search_kwargs` go to `engine.search`.
    `on_phase(name)`, if given, is called at each level's all-reduce, before
    ("level i filtered") and after it ("level i shared"), as the work is enqueued.
    """
    from .engine import search
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    state = {"plan_rows": int(plan_rows)}
    empty = "every shard of a sharded search needs at least one row"

    level = [0]

    def share_bounds(t):
        # both halves of `t` are minimised: see bfk_level_hook_t
        if on_phase is not None:
            on_phase(f"level {level[0]} filtered")
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
        if on_phase is not None:
            on_phase(f"level {level[0]} shared")
        level[0] += 1

    def local_search(Q_, X_, k_, id_offset):
        if world > 1 and state["plan_rows"] <= 0:
            # (largest rows, -smallest rows) over the shards
            sizes = torch.tensor([X_.shape[0], -X_.shape[0]], dtype=torch.int64, device=X_.device)
            dist.all_reduce(sizes, op=dist.ReduceOp.MAX, group=group)
            largest, neg_smallest = (int(v) for v in sizes.tolist())
            if neg_smallest == 0:
                raise ValueError(empty)
            state["plan_rows"] = largest
        if world > 1 and X_.shape[0] == 0:
            # with `plan_rows` given there is no size exchange: the other shards learn
            # of this one when their bound all-reduce runs out of time
            raise ValueError(empty)
        level[0] = 0
        return search(Q_, X_, k_, id_offset=id_offset,
                      bound_hook=share_bounds if world > 1 else None,
                      plan_rows=state["plan_rows"] if world > 1 else 0,
                      shards=world if world > 1 else 0, **search_kwargs)

    return local_search


def sharded_search(Q, X_shard, k: int, row_begin: int, group=None,
                   local_search: Callable | None = None,
                   merge_fn: Callable | None = None, plan_rows: int = 0,
                   on_phase: Callable | None = None,
                   **search_kwargs) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact k-NN over the union of every rank's shard; result on every rank.

    With the CUDA engine, the ranks also share each query's distance bounds
    after every filter level (an all-reduce MIN of 2n floats): the minimum over
    shards of each shard's k-th smallest value, and the maximum over shards of
    each shard's ceil(k / world)-th smallest value, both bound the global k-th
    distance, so every shard filters with the tightest bound and keeps about
    1/world of the candidates.  `plan_rows` (the largest shard's row count;
    looked up with an all-reduce when 0) gives every shard the same levels, so
    all ranks take the same collective steps.

    The exchange is one all-gather of each rank's packed (n, k) lists, distance bits
    then ids (8 n k bytes per rank), merged in place on every rank.

    `local_search(Q, X, k, id_offset)` and `merge_fn(blocks, k)` (blocks: the
    gathered (world, 2, n, k) int32 lists) default to the CUDA engine; tests
    substitute CPU stand-ins to exercise the orchestration over gloo.
    `search_kwargs` go to `engine.search`.  `on_phase(name)`, if given, is called
    as each phase's work has been enqueued ("start", the level phases of
    `make_local_search`, "searched", "gathered", "merged"), e.g. to record events.
    """
    def phase(name):
        if on_phase is not None:
            on_phase(name)

    if local_search is None:
        local_search = make_local_search(group, plan_rows, on_phase=on_phase, **search_kwargs)
    if merge_fn is None:
        from .engine import merge_packed as merge_fn
    phase("start")
    d_, i_ = local_search(Q, X_shard, k, row_begin)
    phase("searched")
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return d_, i_
    blocks = gather_lists(d_, i_, group)
    phase("gathered")
    out = merge_fn(blocks, k)
    phase("merged")
    return out
