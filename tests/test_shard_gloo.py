"""CPU: the multi-GPU partition rule and the measurement reductions, run as a
world-size-2 gloo process group (two spawned ranks on CPU)."""

from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from imba_chess_b200.shard import reduce_max, reduce_sum, shard_games


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, num_games: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard_games(num_games, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        t_max = reduce_max(1.0 + rank)
        n_sum = reduce_sum(len(mine))
        out.put((rank, gathered, t_max, n_sum))
    finally:
        dist.destroy_process_group()


def test_games_partition_across_two_gloo_ranks():
    world, num_games = 2, 37
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, num_games, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, t_max, n_sum in results:
        flat = sorted(g for part in gathered for g in part)
        assert flat == list(range(num_games))            # every game exactly once
        assert all(set(a).isdisjoint(b) for i, a in enumerate(gathered) for b in gathered[i + 1 :])
        assert t_max == 2.0                              # max over ranks
        assert n_sum == num_games


def test_shard_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard_games(10, 2, 2)
    with pytest.raises(ValueError):
        shard_games(10, 0, 0)
    assert shard_games(5, 1, 2) == [1, 3]
