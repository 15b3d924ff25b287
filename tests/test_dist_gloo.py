"""Multi-process host logic on CPU (gloo, world size 2): sequence sharding
covers every row exactly once, and the max-over-ranks timing reduction."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from anima_flat_b200.shard import max_over_ranks, rows_of, shard_sequences


def test_shards_partition_sequences():
    for n in (0, 1, 7, 32):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                s = shard_sequences(n, world, r)
                seen += list(s)
                assert len(s) in (n // world, n // world + 1)
            assert seen == list(range(n))
    assert list(rows_of(range(2, 4), 4096)) == list(range(8192, 16384))
    with pytest.raises(ValueError):
        shard_sequences(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard_sequences(32, world, rank)
        # every rank reduces its own rows; the union must be all rows, once
        rows = torch.zeros(32 * 16, dtype=torch.int32)
        rows[rows_of(mine, 16).start:rows_of(mine, 16).stop] = 1
        dist.all_reduce(rows)
        t = max_over_ranks(1.5 + rank)
        out[rank] = (int(rows.min()), int(rows.max()), t)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_cover_rows_and_take_max():
    world = 2
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn",
                       join=True)
    for rank in range(world):
        lo, hi, t = out[rank]
        assert lo == 1 and hi == 1
        assert t == 2.5
