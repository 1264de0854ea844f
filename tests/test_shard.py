"""Host-side sharding across ranks, exercised with two gloo ranks on CPU."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_accelerator_b200.shard import gather_tokens, shard


def test_shard_blocks_cover_the_batch_once():
    total, world = 64, 8
    ids = [i for r in range(world) for i in shard(total, world, r)]
    assert ids == list(range(total))
    with pytest.raises(ValueError):
        shard(10, 4, 0)
    with pytest.raises(ValueError):
        shard(8, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, total: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard(total, world, rank)
        # each rank's "greedy tokens": a function of the sequence id
        local = torch.tensor([7 * s + 3 for s in mine], dtype=torch.int32)
        got = gather_tokens(local, world)
        out.put((rank, got.tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gather_tokens_reassembles_batch_in_sequence_order(world):
    total = 12
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, total, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [7 * s + 3 for s in range(total)]
    assert all(results[r] == want for r in range(world))
