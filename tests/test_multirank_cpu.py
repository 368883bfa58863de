"""Multi-process host logic on CPU (gloo, world size 2): every rank derives
the same request placement from the seed, the shards are disjoint and cover
the batch, a rank's share is balanced, and the max-over-ranks timing
reduction picks the slowest rank."""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = bench.WORKLOADS["decode_qwen8b_long"]
        lens = bench.request_lengths(wl, 1234)
        mine = bench.place_requests(lens, world)[rank]
        gathered: list = [None] * world
        dist.all_gather_object(gathered, mine)
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out.put((rank, gathered, float(t.item()), int(sum(lens[mine]))))
    finally:
        dist.destroy_process_group()


def test_request_placement_is_consistent_across_ranks():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    views = [r[1] for r in results]
    assert views[0] == views[1], "ranks disagree on placement"
    shards = views[0]
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(256)) and not set(shards[0]) & set(shards[1])
    loads = [r[3] for r in results]
    assert max(loads) / min(loads) < 1.05
    assert all(r[2] == 11.0 for r in results)


def test_placement_balances_tokens_for_8_gpus():
    wl = bench.WORKLOADS["decode_qwen8b_long"]
    lens = bench.request_lengths(wl, 1234)
    shards = bench.place_requests(lens, 8)
    loads = [int(np.sum(lens[s])) for s in shards]
    assert sorted(i for s in shards for i in s) == list(range(256))
    assert max(loads) / min(loads) < 1.05
