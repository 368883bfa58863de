"""Request placement across per-GPU BlockPool shards (barellm_b200.placement).

Single process: longest-first balance, capacity admission (a request that
fits no shard now is deferred and placed once blocks come back), and the
up-front error for a request larger than any shard -- the reference's
admission rule (src/barellm/engine/block_pool.py:14-15,
src/barellm/engine/engine.py:581-596).  Two gloo ranks on CPU: the serving
loop with one rank's shard too small to take every request at once; the
request that does not fit is deferred to a later round, never failed, and
every request's tokens come back to rank 0 over the host channel."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from barellm_b200.block_pool import BlockPool
from barellm_b200.placement import RequestPlacer, place_requests, serve_by_request


def test_place_requests_longest_first_onto_least_loaded():
    lens = [5, 100, 30, 30, 70, 1]
    shards = place_requests(lens, 2)
    assert shards == [[1, 3], [0, 2, 4, 5]]  # 100+30 | 70+30+5+1
    assert sorted(i for s in shards for i in s) == list(range(6))
    loads = [sum(lens[i] for i in s) for s in shards]
    assert abs(loads[0] - loads[1]) <= max(lens)


def test_placement_matches_a_plain_greedy_restatement():
    rs = np.random.RandomState(0)
    lens = np.round(np.exp(rs.uniform(np.log(1024), np.log(32768), size=256))).astype(np.int64)
    for world in (1, 2, 4, 8):
        loads = [0] * world
        want: list[list[int]] = [[] for _ in range(world)]
        for i in sorted(range(len(lens)), key=lambda i: -int(lens[i])):
            g = min(range(world), key=lambda r: (loads[r], r))
            want[g].append(i)
            loads[g] += int(lens[i])
        assert place_requests(lens, world) == [sorted(x) for x in want]


def test_capacity_defers_then_places_after_release():
    # shard 0 holds 4 blocks, shard 1 holds 2 (block_size 16)
    p = RequestPlacer([4, 2], block_size=16)
    p.submit("a", 60)  # 4 blocks: only shard 0
    p.submit("b", 30)  # 2 blocks
    p.submit("c", 20)  # 2 blocks
    first = p.place()
    assert first == {0: ["a"], 1: ["b"]}
    assert list(p.waiting) == ["c"]  # deferred, not failed
    assert p.place() == {0: [], 1: []}
    assert p.release("b") == 1
    assert p.place() == {0: [], 1: ["c"]}
    for rid in ("a", "c"):
        p.release(rid)
    assert not p.has_work() and [s.free_blocks for s in p.shards] == [4, 2]


def test_request_larger_than_every_shard_is_rejected_up_front():
    p = RequestPlacer([4, 2], block_size=16)
    with pytest.raises(ValueError, match="more than any shard"):
        p.submit("huge", 16 * 4 + 1)
    with pytest.raises(ValueError):
        p.submit("empty", 0)


def test_free_blocks_come_from_the_shards_block_pools():
    pools = [BlockPool(10), BlockPool(3)]
    pools[0].allocate(4)
    p = RequestPlacer([len(pool.free_ids) for pool in pools], block_size=16)
    assert [s.free_blocks for s in p.shards] == [6, 3]


# --- two gloo ranks -------------------------------------------------------
def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fake_generate(prompt: list[int], n: int) -> list[int]:
    return [(sum(prompt) + 7 * i) % 1000 for i in range(n)]


def _serve_worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rounds: list[list] = []

        def run_batch(items):
            rounds.append([rid for rid, _, _ in items])
            return {rid: _fake_generate(prompt, n) for rid, prompt, n in items}

        if rank == 0:
            rs = np.random.RandomState(3)
            reqs = {f"r{i}": (list(rs.randint(0, 100, size=int(rs.randint(8, 60)))), 8) for i in range(6)}
            # the requests need 3-4 blocks each (23 in all); the shards hold
            # 8 and 5, so only three fit in the first round and the rest wait
            stats: dict = {}
            res = serve_by_request(run_batch, reqs, [8, 5], block_size=16, stats=stats)
            ok = all(res[rid] == _fake_generate(p, n) for rid, (p, n) in reqs.items()) and len(res) == len(reqs)
            first = stats["placed_per_round"][0]
            ok = ok and stats["rounds"] >= 2 and sorted(first[0] + first[1]) == ["r0", "r2", "r4"]
        else:
            res = serve_by_request(run_batch, None, None, block_size=16)
            ok = res is None
        out.put((rank, ok, rounds))
    finally:
        dist.destroy_process_group()


def test_two_rank_serving_defers_when_a_shard_is_full():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_serve_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in results)
    served = [rid for _, _, rounds in results for batch in rounds for rid in batch]
    assert sorted(served) == sorted(f"r{i}" for i in range(6))  # each request exactly once
    rank1_rounds = results[1][2]
    assert len(rank1_rounds) >= 2  # the 5-block shard served requests in more than one round
    assert all(len(batch) == 1 for batch in rank1_rounds)  # and holds one 4-block request at a time


def _failing_worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def run_batch(items):
            if rank == 1:
                raise RuntimeError("engine on rank 1 failed")
            return {rid: [1] for rid, _, _ in items}

        reqs = {f"r{i}": ([1] * 20, 4) for i in range(4)} if rank == 0 else None
        try:
            serve_by_request(run_batch, reqs, [100, 100] if rank == 0 else None, block_size=16)
            out.put((rank, "returned"))
        except RuntimeError as exc:
            out.put((rank, str(exc)))
    finally:
        dist.destroy_process_group()


def test_a_failing_rank_ends_the_serving_loop_on_every_rank():
    """A rank whose engine raises still takes the round's collective steps;
    the error reaches every rank as a RuntimeError in the next round, so no
    rank is left waiting in a collective."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all("engine on rank 1 failed" in msg for _, msg in results), results
