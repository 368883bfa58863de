"""Request placement across per-GPU BlockPool shards (data-parallel by request).

The reference runs one engine on one device: its Scheduler offers waiting
requests in FIFO order up to ``max_batch`` (src/barellm/engine/scheduler.py:16-18)
and the engine admits one only when the BlockPool can allocate the blocks it
needs (src/barellm/engine/block_pool.py:14-15, kv_cache_manager.py:27-39,
engine.py:581-596); a request that does not fit waits for a later step.

Across the GPUs of a node each GPU owns a BlockPool shard (block ids local to
that GPU) and a PagedKVCache, and every request lives on exactly one GPU, so
the decode path needs no collective.  ``RequestPlacer`` decides which shard
serves each whole request: longest request first, onto the least-loaded shard
(fewest tokens placed) among the shards whose free blocks can hold the
request's full length (prompt + new tokens, reserved at placement so decode
never runs out of blocks).  A request that fits no shard right now is
deferred, not failed, and is placed once a finished request returns its
blocks.  ``serve_by_request`` runs that protocol over a process group: rank 0
owns the placer, each round broadcasts the assignments, every rank runs its
share, and the generated tokens come back to rank 0 over the host channel
(object collectives; gloo or NCCL).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass, field

import numpy as np


def place_requests(lengths: Sequence[int] | np.ndarray, world: int) -> list[list[int]]:
    """Index lists, one per shard, for requests of the given lengths on
    ``world`` shards without a capacity limit: longest first onto the shard
    with the fewest tokens so far (lowest index on ties).  Deterministic, so
    every rank derives the same placement from the same lengths."""
    placer = RequestPlacer([None] * world, block_size=1)
    for i, n in enumerate(lengths):
        placer.submit(i, int(n))
    assigned = placer.place()
    return [sorted(assigned[g]) for g in range(world)]


@dataclass
class _Shard:
    free_blocks: int | None  # None: no capacity limit
    load_tokens: int = 0
    requests: set = field(default_factory=set)


class RequestPlacer:
    """Places whole requests onto BlockPool shards.

    ``free_blocks[g]`` is shard g's free block count (its BlockPool's
    ``len(free_ids)``), or None for a shard without a limit.  ``submit``
    queues a request with the number of KV tokens it will hold;
    ``place`` assigns every waiting request that fits somewhere and leaves
    the rest waiting; ``release`` returns a finished request's blocks."""

    def __init__(self, free_blocks: Sequence[int | None], block_size: int) -> None:
        if len(free_blocks) == 0:
            raise ValueError("at least one shard is required")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.block_size = block_size
        self.shards = [_Shard(None if f is None else int(f)) for f in free_blocks]
        self._capacity = [s.free_blocks for s in self.shards]
        self.waiting: dict = {}  # request id -> tokens, in submission order
        self.placed: dict = {}  # request id -> (shard, tokens, blocks)

    def blocks_needed(self, tokens: int) -> int:
        return -(-int(tokens) // self.block_size)

    def submit(self, request_id, tokens: int) -> None:
        if tokens <= 0:
            raise ValueError("a request must hold at least one token")
        if request_id in self.waiting or request_id in self.placed:
            raise ValueError(f"request {request_id!r} is already queued")
        need = self.blocks_needed(tokens)
        if all(c is not None and need > c for c in self._capacity):
            raise ValueError(f"request {request_id!r} needs {need} KV blocks, more than any shard holds")
        self.waiting[request_id] = int(tokens)

    def place(self) -> dict[int, list]:
        """Assigns waiting requests, longest first (submission order on ties).
        Returns ``{shard: [request ids placed now]}`` for every shard."""
        out: dict[int, list] = {g: [] for g in range(len(self.shards))}
        order = sorted(self.waiting.items(), key=lambda kv: -kv[1])
        for rid, tokens in order:
            need = self.blocks_needed(tokens)
            fits = [g for g, s in enumerate(self.shards) if s.free_blocks is None or s.free_blocks >= need]
            if not fits:
                continue  # deferred until blocks come back
            g = min(fits, key=lambda i: (self.shards[i].load_tokens, i))
            s = self.shards[g]
            if s.free_blocks is not None:
                s.free_blocks -= need
            s.load_tokens += tokens
            s.requests.add(rid)
            self.placed[rid] = (g, tokens, need)
            del self.waiting[rid]
            out[g].append(rid)
        return out

    def release(self, request_id) -> int:
        """Returns a placed request's blocks to its shard; gives the shard."""
        g, tokens, need = self.placed.pop(request_id)
        s = self.shards[g]
        if s.free_blocks is not None:
            s.free_blocks += need
        s.load_tokens -= tokens
        s.requests.discard(request_id)
        return g

    def has_work(self) -> bool:
        return bool(self.waiting or self.placed)

    def loads(self) -> list[int]:
        return [s.load_tokens for s in self.shards]


# a rank's runner: [(request id, prompt token ids, max new tokens)] -> {request id: generated token ids}
BatchRunner = Callable[[list[tuple]], dict]


def serve_by_request(run_batch: BatchRunner, requests: dict | None, free_blocks: Sequence[int] | None,
                     block_size: int, group=None, max_rounds: int = 1 << 20, stats: dict | None = None
                     ) -> dict | None:
    """Serves a request set data-parallel by request over a process group.

    Every rank calls this with its own ``run_batch`` (the engine of its GPU).
    Rank 0 passes ``requests`` (``{id: (prompt token ids, max_new_tokens)}``)
    and ``free_blocks`` (each rank's BlockPool free count); the other ranks
    pass None for both.  Each round rank 0 places what fits, broadcasts the
    assignments, every rank runs its share, and the tokens are gathered back
    to rank 0, which releases the finished requests' blocks before the next
    round.  Requests that fit no shard in a round wait for a later one.
    Returns ``{id: tokens}`` on rank 0 and None elsewhere.  All ranks take the
    same collective steps in the same order.  On rank 0, ``stats`` (if given)
    receives the number of rounds and, per round, the requests placed."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    placer = None
    results: dict = {}
    failure: str | None = None  # rank 0: the error every rank raises next round
    if rank == 0:
        try:
            if requests is None or free_blocks is None or len(free_blocks) != world:
                raise ValueError("rank 0 needs the requests and one free block count per rank")
            placer = RequestPlacer(list(free_blocks), block_size)
            for rid, (prompt, max_new) in requests.items():
                placer.submit(rid, len(prompt) + int(max_new))
        except (ValueError, TypeError) as exc:
            failure = f"{type(exc).__name__}: {exc}"
    for _ in range(max_rounds):
        # message: None = done, ("error", text) = every rank raises, else {rank: [(id, prompt, max_new)]}
        msg: list = [None]
        if rank == 0:
            if failure is not None:
                msg = [("error", failure)]
            elif placer.has_work():
                assigned = placer.place()
                msg = [{g: [(rid, requests[rid][0], requests[rid][1]) for rid in ids] for g, ids in assigned.items()}]
                if stats is not None:
                    stats.setdefault("placed_per_round", []).append({g: list(ids) for g, ids in assigned.items()})
                    stats["rounds"] = len(stats["placed_per_round"])
        dist.broadcast_object_list(msg, src=0, group=group)
        if msg[0] is None:
            return results if rank == 0 else None
        if isinstance(msg[0], tuple):
            raise RuntimeError(f"request serving failed: {msg[0][1]}")
        mine = msg[0].get(rank, [])
        try:
            out = ("ok", run_batch(mine) if mine else {})
        except Exception as exc:  # reported to every rank through rank 0 next round
            out = ("error", f"rank {rank}: {type(exc).__name__}: {exc}")
        gathered: list | None = [None] * world if rank == 0 else None
        dist.gather_object(out, gathered, dst=0, group=group)
        if rank == 0:
            for status, part in gathered:
                if status != "ok":
                    failure = failure or part
                    continue
                for rid, toks in part.items():
                    results[rid] = toks
                    placer.release(rid)
    raise RuntimeError("serve_by_request: round limit reached")
