"""Free list of physical KV blocks, one per GPU shard.

Same contract as the reference's BlockPool (src/barellm/engine/block_pool.py:9-28):
``allocate(n)`` hands out the most recently freed / highest ids first and
returns ``[]`` when the pool cannot satisfy the request; ``free`` returns blocks
to the top of the stack.  Keeping that order keeps block tables identical to
the reference's for the same sequence of calls.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(slots=True)
class KVCacheBlock:
    block_id: int


class BlockPool:
    def __init__(self, max_blocks: int) -> None:
        self.blocks = [KVCacheBlock(i) for i in range(max_blocks)]
        # stack of free ids; the top of the stack is the end of the list
        self.free_ids: list[int] = list(range(max_blocks))

    @property
    def num_free(self) -> int:
        return len(self.free_ids)

    def can_allocate(self, num_blocks: int) -> bool:
        return num_blocks <= len(self.free_ids)

    def allocate(self, num_blocks: int) -> list[KVCacheBlock]:
        if num_blocks > len(self.free_ids):
            return []
        if num_blocks <= 0:
            return []
        taken = self.free_ids[-num_blocks:]
        del self.free_ids[-num_blocks:]
        return [self.blocks[i] for i in reversed(taken)]

    def free(self, blocks: list[KVCacheBlock]) -> None:
        self.free_ids.extend(b.block_id for b in blocks)
