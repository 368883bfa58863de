"""Per-request block accounting on top of a BlockPool shard.

Contract of the reference's KVCacheManager (src/barellm/engine/kv_cache_manager.py:8-45):
``allocate_request`` tops a request up to ``ceil(seq_len / block_size)``
blocks and registers the (grown) list with the paged cache; it returns False,
allocating nothing, when the shard lacks free blocks.  ``free_request`` returns
the blocks and drops the request's pages.
"""

from __future__ import annotations

from typing import Protocol

from .block_pool import BlockPool, KVCacheBlock
from .paged_kv_cache import PagedKVCache, PagedKVCacheView


class HasSeqLen(Protocol):
    id: str

    @property
    def seq_len(self) -> int: ...


class KVCacheManager:
    def __init__(self, block_size: int, block_pool: BlockPool, paged_kv_cache: PagedKVCache) -> None:
        self.block_size = block_size
        self.block_pool = block_pool
        self.paged_kv_cache = paged_kv_cache
        self.request_id_to_blocks: dict[str, list[KVCacheBlock]] = {}

    def blocks_needed(self, seq_len: int) -> int:
        return -(-seq_len // self.block_size)

    def get_cache(self, req: HasSeqLen) -> PagedKVCacheView:
        if req.id not in self.request_id_to_blocks:
            raise KeyError(f"Unknown request: {req.id}")
        return self.paged_kv_cache.get_cache(req.id)

    def allocate_request(self, req: HasSeqLen) -> bool:
        owned = self.request_id_to_blocks.get(req.id, [])
        missing = max(self.blocks_needed(req.seq_len) - len(owned), 0)
        if not self.block_pool.can_allocate(missing):
            return False
        grown = owned + self.block_pool.allocate(missing)
        self.request_id_to_blocks[req.id] = grown
        self.paged_kv_cache.register_request(req.id, grown)
        return True

    def free_request(self, request_id: str) -> None:
        blocks = self.request_id_to_blocks.pop(request_id, None)
        if blocks is not None:
            self.block_pool.free(blocks)
        self.paged_kv_cache.unregister_request(request_id)
