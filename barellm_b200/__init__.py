"""barellm_b200 -- B200 (sm_100a) paged-KV hot path for BareLLM.

Drop-in replacements for the reference's paged cache write/read path and its
attention backend, backed by hand-written CUDA kernels behind a C ABI
(``include/barellm_b200.h``):

    PagedKVCache / PagedKVCacheView / PagedLayerKV   paged_kv_cache.py
    BatchKVCache / BatchLayerKV                      batched_kv_cache.py
    PackedBatchKVCache / PackedBatchLayerKV          batched_kv_cache.py (batched chunked prefill)
    BlockPool / KVCacheBlock, KVCacheManager         block_pool.py, kv_cache_manager.py
    CudaPagedAttentionBackend, create_attention_backend  backend.py
    ops (tensor-level kernel wrappers)                ops.py
"""

from . import ops
from .backend import AttentionBackendName, CudaPagedAttentionBackend, create_attention_backend
from .batched_kv_cache import BatchKVCache, BatchLayerKV, PackedBatchKVCache, PackedBatchLayerKV
from .block_pool import BlockPool, KVCacheBlock
from .kv_cache_manager import KVCacheManager
from .paged_kv_cache import (
    BlockTableArena,
    PagedBatchKVMetadata,
    PagedKVCache,
    PagedKVCacheView,
    PagedKVMetadata,
    PagedLayerKV,
)

__all__ = [
    "AttentionBackendName",
    "BatchKVCache",
    "BatchLayerKV",
    "BlockPool",
    "BlockTableArena",
    "CudaPagedAttentionBackend",
    "KVCacheBlock",
    "KVCacheManager",
    "PackedBatchKVCache",
    "PackedBatchLayerKV",
    "PagedBatchKVMetadata",
    "PagedKVCache",
    "PagedKVCacheView",
    "PagedKVMetadata",
    "PagedLayerKV",
    "create_attention_backend",
    "ops",
]
