"""Host-side logic that needs no GPU: block pool order, request accounting,
the block-table arena and the reference-style argument checks."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from barellm_b200 import BlockPool, KVCacheManager, PagedKVCache
from barellm_b200.paged_kv_cache import BlockTableArena


class Req:
    def __init__(self, rid: str, n: int):
        self.id = rid
        self.seq_len = n


def test_block_pool_hands_out_highest_ids_first_like_the_reference():
    pool = BlockPool(5)
    assert [b.block_id for b in pool.allocate(2)] == [4, 3]
    got = pool.allocate(2)
    assert [b.block_id for b in got] == [2, 1]
    pool.free(got)
    assert [b.block_id for b in pool.allocate(1)] == [1]
    assert pool.allocate(10) == []
    assert pool.allocate(0) == []
    assert pool.can_allocate(2) and not pool.can_allocate(3)


def test_block_pool_matches_reference_stack_semantics_on_random_ops():
    """Against a literal pop-one-at-a-time model of the reference pool
    (src/barellm/engine/block_pool.py:17-28)."""
    rs = np.random.RandomState(0)
    pool = BlockPool(64)
    model = list(range(64))
    held = []
    for _ in range(500):
        if held and rs.rand() < 0.4:
            blocks = held.pop(rs.randint(len(held)))
            pool.free(blocks)
            model.extend(b.block_id for b in blocks)
        else:
            n = int(rs.randint(0, 6))
            got = pool.allocate(n)
            if n > len(model):
                assert got == []
                continue
            expect = [model.pop() for _ in range(n)]
            assert [b.block_id for b in got] == expect
            held.append(got)
    assert sorted(pool.free_ids) == sorted(model)


def test_manager_allocates_grows_and_frees():
    storage = PagedKVCache(num_layers=1, max_blocks=4, num_kv_heads=1, block_size=2, head_dim=2)
    pool = BlockPool(4)
    mgr = KVCacheManager(2, pool, storage)
    r = Req("A", 3)
    assert mgr.allocate_request(r)
    assert len(mgr.request_id_to_blocks["A"]) == 2
    r.seq_len = 5
    assert mgr.allocate_request(r)
    assert storage.request_pages["A"].block_table.tolist() == [3, 2, 1]
    assert not mgr.allocate_request(Req("B", 3))  # only one block left
    assert "B" not in mgr.request_id_to_blocks
    mgr.free_request("A")
    assert len(pool.free_ids) == 4
    with pytest.raises(KeyError, match="Unknown request"):
        mgr.get_cache(r)


def test_arena_uploads_only_changed_entries_and_grows():
    arena = BlockTableArena(torch.device("cpu"), rows=2, width=2)
    r0 = arena.alloc_row()
    arena.set_row(r0, [5, 6])
    arena.set_row(r0, [5, 6, 7, 8, 9])  # grows width to 8
    assert arena.width == 8
    assert arena.row_view(r0).tolist() == [5, 6, 7, 8, 9]
    r1 = arena.alloc_row()
    r2 = arena.alloc_row()  # grows rows
    assert len({r0, r1, r2}) == 3
    arena.set_row(r2, [1])
    assert arena.table[r2, :1].tolist() == [1]
    arena.free_row(r1)
    assert arena.alloc_row() == r1
    # a rewritten prefix is re-uploaded from the first differing entry
    arena.set_row(r0, [5, 42, 7])
    assert arena.row_view(r0).tolist() == [5, 42, 7]


def test_paged_cache_argument_checks():
    with pytest.raises(ValueError, match="num_layers must be positive"):
        PagedKVCache(0, 4, 1, 2, 2)
    with pytest.raises(ValueError, match="block_size must be positive"):
        PagedKVCache(1, 4, 1, 0, 2)
    storage = PagedKVCache(num_layers=2, max_blocks=4, num_kv_heads=2, block_size=2, head_dim=3)
    storage.register_request("A", BlockPool(4).allocate(1))
    layer = storage.get_cache("A").layer(0)
    with pytest.raises(ValueError, match="enough allocated"):
        layer.check_capacity(3)
    with pytest.raises(ValueError, match="KV-head count cannot change"):
        layer.check_new_kv(torch.zeros(1, 3, 1, 3), torch.zeros(1, 3, 1, 3))
    with pytest.raises(IndexError, match="Invalid layer index"):
        storage.get_cache("A").layer(2)
    with pytest.raises(ValueError, match="empty"):
        layer.read()
    storage.unregister_request("A")
    with pytest.raises(KeyError, match="Unknown request"):
        storage.get_cache("A")


def test_kernels_refuse_cpu_tensors():
    from barellm_b200 import ops

    kc = torch.zeros((1, 4, 2, 2, 3))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_gather(kc, kc.clone(), 0, torch.zeros((1, 1), dtype=torch.int32), torch.ones(1, dtype=torch.int32), 1)


def test_backend_factory_names():
    from barellm_b200 import CudaPagedAttentionBackend, create_attention_backend

    assert isinstance(create_attention_backend("cuda"), CudaPagedAttentionBackend)
    assert isinstance(create_attention_backend("auto"), CudaPagedAttentionBackend)
    with pytest.raises(RuntimeError, match="Triton"):
        create_attention_backend("triton")
    with pytest.raises(ValueError, match="Unknown attention backend"):
        create_attention_backend("flash")  # type: ignore[arg-type]


def test_prefill_chunk_plan_packs_and_splits_prompts_in_order():
    from barellm_b200.engine import plan_prefill_chunks

    groups = plan_prefill_chunks([5, 3, 10, 2], 6)
    assert groups == [[(0, 0, 5), (1, 0, 1)], [(1, 1, 2), (2, 0, 4)], [(2, 4, 6)], [(3, 0, 2)]]
    assert all(sum(n for _, _, n in g) <= 6 for g in groups)
    # every prompt token is covered exactly once, in order
    for lens, budget in (([1] * 9, 4), ([17, 1, 33], 8), ([100], 7), ([3, 4, 5], 1000)):
        seen = {}
        for g in plan_prefill_chunks(lens, budget):
            assert len({r for r, _, _ in g}) == len(g)  # a request appears once per group
            for r, s, n in g:
                assert s == seen.get(r, 0) and n > 0
                seen[r] = s + n
        assert [seen[r] for r in range(len(lens))] == lens
    with pytest.raises(ValueError):
        plan_prefill_chunks([3, 0], 4)
