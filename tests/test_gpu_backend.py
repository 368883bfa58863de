"""The drop-in layer on the GPU: the reference's storage scenarios
(tests/test_paged_kv_cache.py, test_benchmark_paged_cache.py,
test_kv_cache_manager.py of the reference) replayed through barellm_b200's
PagedKVCache / BatchKVCache, and the CUDA attention backend against the
oracle and against itself (batched vs independent rows)."""

from __future__ import annotations

from typing import cast

import numpy as np
import pytest
import torch

import gpu_helpers as gh
from barellm_b200 import (
    BatchKVCache,
    BatchLayerKV,
    BlockPool,
    CudaPagedAttentionBackend,
    KVCacheManager,
    PagedKVCache,
    PagedLayerKV,
)
from oracle import paged_oracle as orc

pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_storage(num_layers=2, max_blocks=4, num_kv_heads=2, block_size=2, head_dim=3, dtype=torch.float32):
    storage = PagedKVCache(num_layers, max_blocks, num_kv_heads, block_size, head_dim, dtype=dtype, device=DEV)
    return storage, BlockPool(max_blocks)


def close(a, b):
    torch.testing.assert_close(a.cpu(), b.cpu(), atol=0, rtol=0)


# ---- reference storage scenarios ------------------------------------------------
def test_append_gathers_across_block_boundary(native_lib):
    storage, pool = make_storage(block_size=2)
    storage.register_request("A", pool.allocate(2))
    layer = cast(PagedLayerKV, storage.get_cache("A").layer(0))
    key = torch.arange(18, dtype=torch.float32, device=DEV).reshape(1, 2, 3, 3)
    value = key + 100
    rk, rv = layer.append(key, value)
    assert layer.seq_len == 3
    close(rk, key)
    close(rv, value)


def test_append_only_exposes_int32_metadata(native_lib):
    storage, pool = make_storage(block_size=2)
    storage.register_request("A", pool.allocate(2))
    layer = cast(PagedLayerKV, storage.get_cache("A").layer(0))
    key = torch.arange(18, dtype=torch.float32, device=DEV).reshape(1, 2, 3, 3)
    layer.append_only(key, key + 100)
    meta = layer.paged_metadata_post_append()
    assert (meta.seq_len, meta.block_size, meta.layer_idx) == (3, 2, 0)
    assert meta.block_table.dtype == torch.int32
    assert meta.block_table.tolist() == [3, 2]
    close(layer.read()[0], key)


def test_batched_metadata_is_rectangular_and_device_resident(native_lib):
    storage, pool = make_storage(block_size=2, max_blocks=4)
    storage.register_request("A", pool.allocate(1))
    storage.register_request("B", pool.allocate(2))
    layer = cast(BatchLayerKV, BatchKVCache([storage.get_cache("A"), storage.get_cache("B")]).layer(0))
    layer.append_only(torch.randn(2, 2, 1, 3, device=DEV), torch.randn(2, 2, 1, 3, device=DEV))
    meta = layer.paged_metadata_post_append()
    assert meta.block_tables.shape == (2, 2)
    assert meta.block_tables.dtype == torch.int32
    assert meta.block_tables.tolist() == [[3, -1], [2, 1]]
    assert meta.seq_lens.tolist() == [1, 1]
    assert meta.block_tables.device == storage.device


def test_block_table_refreshes_when_request_grows(native_lib):
    storage, pool = make_storage(block_size=2, max_blocks=2)
    blocks = pool.allocate(1)
    storage.register_request("A", blocks)
    layer = storage.get_cache("A").layer(0)
    key = torch.arange(18, dtype=torch.float32, device=DEV).reshape(1, 2, 3, 3)
    layer.append(key[:, :, :2], (key + 100)[:, :, :2])
    grown = blocks + pool.allocate(1)
    storage.register_request("A", grown)
    layer.append(key[:, :, 2:], (key + 100)[:, :, 2:])
    assert storage.request_pages["A"].block_table.tolist() == [b.block_id for b in grown]
    k, v = layer.read()
    close(k, key)
    close(v, key + 100)


def test_decode_appends_across_multiple_boundaries(native_lib):
    storage, pool = make_storage(block_size=2, max_blocks=3)
    storage.register_request("A", pool.allocate(3))
    layer = storage.get_cache("A").layer(0)
    key = torch.arange(24, dtype=torch.float32, device=DEV).reshape(1, 2, 4, 3)
    layer.append(key[:, :, :2], key[:, :, :2] + 100)
    layer.append(key[:, :, 2:3], key[:, :, 2:3] + 100)
    layer.append(key[:, :, 3:4], key[:, :, 3:4] + 100)
    assert layer.seq_len == 4
    close(layer.read()[0], key)


def test_requests_and_layers_are_isolated(native_lib):
    storage, pool = make_storage(max_blocks=3)
    storage.register_request("A", pool.allocate(1))
    storage.register_request("B", pool.allocate(1))
    a = storage.get_cache("A")
    b = storage.get_cache("B")
    a.layer(0).append(torch.ones(1, 2, 1, 3, device=DEV), torch.ones(1, 2, 1, 3, device=DEV))
    b.layer(0).append(torch.full((1, 2, 1, 3), 2.0, device=DEV), torch.full((1, 2, 1, 3), 2.0, device=DEV))
    assert float(a.layer(0).read()[0].sum()) == 6.0
    assert float(b.layer(0).read()[0].sum()) == 12.0
    assert a.layer(1).seq_len == 0
    with pytest.raises(ValueError, match="empty"):
        a.layer(1).read()


def test_insufficient_blocks_rejected(native_lib):
    storage, pool = make_storage(block_size=2)
    storage.register_request("A", pool.allocate(1))
    with pytest.raises(ValueError, match="enough allocated"):
        storage.get_cache("A").layer(0).append(torch.randn(1, 2, 3, 3, device=DEV), torch.randn(1, 2, 3, 3, device=DEV))


def test_reused_block_does_not_expose_previous_cache(native_lib):
    storage = PagedKVCache(1, 1, 1, 2, 2, device=DEV)
    mgr = KVCacheManager(2, BlockPool(1), storage)

    class R:
        def __init__(self, rid):
            self.id, self.seq_len = rid, 1

    a, b = R("A"), R("B")
    assert mgr.allocate_request(a)
    mgr.get_cache(a).layer(0).append(torch.full((1, 1, 1, 2), 11.0, device=DEV), torch.full((1, 1, 1, 2), 22.0, device=DEV))
    mgr.free_request("A")
    assert mgr.allocate_request(b)
    layer = mgr.get_cache(b).layer(0)
    with pytest.raises(ValueError, match="empty"):
        layer.read()
    layer.append(torch.full((1, 1, 1, 2), 33.0, device=DEV), torch.full((1, 1, 1, 2), 44.0, device=DEV))
    assert layer.read()[0].tolist() == [[[[33.0, 33.0]]]]


def test_batched_read_pads_unequal_histories(native_lib):
    bs = 16
    lengths = [15, 33]
    storage = PagedKVCache(2, 4, 2, bs, 3, device=DEV)
    mgr = KVCacheManager(bs, BlockPool(4), storage)

    class R:
        def __init__(self, rid, n):
            self.id, self.seq_len = rid, n

    reqs = [R(f"r{i}", n) for i, n in enumerate(lengths)]
    for r in reqs:
        assert mgr.allocate_request(r)
    caches = [mgr.get_cache(r) for r in reqs]
    for i, (c, n) in enumerate(zip(caches, lengths)):
        c.layer(0).append(torch.full((1, 2, n, 3), float(i + 1), device=DEV), torch.full((1, 2, n, 3), float(i + 101), device=DEV))
    k, v = BatchKVCache(caches).layer(0).read()
    assert k.shape == (2, 2, 33, 3)
    assert torch.count_nonzero(k[0, :, 15:]) == 0 and torch.count_nonzero(v[0, :, 15:]) == 0
    assert bool((k[0, :, :15] == 1).all()) and bool((v[1] == 102).all())


def test_batched_read_and_mask_match_the_reference_golden(native_lib):
    """The reference's batched read scenario (tests/golden/batch_read.npz,
    made by its PagedKVCache / KVCacheManager / BatchKVCache: boundary lengths
    15..33 at block_size 16, two layers, pool pre-filled with a sentinel)
    replayed call for call through the drop-in classes: same block tables,
    same pool bytes, same zero-padded reads and the same [B, 1, 1, Tmax]
    attention mask (batched_kv_cache.py:65-102), element for element."""
    from pathlib import Path

    import cases
    from barellm_b200.block_pool import KVCacheBlock  # noqa: F401  (the manager hands these out)

    g = np.load(Path(__file__).resolve().parent / "golden" / "batch_read.npz")
    lengths = [int(n) for n in g["lengths"]]
    bs = 16
    max_blocks = sum(-(-n // bs) for n in lengths)
    storage = PagedKVCache(2, max_blocks, 2, bs, 3, device=DEV)
    storage.key_cache.fill_(-7.0)
    storage.value_cache.fill_(-7.0)
    mgr = KVCacheManager(bs, BlockPool(max_blocks), storage)

    class R:
        def __init__(self, rid, n):
            self.id, self.seq_len = rid, n

    caches = []
    for i, n in enumerate(lengths):
        req = R(f"b{i}", n)
        assert mgr.allocate_request(req)
        cache = mgr.get_cache(req)
        for layer in range(2):
            k = torch.from_numpy(cases.pattern_tensor(i, layer, n, 2, 3, 0.0)).to(DEV)
            v = torch.from_numpy(cases.pattern_tensor(i, layer, n, 2, 3, 0.5)).to(DEV)
            cache.layer(layer).append_only(k, v)
        caches.append(cache)
    tables = [storage.request_pages[f"b{i}"].block_table.cpu().numpy() for i in range(len(lengths))]
    np.testing.assert_array_equal(gh.padded_tables(tables, g["block_tables"].shape[1]), g["block_tables"])
    np.testing.assert_array_equal(storage.key_cache.cpu().numpy(), g["key_cache"])
    np.testing.assert_array_equal(storage.value_cache.cpu().numpy(), g["value_cache"])
    for layer in range(2):
        batch_layer = BatchKVCache(caches).layer(layer)
        k, v = batch_layer.read()
        np.testing.assert_array_equal(k.cpu().numpy(), g[f"k{layer}"])
        np.testing.assert_array_equal(v.cpu().numpy(), g[f"v{layer}"])
        mask = batch_layer.attention_mask(1)
        assert mask.dtype == torch.bool and mask.device.type == "cuda"
        np.testing.assert_array_equal(mask.cpu().numpy(), g[f"mask{layer}"])


# ---- the attention backend ---------------------------------------------------------
def build_requests(lengths, hq, hkv, d, bs, dtype, seed=0, extra=1, max_blocks=None):
    rs = np.random.RandomState(seed)
    need = sum(-(-(n + extra) // bs) for n in lengths)
    p = max_blocks or need + 8
    storage = PagedKVCache(1, p, hkv, bs, d, dtype=dtype, device=DEV)
    pool = BlockPool(p)
    pool.free_ids = [int(x) for x in rs.permutation(p)]
    mgr = KVCacheManager(bs, pool, storage)

    class R:
        def __init__(self, rid, n):
            self.id, self.seq_len = rid, n

    reqs = [R(f"r{i}", n + extra) for i, n in enumerate(lengths)]
    for r in reqs:
        assert mgr.allocate_request(r)
    caches = [mgr.get_cache(r) for r in reqs]
    for c, n in zip(caches, lengths):
        k = torch.from_numpy(rs.standard_normal((1, hkv, n, d)).astype(np.float32)).to(dtype).to(DEV)
        v = torch.from_numpy(rs.standard_normal((1, hkv, n, d)).astype(np.float32)).to(dtype).to(DEV)
        c.layer(0).append_only(k, v)
    return storage, caches


def oracle_decode(storage, caches, q):
    kc = storage.key_cache.float().cpu().numpy()
    vc = storage.value_cache.float().cpu().numpy()
    tables = [storage.request_pages[c.request_id].block_table.cpu().numpy() for c in caches]
    lens = [c.layer(0).seq_len for c in caches]
    return orc.decode_attention(q.float().cpu().numpy(), kc, vc, 0, tables, lens)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (4, 4), (4, 1)])
def test_backend_batched_decode_vs_oracle(native_lib, dtype, hq, hkv):
    lengths = [1, 17, 500, 1200, 64, 33]
    storage, caches = build_requests(lengths, hq, hkv, 128, 16, dtype, seed=hq + hkv)
    q = torch.randn(len(lengths), hq, 1, 128, device=DEV).to(dtype)
    k = torch.randn(len(lengths), hkv, 1, 128, device=DEV).to(dtype)
    v = torch.randn(len(lengths), hkv, 1, 128, device=DEV).to(dtype)
    out = CudaPagedAttentionBackend().attend(q, k, v, BatchKVCache(caches).layer(0), hq // hkv)
    assert out.shape == q.shape
    storage.check_device_errors()
    ref = oracle_decode(storage, caches, q)
    err = np.abs(out.float().cpu().numpy() - ref)
    if dtype == torch.float32:
        assert err.max() <= 1e-5
    else:
        assert err.max() <= 2e-2 and err.mean() <= 2e-3


def test_backend_batched_equals_independent_decodes(native_lib):
    """Batched decode through BatchKVCache equals per-request decodes bit for
    bit (the reference checks this at 1e-5: tests/test_batched_kv_cache.py:92-150)."""
    lengths = [700, 3, 1500, 2049]
    s1, c1 = build_requests(lengths, 32, 8, 128, 16, torch.bfloat16, seed=3)
    s2, c2 = build_requests(lengths, 32, 8, 128, 16, torch.bfloat16, seed=3)
    q = torch.randn(4, 32, 1, 128, device=DEV).bfloat16()
    k = torch.randn(4, 8, 1, 128, device=DEV).bfloat16()
    v = torch.randn(4, 8, 1, 128, device=DEV).bfloat16()
    be = CudaPagedAttentionBackend()
    batched = be.attend(q, k, v, BatchKVCache(c1).layer(0), 4)
    for i, c in enumerate(c2):
        alone = be.attend(q[i : i + 1], k[i : i + 1], v[i : i + 1], c.layer(0), 4)
        assert torch.equal(alone, batched[i : i + 1])


def test_backend_layers_share_one_step_plan(native_lib):
    """Two layers of one step through the same BatchKVCache: the second layer
    reuses the first layer's metadata and plan and is still correct."""
    lengths = [900, 40, 1300]
    hq, hkv, d, bs = 16, 8, 128, 16
    rs = np.random.RandomState(1)
    need = sum(-(-(n + 1) // bs) for n in lengths)
    storage = PagedKVCache(2, need + 4, hkv, bs, d, dtype=torch.bfloat16, device=DEV)
    mgr = KVCacheManager(bs, BlockPool(need + 4), storage)

    class R:
        def __init__(self, rid, n):
            self.id, self.seq_len = rid, n

    reqs = [R(f"r{i}", n + 1) for i, n in enumerate(lengths)]
    for r in reqs:
        assert mgr.allocate_request(r)
    caches = [mgr.get_cache(r) for r in reqs]
    for layer in range(2):
        for c, n in zip(caches, lengths):
            t = torch.from_numpy(rs.standard_normal((1, hkv, n, d)).astype(np.float32)).bfloat16().to(DEV)
            c.layer(layer).append_only(t, t * 0.5)
    batch = BatchKVCache(caches)
    be = CudaPagedAttentionBackend()
    outs = []
    qs = []
    for layer in range(2):
        q = torch.randn(3, hq, 1, d, device=DEV).bfloat16()
        k = torch.randn(3, hkv, 1, d, device=DEV).bfloat16()
        qs.append(q)
        outs.append(be.attend(q, k, k * 0.5, batch.layer(layer), hq // hkv))
    assert len(batch._meta) == 1
    kc = storage.key_cache.float().cpu().numpy()
    vc = storage.value_cache.float().cpu().numpy()
    tables = [storage.request_pages[c.request_id].block_table.cpu().numpy() for c in caches]
    for layer in range(2):
        ref = orc.decode_attention(qs[layer].float().cpu().numpy(), kc, vc, layer, tables, [n + 1 for n in lengths])
        err = np.abs(outs[layer].float().cpu().numpy() - ref)
        assert err.max() <= 2e-2 and err.mean() <= 2e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_backend_prefill_then_chunked_prefill_then_decode(native_lib, dtype):
    """Single-request path (Engine._prefill): a first chunk (= the reference's
    is_causal prefill), a second chunk over the paged prefix (chunked
    prefill), then a one-token decode; each against the oracle."""
    hq, hkv, d, bs = 32, 8, 128, 16
    c1, c2 = 70, 45
    storage = PagedKVCache(1, 64, hkv, bs, d, dtype=dtype, device=DEV)
    pool = BlockPool(64)
    pool.free_ids = [int(x) for x in np.random.RandomState(2).permutation(64)]
    mgr = KVCacheManager(bs, pool, storage)

    class R:
        id, seq_len = "A", c1 + c2 + 1

    assert mgr.allocate_request(R)
    layer = mgr.get_cache(R).layer(0)
    be = CudaPagedAttentionBackend()
    tol = (1e-5, 1e-5) if dtype == torch.float32 else (2e-2, 2e-3)
    for t in (c1, c2, 1):
        q = torch.randn(1, hq, t, d, device=DEV).to(dtype)
        k = torch.randn(1, hkv, t, d, device=DEV).to(dtype)
        out = be.attend(q, k, k * 0.25, layer, hq // hkv)
        kc = storage.key_cache.float().cpu().numpy()
        vc = storage.value_cache.float().cpu().numpy()
        ref = orc.prefill_attention(q.float().cpu().numpy(), kc, vc, 0,
                                    storage.request_pages["A"].block_table.cpu().numpy(), layer.seq_len)
        err = np.abs(out.float().cpu().numpy() - ref)
        assert err.max() <= tol[0] and err.mean() <= tol[1], (t, err.max())
    # the returned layout makes the model's transpose + reshape free
    assert out.transpose(1, 2).is_contiguous()


def test_backend_uncached_full_forward_is_causal(native_lib):
    b, hq, hkv, t, d = 2, 16, 8, 50, 128
    q = torch.randn(b, hq, t, d, device=DEV).bfloat16()
    k = torch.randn(b, hkv, t, d, device=DEV).bfloat16()
    v = torch.randn(b, hkv, t, d, device=DEV).bfloat16()
    out = CudaPagedAttentionBackend().attend(q, k, v, None, hq // hkv)
    g = hq // hkv
    ref = orc.sdpa(q.float().cpu().numpy(), np.repeat(k.float().cpu().numpy(), g, 1),
                   np.repeat(v.float().cpu().numpy(), g, 1), is_causal=True)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3


def test_backend_batched_multi_token_rows(native_lib):
    """q_len > 1 through BatchKVCache (several tokens per row, e.g. drafted
    tokens) runs the paged prefill kernel; each row vs the oracle."""
    lengths = [30, 200, 5]
    hq, hkv, d, t = 16, 8, 128, 4
    storage, caches = build_requests(lengths, hq, hkv, d, 16, torch.bfloat16, seed=9, extra=t)
    q = torch.randn(3, hq, t, d, device=DEV).bfloat16()
    k = torch.randn(3, hkv, t, d, device=DEV).bfloat16()
    out = CudaPagedAttentionBackend().attend(q, k, k, BatchKVCache(caches).layer(0), hq // hkv)
    kc = storage.key_cache.float().cpu().numpy()
    vc = storage.value_cache.float().cpu().numpy()
    for i, c in enumerate(caches):
        bt = storage.request_pages[c.request_id].block_table.cpu().numpy()
        ref = orc.prefill_attention(q[i : i + 1].float().cpu().numpy(), kc, vc, 0, bt, c.layer(0).seq_len)
        err = np.abs(out[i : i + 1].float().cpu().numpy() - ref)
        assert err.max() <= 2e-2 and err.mean() <= 2e-3


def test_backend_rejects_unknown_cache_types(native_lib):
    class Contiguous:
        pass

    x = torch.zeros(1, 2, 1, 128, device=DEV).bfloat16()
    with pytest.raises(TypeError, match="paged"):
        CudaPagedAttentionBackend().attend(x, x, x, Contiguous(), 1)


def test_successive_batches_reuse_and_protect_step_metadata(native_lib):
    """An engine builds a new BatchKVCache over the same requests every decode
    step: the new batch renews the previous one's device metadata in place.
    A batch whose metadata another batch has renewed since (interleaved use)
    falls back to private metadata and stays correct."""
    lengths = [700, 33, 1030]
    hq, hkv, d, bs = 16, 8, 128, 16
    rs = np.random.RandomState(7)
    need = sum(-(-(n + 3) // bs) for n in lengths)
    storage = PagedKVCache(2, need + 4, hkv, bs, d, dtype=torch.bfloat16, device=DEV)
    mgr = KVCacheManager(bs, BlockPool(need + 4), storage)

    class R:
        def __init__(self, rid, n):
            self.id, self.seq_len = rid, n

    reqs = [R(f"r{i}", n + 3) for i, n in enumerate(lengths)]
    for r in reqs:
        assert mgr.allocate_request(r)
    caches = [mgr.get_cache(r) for r in reqs]
    for layer in range(2):
        for c, n in zip(caches, lengths):
            t = torch.from_numpy(rs.standard_normal((1, hkv, n, d)).astype(np.float32)).bfloat16().to(DEV)
            c.layer(layer).append_only(t, t * 0.5)
    be = CudaPagedAttentionBackend()

    def step(batch, layer):
        q = torch.randn(3, hq, 1, d, device=DEV).bfloat16()
        k = torch.randn(3, hkv, 1, d, device=DEV).bfloat16()
        out = be.attend(q, k, k * 0.5, batch.layer(layer), hq // hkv)
        seq = [int(x) for x in storage.arena.lens[batch.rows, layer]]
        kc = storage.key_cache.float().cpu().numpy()
        vc = storage.value_cache.float().cpu().numpy()
        tables = [storage.request_pages[c.request_id].block_table.cpu().numpy() for c in caches]
        ref = orc.decode_attention(q.float().cpu().numpy(), kc, vc, layer, tables, seq)
        err = np.abs(out.float().cpu().numpy() - ref)
        assert err.max() <= 2e-2 and err.mean() <= 2e-3

    first = BatchKVCache(caches)
    step(first, 0)
    step(first, 1)
    second = BatchKVCache(caches)  # next step: renews the first batch's buffers
    step(second, 0)
    (meta_a, _), = first._meta.values()
    (meta_b, _), = second._meta.values()
    assert meta_a is meta_b
    third = BatchKVCache(caches)  # a third step starts on layer 0 ...
    step(third, 0)
    step(second, 1)  # ... before the second finishes layer 1: private metadata
    (meta_b2, _), = second._meta.values()
    assert meta_b2 is not meta_b
    step(third, 1)
