"""Generates the golden fixtures in this folder by running the reference itself.

The reference (quanhua92/barellm) is pure Python on PyTorch and imports on a
CPU; this script drives its own classes -- PagedKVCache, BlockPool,
KVCacheManager, BatchKVCache, SDPAAttentionBackend -- on the seeded inputs of
``cases.py`` and stores their outputs.  It imports the reference package from
``$BARELLM_REFERENCE`` when that is set (a source tree whose ``src`` holds the
package, or a directory holding ``barellm`` itself), else from the installed
copy under ``baseline/_ref`` at the repository root.  The fixtures are
committed, so the tests themselves never need the reference.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
_REF = Path(os.environ.get("BARELLM_REFERENCE", HERE.parents[1] / "baseline" / "_ref"))
REF_SRC = _REF / "src" if (_REF / "src" / "barellm").is_dir() else _REF
sys.path.insert(0, str(REF_SRC))

import cases  # noqa: E402
from barellm.attention.backend import SDPAAttentionBackend  # noqa: E402
from barellm.engine.batched_kv_cache import BatchKVCache  # noqa: E402
from barellm.engine.block_pool import BlockPool  # noqa: E402
from barellm.engine.kv_cache_manager import KVCacheManager  # noqa: E402
from barellm.engine.paged_kv_cache import PagedKVCache  # noqa: E402
from barellm.engine.request import Request  # noqa: E402
from barellm.models.norm import RMSNorm  # noqa: E402
from barellm.models.rope import RotaryEmbedding, apply_rope  # noqa: E402

SENTINEL = -7.0  # pool fill so untouched slots are known


def t(x: np.ndarray, dtype=torch.float32) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype)


def f32(x: torch.Tensor) -> np.ndarray:
    return x.detach().to(torch.float32).numpy()


def padded_tables(tables: list[np.ndarray]) -> np.ndarray:
    width = max(len(x) for x in tables)
    out = np.full((len(tables), width), -1, dtype=np.int32)
    for i, x in enumerate(tables):
        out[i, : len(x)] = x
    return out


def run_decode(case: cases.DecodeCase, dtype: torch.dtype):
    storage = PagedKVCache(1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim, dtype=dtype)
    storage.key_cache.fill_(SENTINEL)
    storage.value_cache.fill_(SENTINEL)
    pool = BlockPool(case.num_blocks)
    pool.free_ids = [int(x) for x in case.free_ids]
    manager = KVCacheManager(case.block_size, pool, storage)
    caches = []
    for b, n in enumerate(case.lengths):
        req = Request(id=f"r{b}", token_ids=torch.zeros((1, int(n) + 1), dtype=torch.long))
        assert manager.allocate_request(req)
        cache = manager.get_cache(req)
        cache.layer(0).append_only(t(case.k_hist[b], dtype), t(case.v_hist[b], dtype))
        caches.append(cache)
    tables = [storage.request_pages[f"r{b}"].block_table.numpy().copy() for b in range(case.batch)]
    for mine, theirs in zip(case.block_tables(), tables):
        assert np.array_equal(mine, theirs), "block allocation order differs from the reference"
    backend = SDPAAttentionBackend()
    layer = BatchKVCache(caches).layer(0)
    out = backend.attend(t(case.q, dtype), t(case.k_new, dtype), t(case.v_new, dtype), layer,
                         group_size=case.num_q_heads // case.num_kv_heads)
    lens_after = np.array([c.layer(0).seq_len for c in caches], dtype=np.int32)
    return f32(out), padded_tables(tables), lens_after


def gen_decode() -> None:
    for name in cases.DECODE_CASES:
        case = cases.decode_case(name)
        out32, tables, lens = run_decode(case, torch.float32)
        out16, _, _ = run_decode(case, torch.bfloat16)
        np.savez_compressed(HERE / f"{name}.npz", out_f32=out32, out_bf16=out16, block_tables=tables,
                            seq_lens=lens, checksum=np.float64(case.checksum()))
        print(name, out32.shape, "tables", tables.shape)


def run_prefill(case: cases.PrefillCase, dtype: torch.dtype) -> np.ndarray:
    storage = PagedKVCache(1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim, dtype=dtype)
    storage.key_cache.fill_(SENTINEL)
    storage.value_cache.fill_(SENTINEL)
    pool = BlockPool(case.num_blocks)
    pool.free_ids = [int(x) for x in case.free_ids]
    manager = KVCacheManager(case.block_size, pool, storage)
    req = Request(id="r0", token_ids=torch.zeros((1, case.prefix + case.chunk), dtype=torch.long))
    assert manager.allocate_request(req)
    table = storage.request_pages["r0"].block_table.numpy()
    assert np.array_equal(table, case.block_table())
    layer = manager.get_cache(req).layer(0)
    group = case.num_q_heads // case.num_kv_heads
    q = t(case.q, dtype)
    if case.prefix == 0:
        # the reference prefill: append + dense read + SDPA(is_causal=True)
        out = SDPAAttentionBackend().attend(q, t(case.k_chunk, dtype), t(case.v_chunk, dtype), layer, group)
        return f32(out)
    # chunked prefill: the reference has no implementation; its parts are
    # composed with the bottom-right causal mask
    layer.append_only(t(case.k_prefix, dtype), t(case.v_prefix, dtype))
    layer.append_only(t(case.k_chunk, dtype), t(case.v_chunk, dtype))
    k, v = layer.read()
    total = case.prefix + case.chunk
    mask = torch.arange(total)[None, :] <= (case.prefix + torch.arange(case.chunk))[:, None]
    out = F.scaled_dot_product_attention(q, k.repeat_interleave(group, dim=1), v.repeat_interleave(group, dim=1),
                                         attn_mask=mask[None, None])
    return f32(out)


def gen_prefill() -> None:
    for name in cases.PREFILL_CASES:
        case = cases.prefill_case(name)
        out32 = run_prefill(case, torch.float32)
        out16 = run_prefill(case, torch.bfloat16)
        np.savez_compressed(HERE / f"{name}.npz", out_f32=out32, out_bf16=out16,
                            block_table=case.block_table().astype(np.int32), checksum=np.float64(case.checksum()))
        print(name, out32.shape)


def gen_storage_sequence() -> None:
    """Known-answer append/read sequence modelled on the reference's storage
    tests (tests/test_paged_kv_cache.py:28-136): block_size 2, head_dim 3,
    arange keys, values = keys + 100, block-boundary crossings, growth of a
    request's block list, two requests and two layers."""
    storage = PagedKVCache(num_layers=2, max_blocks=6, num_kv_heads=2, block_size=2, head_dim=3)
    storage.key_cache.fill_(SENTINEL)
    storage.value_cache.fill_(SENTINEL)
    pool = BlockPool(6)
    steps = []
    storage.register_request("A", pool.allocate(2))
    ka = torch.arange(18, dtype=torch.float32).reshape(1, 2, 3, 3)
    storage.get_cache("A").layer(0).append_only(ka, ka + 100)
    steps.append(("A", 0, 0, ka.numpy()))
    k1 = torch.arange(6, dtype=torch.float32).reshape(1, 2, 1, 3) + 50
    storage.get_cache("A").layer(1).append_only(k1, k1 + 100)
    steps.append(("A", 1, 0, k1.numpy()))
    storage.register_request("B", pool.allocate(1))
    kb = torch.full((1, 2, 2, 3), 2.0)
    storage.get_cache("B").layer(0).append_only(kb, kb + 100)
    steps.append(("B", 0, 0, kb.numpy()))
    blocks_a = storage.request_pages["A"].blocks + pool.allocate(1)
    storage.register_request("A", blocks_a)
    for i in range(2):
        kn = torch.arange(6, dtype=torch.float32).reshape(1, 2, 1, 3) * (i + 3)
        start = storage.get_cache("A").layer(0).seq_len
        storage.get_cache("A").layer(0).append_only(kn, kn + 100)
        steps.append(("A", 0, start, kn.numpy()))
    reads = {}
    for rid, layer in (("A", 0), ("A", 1), ("B", 0)):
        k, v = storage.get_cache(rid).layer(layer).read()
        reads[f"read_{rid}{layer}_k"] = k.numpy()
        reads[f"read_{rid}{layer}_v"] = v.numpy()
    tables = {f"table_{rid}": storage.request_pages[rid].block_table.numpy().astype(np.int32) for rid in ("A", "B")}
    np.savez_compressed(
        HERE / "storage_sequence.npz",
        key_cache=storage.key_cache.numpy(),
        value_cache=storage.value_cache.numpy(),
        step_rid=np.array([s[0] for s in steps]),
        step_layer=np.array([s[1] for s in steps], dtype=np.int32),
        step_start=np.array([s[2] for s in steps], dtype=np.int32),
        **{f"step{i}_key": s[3] for i, s in enumerate(steps)},
        **reads,
        **tables,
    )
    print("storage_sequence", [s[:3] for s in steps])


def gen_batch_read() -> None:
    """Boundary lengths 15..33 at block_size 16 (tests/test_benchmark_paged_cache.py:35-86)
    with the benchmark's pattern values; batched read zero-pads to the longest."""
    lengths = [15, 16, 17, 31, 32, 33]
    bs = 16
    max_blocks = sum((n + bs - 1) // bs for n in lengths)
    pool = BlockPool(max_blocks)
    storage = PagedKVCache(num_layers=2, max_blocks=max_blocks, num_kv_heads=2, block_size=bs, head_dim=3)
    storage.key_cache.fill_(SENTINEL)
    storage.value_cache.fill_(SENTINEL)
    manager = KVCacheManager(bs, pool, storage)
    caches = []
    for i, n in enumerate(lengths):
        req = Request(id=f"b{i}", token_ids=torch.zeros((1, n), dtype=torch.long))
        assert manager.allocate_request(req)
        cache = manager.get_cache(req)
        for layer in range(2):
            key = t(cases.pattern_tensor(i, layer, n, 2, 3, 0.0))
            value = t(cases.pattern_tensor(i, layer, n, 2, 3, 0.5))
            cache.layer(layer).append_only(key, value)
        caches.append(cache)
    out = {}
    for layer in range(2):
        batch_layer = BatchKVCache(caches).layer(layer)
        k, v = batch_layer.read()
        out[f"k{layer}"] = k.numpy()
        out[f"v{layer}"] = v.numpy()
        out[f"mask{layer}"] = batch_layer.attention_mask(1).numpy()
    tables = padded_tables([storage.request_pages[f"b{i}"].block_table.numpy() for i in range(len(lengths))])
    np.savez_compressed(HERE / "batch_read.npz", lengths=np.array(lengths, dtype=np.int32), block_tables=tables,
                        key_cache=storage.key_cache.numpy(), value_cache=storage.value_cache.numpy(), **out)
    print("batch_read", tables.shape)


def run_qk_prep(case: cases.QkPrepCase, dtype: torch.dtype) -> dict:
    """The reference's QK-norm + RoPE (models/attention.py:161-169) on the case."""
    d = case.head_dim
    q_norm = RMSNorm(d, eps=case.eps)
    k_norm = RMSNorm(d, eps=case.eps)
    with torch.no_grad():
        q_norm.weight.copy_(t(case.q_weight))
        k_norm.weight.copy_(t(case.k_weight))
    q_norm, k_norm = q_norm.to(dtype), k_norm.to(dtype)
    rope = RotaryEmbedding(d, theta=case.theta)
    q, k = t(case.q, dtype), t(case.k, dtype)
    with torch.no_grad():
        cos, sin = rope(q, torch.from_numpy(case.positions()))
        q_out = apply_rope(q_norm(q), cos, sin)
        k_out = apply_rope(k_norm(k), cos, sin)
    return {"q_out": f32(q_out), "k_out": f32(k_out), "cos": f32(cos), "sin": f32(sin),
            "q_weight": f32(q_norm.weight), "k_weight": f32(k_norm.weight)}


def gen_qk_prep() -> None:
    for name in cases.QK_PREP_CASES:
        case = cases.qk_prep_case(name)
        out = {}
        for tag, dtype in (("f32", torch.float32), ("bf16", torch.bfloat16)):
            for key, val in run_qk_prep(case, dtype).items():
                out[f"{key}_{tag}"] = val
        np.savez_compressed(HERE / f"{name}.npz", checksum=case.checksum(), **out)
        print(name, out["q_out_f32"].shape)


if __name__ == "__main__":
    torch.manual_seed(0)
    gen_storage_sequence()
    gen_batch_read()
    gen_decode()
    gen_prefill()
    gen_qk_prep()
