"""Seeded synthetic inputs shared by the golden generator and the tests.

Inputs come from ``numpy.random.RandomState`` (stable across numpy versions),
so the fixtures only store the reference's outputs plus a checksum of the
inputs that produced them.  Shapes follow the workloads the reference's
paged-cache path is exercised on (Qwen3-0.6B attention: 16 query heads, 8 KV
heads, head_dim 128, block_size 16; Qwen3-8B attention: 32 / 8 / 128 / 16).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def pattern_tensor(request_index: int, layer_index: int, length: int, num_kv_heads: int, head_dim: int,
                   offset: float) -> np.ndarray:
    """The deterministic ``(i % 97) / 97 + request + layer + offset`` K/V pattern
    of the reference's paged-cache benchmark (examples/benchmark_paged_cache.py:71-85),
    ``[1, H, T, D]`` float32."""
    count = num_kv_heads * length * head_dim
    values = (np.arange(count, dtype=np.float32) % 97) / np.float32(97.0) + request_index + layer_index
    return (values.reshape(1, num_kv_heads, length, head_dim) + np.float32(offset)).astype(np.float32)


@dataclass
class DecodeCase:
    """One batched decode step over a shuffled paged pool.

    Each request already holds ``lengths[b]`` tokens (its history) and appends
    one more; ``free_ids`` is the pool's free list (``BlockPool.free_ids``),
    from whose end blocks are popped as the reference's BlockPool does
    (src/barellm/engine/block_pool.py:17-24)."""

    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    lengths: np.ndarray          # [B] history lengths (pre-append)
    free_ids: np.ndarray         # [P] free list
    k_hist: list[np.ndarray]     # [1, Hkv, len_b, D] float32
    v_hist: list[np.ndarray]
    k_new: np.ndarray            # [B, Hkv, 1, D]
    v_new: np.ndarray
    q: np.ndarray                # [B, Hq, 1, D]

    @property
    def batch(self) -> int:
        return len(self.lengths)

    def block_tables(self) -> list[np.ndarray]:
        """Blocks each request owns after allocating for len+1 tokens, in the
        order the reference's KVCacheManager registers them."""
        free = list(int(x) for x in self.free_ids)
        tables = []
        for n in self.lengths:
            need = (int(n) + 1 + self.block_size - 1) // self.block_size
            tables.append(np.array([free.pop() for _ in range(need)], dtype=np.int64))
        return tables

    def checksum(self) -> float:
        tot = float(np.abs(self.q).sum() + np.abs(self.k_new).sum() + np.abs(self.v_new).sum())
        tot += sum(float(np.abs(k).sum() + np.abs(v).sum()) for k, v in zip(self.k_hist, self.v_hist))
        return tot


def make_decode_case(seed: int, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                     block_size: int, num_blocks: int, len_lo: int, len_hi: int,
                     scale: float = 1.0) -> DecodeCase:
    """Lengths ~ U{len_lo..len_hi}, free list a random permutation, Q/K/V ~ N(0,1)*scale."""
    rs = np.random.RandomState(seed)
    lengths = rs.randint(len_lo, len_hi + 1, size=batch).astype(np.int64)
    free_ids = rs.permutation(num_blocks).astype(np.int64)
    k_hist, v_hist = [], []
    for n in lengths:
        k_hist.append((rs.standard_normal((1, num_kv_heads, int(n), head_dim)) * scale).astype(np.float32))
        v_hist.append((rs.standard_normal((1, num_kv_heads, int(n), head_dim)) * scale).astype(np.float32))
    k_new = (rs.standard_normal((batch, num_kv_heads, 1, head_dim)) * scale).astype(np.float32)
    v_new = (rs.standard_normal((batch, num_kv_heads, 1, head_dim)) * scale).astype(np.float32)
    q = (rs.standard_normal((batch, num_q_heads, 1, head_dim)) * scale).astype(np.float32)
    return DecodeCase(num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, lengths, free_ids,
                      k_hist, v_hist, k_new, v_new, q)


@dataclass
class PrefillCase:
    """One request: a paged prefix of ``prefix`` tokens plus a new chunk of
    ``chunk`` tokens that is appended and then attends causally (bottom-right)."""

    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    prefix: int
    chunk: int
    free_ids: np.ndarray
    k_prefix: np.ndarray   # [1, Hkv, prefix, D]
    v_prefix: np.ndarray
    k_chunk: np.ndarray    # [1, Hkv, chunk, D]
    v_chunk: np.ndarray
    q: np.ndarray          # [1, Hq, chunk, D]

    def block_table(self) -> np.ndarray:
        free = list(int(x) for x in self.free_ids)
        need = (self.prefix + self.chunk + self.block_size - 1) // self.block_size
        return np.array([free.pop() for _ in range(need)], dtype=np.int64)

    def checksum(self) -> float:
        return float(sum(np.abs(x).sum() for x in (self.k_prefix, self.v_prefix, self.k_chunk,
                                                    self.v_chunk, self.q)))


def make_prefill_case(seed: int, num_q_heads: int, num_kv_heads: int, head_dim: int, block_size: int,
                      num_blocks: int, prefix: int, chunk: int) -> PrefillCase:
    rs = np.random.RandomState(seed)
    free_ids = rs.permutation(num_blocks).astype(np.int64)

    def randn(*shape):
        return rs.standard_normal(shape).astype(np.float32)

    return PrefillCase(num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, prefix, chunk, free_ids,
                       randn(1, num_kv_heads, prefix, head_dim), randn(1, num_kv_heads, prefix, head_dim),
                       randn(1, num_kv_heads, chunk, head_dim), randn(1, num_kv_heads, chunk, head_dim),
                       randn(1, num_q_heads, chunk, head_dim))


# ---------------------------------------------------------------------------
# the fixture set
# ---------------------------------------------------------------------------
DECODE_CASES = {
    # name: (seed, B, Hq, Hkv, D, bs, P, len_lo, len_hi)
    "decode_tiny_mha": (11, 3, 4, 4, 8, 4, 64, 1, 21),
    "decode_tiny_gqa": (12, 3, 4, 2, 8, 4, 64, 1, 21),
    "decode_tiny_mqa": (13, 3, 4, 1, 8, 4, 64, 1, 21),
    # Qwen3-0.6B attention, 4 requests, lengths U{1..512}, 4096-block pool
    "decode_qwen06b_b4": (0, 4, 16, 8, 128, 16, 4096, 1, 512),
    # Qwen3-8B attention (G=4), lengths long enough to need split-K
    "decode_qwen8b_b3": (1, 3, 32, 8, 128, 16, 2048, 600, 1800),
}

PREFILL_CASES = {
    # name: (seed, Hq, Hkv, D, bs, P, prefix, chunk)
    "prefill_tiny": (21, 4, 2, 8, 4, 32, 0, 11),
    "prefill_qwen06b": (22, 16, 8, 128, 16, 64, 0, 37),
    "chunked_prefill_tiny": (23, 4, 2, 8, 4, 64, 13, 9),
    "chunked_prefill_qwen8b": (24, 32, 8, 128, 16, 128, 150, 77),
}


def decode_case(name: str) -> DecodeCase:
    seed, b, hq, hkv, d, bs, p, lo, hi = DECODE_CASES[name]
    return make_decode_case(seed, b, hq, hkv, d, bs, p, lo, hi)


def prefill_case(name: str) -> PrefillCase:
    seed, hq, hkv, d, bs, p, prefix, chunk = PREFILL_CASES[name]
    return make_prefill_case(seed, hq, hkv, d, bs, p, prefix, chunk)


# ---------------------------------------------------------------------------
# QK-RMSNorm + RoPE + append (the step before the attention)
# ---------------------------------------------------------------------------
@dataclass
class QkPrepCase:
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    eps: float
    theta: float
    starts: np.ndarray     # [B] cached tokens before this step
    free_ids: np.ndarray
    q: np.ndarray          # [B, Hq, T, D] projections before the norm
    k: np.ndarray          # [B, Hkv, T, D]
    v: np.ndarray
    q_weight: np.ndarray   # [D]
    k_weight: np.ndarray

    @property
    def batch(self) -> int:
        return self.q.shape[0]

    @property
    def new_tokens(self) -> int:
        return self.q.shape[2]

    def positions(self) -> np.ndarray:
        return self.starts[:, None] + np.arange(self.new_tokens)[None, :]

    def block_tables(self) -> list[np.ndarray]:
        free = list(int(x) for x in self.free_ids)
        out = []
        for s in self.starts:
            need = (int(s) + self.new_tokens + self.block_size - 1) // self.block_size
            out.append(np.array([free.pop() for _ in range(need)], dtype=np.int64))
        return out

    def checksum(self) -> float:
        return float(sum(np.abs(x).sum() for x in (self.q, self.k, self.v, self.q_weight, self.k_weight)))


def make_qk_prep_case(seed: int, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int, block_size: int,
                      num_blocks: int, new_tokens: int, max_start: int) -> QkPrepCase:
    rs = np.random.RandomState(seed)
    starts = rs.randint(0, max_start + 1, size=batch).astype(np.int64)
    free_ids = rs.permutation(num_blocks).astype(np.int64)

    def randn(*shape, scale=1.0):
        return (rs.standard_normal(shape) * scale).astype(np.float32)

    return QkPrepCase(num_q_heads, num_kv_heads, head_dim, block_size, num_blocks, 1e-6, 1_000_000.0, starts,
                      free_ids, randn(batch, num_q_heads, new_tokens, head_dim, scale=2.0),
                      randn(batch, num_kv_heads, new_tokens, head_dim, scale=2.0),
                      randn(batch, num_kv_heads, new_tokens, head_dim),
                      (1.0 + 0.1 * rs.standard_normal(head_dim)).astype(np.float32),
                      (1.0 + 0.1 * rs.standard_normal(head_dim)).astype(np.float32))


QK_PREP_CASES = {
    # name: (seed, B, Hq, Hkv, D, bs, P, T, max_start)
    "qk_prep_tiny": (31, 2, 4, 2, 64, 4, 64, 3, 20),
    # Qwen3-0.6B attention shapes: one decode token per request, long positions
    "qk_prep_qwen06b_decode": (32, 5, 16, 8, 128, 16, 4096, 1, 12000),
    # Qwen3-8B attention shapes: a short prefill chunk over a prefix
    "qk_prep_qwen8b_chunk": (33, 2, 32, 8, 128, 16, 512, 19, 300),
}


def qk_prep_case(name: str) -> QkPrepCase:
    seed, b, hq, hkv, d, bs, p, t, max_start = QK_PREP_CASES[name]
    return make_qk_prep_case(seed, b, hq, hkv, d, bs, p, t, max_start)
