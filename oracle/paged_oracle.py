"""CPU oracle for the paged-KV hot path.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference`` arm) may import this module, and
only as the checker or the timed CPU baseline.  The product path
(``barellm_b200``) never calls it.

It restates, in numpy, the reference's own algorithm for every step of the
path (quanhua92/barellm, file:line cited per function).  Copies are exact;
attention is evaluated in float64 from the stored element values, following
the semantics of ``torch.nn.functional.scaled_dot_product_attention`` (a
third-party dependency of the reference, pinned at torch 2.6.0 in
``uv.lock:51``; its call sites are src/barellm/attention/backend.py:55-61 and
examples/benchmark_paged_cache.py:248-254).

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here
against golden vectors that ``tests/golden/make_golden.py`` produced by running
the reference's own classes (PagedKVCache, BatchKVCache, SDPAAttentionBackend).
"""

from __future__ import annotations

import numpy as np


def positions_to_slots(block_table: np.ndarray, start: int, end: int, block_size: int):
    """Logical positions -> (physical block, offset); paged_kv_cache.py:176-181."""
    pos = np.arange(start, end, dtype=np.int64)
    logical = pos // block_size
    offsets = pos % block_size
    return np.asarray(block_table, dtype=np.int64)[logical], offsets


def append_only(key_cache, value_cache, layer, block_table, start, key, value) -> int:
    """PagedLayerKV.append_only, src/barellm/engine/paged_kv_cache.py:151-193.

    ``key``/``value``: [1, H, T, D].  Writes token t of every head into
    ``cache[layer, phys(start+t), :, off(start+t), :]``; returns the new length.
    """
    if key.ndim != 4 or key.shape != value.shape or key.shape[0] != 1:
        raise ValueError("K/V must have shape [1, H, T, D]")
    t = key.shape[2]
    if t <= 0:
        raise ValueError("K/V sequence length must be greater than zero")
    bs = key_cache.shape[3]
    end = start + t
    if (end + bs - 1) // bs > len(block_table):
        raise ValueError("request does not have enough allocated KV blocks")
    phys, off = positions_to_slots(block_table, start, end, bs)
    key_cache[layer, phys, :, off, :] = np.transpose(key[0], (1, 0, 2))
    value_cache[layer, phys, :, off, :] = np.transpose(value[0], (1, 0, 2))
    return end


def read(key_cache, value_cache, layer, block_table, seq_len):
    """PagedLayerKV.read, src/barellm/engine/paged_kv_cache.py:215-240 -> [1, H, T, D] x2."""
    if seq_len <= 0:
        raise ValueError("KV cache is empty")
    phys, off = positions_to_slots(block_table, 0, seq_len, key_cache.shape[3])
    k = key_cache[layer, phys, :, off, :]  # [T, H, D]
    v = value_cache[layer, phys, :, off, :]
    return np.transpose(k, (1, 0, 2))[None], np.transpose(v, (1, 0, 2))[None]


def batch_read_pad(key_cache, value_cache, layer, block_tables, seq_lens):
    """BatchLayerKV.read + _pad, src/barellm/engine/batched_kv_cache.py:65-95.

    Zero-padded dense ``[B, H, Tmax, D]`` K and V."""
    tmax = max(int(x) for x in seq_lens)
    b = len(seq_lens)
    _, _, h, _, d = key_cache.shape
    k_out = np.zeros((b, h, tmax, d), dtype=key_cache.dtype)
    v_out = np.zeros_like(k_out)
    for row, (bt, n) in enumerate(zip(block_tables, seq_lens)):
        k, v = read(key_cache, value_cache, layer, bt, int(n))
        k_out[row, :, : int(n)] = k[0]
        v_out[row, :, : int(n)] = v[0]
    return k_out, v_out


def attention_mask(seq_lens, q_len: int) -> np.ndarray:
    """BatchLayerKV.attention_mask, src/barellm/engine/batched_kv_cache.py:97-102.

    ``[B, 1, q_len, Tmax]`` bool, True where the key exists."""
    lens = np.asarray(seq_lens, dtype=np.int64)
    valid = np.arange(int(lens.max()))[None, :] < lens[:, None]
    return np.broadcast_to(valid[:, None, None, :], (len(lens), 1, q_len, valid.shape[1]))


def repeat_kv(x: np.ndarray, group: int) -> np.ndarray:
    """``repeat_interleave(group, dim=1)``: query head h reads KV head h // group
    (src/barellm/attention/backend.py:47-48)."""
    return np.repeat(x, group, axis=1)


def sdpa(q, k, v, attn_mask=None, is_causal=False, scale=None) -> np.ndarray:
    """Scaled dot-product attention in float64.

    softmax(q k^T * scale [+ -inf where the bool mask is False or, with
    is_causal, above the upper-left aligned diagonal]) @ v; scale defaults to
    1/sqrt(D).  Returns float64 ``[B, H, Lq, D]``."""
    q = q.astype(np.float64)
    k = k.astype(np.float64)
    v = v.astype(np.float64)
    d = q.shape[-1]
    s = (1.0 / np.sqrt(d)) if scale is None else scale
    logits = np.einsum("bhqd,bhkd->bhqk", q, k) * s
    lq, lk = q.shape[-2], k.shape[-2]
    if is_causal:
        causal = np.tril(np.ones((lq, lk), dtype=bool))
        logits = np.where(causal, logits, -np.inf)
    if attn_mask is not None:
        logits = np.where(attn_mask, logits, -np.inf)
    m = logits.max(axis=-1, keepdims=True)
    p = np.exp(logits - m)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v)


def decode_attention(q, key_cache, value_cache, layer, block_tables, seq_lens, scale=None):
    """The batched decode step of SDPAAttentionBackend.attend after the append
    (src/barellm/attention/backend.py:34-61 with a BatchLayerKV cache):
    read + pad -> repeat_interleave(G) -> padding mask -> SDPA.

    ``q``: [B, Hq, 1, D]; ``seq_lens`` are post-append lengths.  float64 out."""
    k, v = batch_read_pad(key_cache, value_cache, layer, block_tables, seq_lens)
    group = q.shape[1] // k.shape[1]
    mask = attention_mask(seq_lens, q.shape[2])
    return sdpa(q, repeat_kv(k, group), repeat_kv(v, group), attn_mask=mask, scale=scale)


def causal_mask_bottom_right(q_len: int, k_len: int) -> np.ndarray:
    """Query i of a chunk that ends at key k_len-1 sees keys 0 .. k_len-q_len+i."""
    return np.arange(k_len)[None, :] <= (k_len - q_len + np.arange(q_len))[:, None]


def prefill_attention(q, key_cache, value_cache, layer, block_table, seq_len, scale=None):
    """Prefill / chunked prefill of one request after its append.

    Empty prefix: the reference prefill, SDPA(is_causal=True) over the appended
    K/V (src/barellm/attention/backend.py:52-61, engine.py:226-257).  Non-empty
    prefix (chunked prefill, which the reference lists as future work in
    docs/ROADMAP.md:131): the dense read (paged_kv_cache.py:215-240) +
    repeat_interleave + SDPA with the bottom-right aligned causal mask.
    ``q``: [1, Hq, C, D].  float64 out."""
    k, v = read(key_cache, value_cache, layer, block_table, seq_len)
    group = q.shape[1] // k.shape[1]
    c = q.shape[2]
    mask = causal_mask_bottom_right(c, seq_len)[None, None]
    return sdpa(q, repeat_kv(k, group), repeat_kv(v, group), attn_mask=mask, scale=scale)


def _identity(x):
    return x


def rms_norm(x, weight, eps: float, round_fn=None) -> np.ndarray:
    """RMSNorm over the last axis; models/norm.py:14-21 (mean square, rsqrt
    and the weight in float; one rounding to the element type at the end)."""
    rnd = round_fn or _identity
    xf = np.asarray(x, dtype=np.float64)
    ms = np.mean(xf * xf, axis=-1, keepdims=True)
    return rnd(xf / np.sqrt(ms + eps) * np.asarray(weight, dtype=np.float64))


def rotate_half(x: np.ndarray) -> np.ndarray:
    """models/rope.py:53-60: cat(-x[..., D/2:], x[..., :D/2])."""
    half = x.shape[-1] // 2
    return np.concatenate((-x[..., half:], x[..., :half]), axis=-1)


def apply_rope(x, cos, sin, round_fn=None) -> np.ndarray:
    """models/rope.py:63-68: x * cos + rotate_half(x) * sin, each tensor op
    rounded to the element type (``round_fn``)."""
    rnd = round_fn or _identity
    x = np.asarray(x, dtype=np.float64)
    return rnd(rnd(x * cos) + rnd(rotate_half(x) * sin))


def qk_norm_rope(x, weight, cos, sin, eps: float, round_fn=None) -> np.ndarray:
    """apply_rope(norm(x), cos, sin); models/attention.py:161-169."""
    return apply_rope(rms_norm(x, weight, eps, round_fn), cos, sin, round_fn)


def decode_attention_rows(q, k_rows, v_rows, scale=None):
    """Decode attention from per-row dense histories (the pool already gathered).

    ``q``: [B, Hq, D]; ``k_rows[b]``/``v_rows[b]``: [Hkv, len_b, D].  Used for
    large parity cases where materialising a padded batch is wasteful."""
    out = np.empty(q.shape, dtype=np.float64)
    for b in range(q.shape[0]):
        kb = k_rows[b].astype(np.float64)
        vb = v_rows[b].astype(np.float64)
        group = q.shape[1] // kb.shape[0]
        qb = q[b].astype(np.float64).reshape(kb.shape[0], group, -1)  # [Hkv, G, D]
        s = (1.0 / np.sqrt(q.shape[-1])) if scale is None else scale
        logits = np.einsum("hgd,htd->hgt", qb, kb) * s
        logits -= logits.max(axis=-1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=-1, keepdims=True)
        out[b] = np.einsum("hgt,htd->hgd", p, vb).reshape(q.shape[1], -1)
    return out


# ---------------------------------------------------------------------------
# Timed CPU baseline (bench.py's cpu_baseline leg and --impl reference arm)
# ---------------------------------------------------------------------------
def _sdpa_f32(q, k, v, attn_mask):
    """float32 SDPA with a bool padding mask, as the reference runs on a CPU."""
    d = q.shape[-1]
    logits = np.einsum("bhqd,bhkd->bhqk", q, k, optimize=True) * np.float32(1.0 / np.sqrt(d))
    logits = np.where(attn_mask, logits, np.float32(-np.inf))
    logits -= logits.max(axis=-1, keepdims=True)
    p = np.exp(logits, dtype=np.float32)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhqk,bhkd->bhqd", p, v, optimize=True)


def decode_step_cpu(key_cache, value_cache, layer, block_tables, starts, q, k_new, v_new, executor=None,
                    rows_per_task: int = 1):
    """One batched decode step exactly as the reference runs it on a CPU, in
    float32: per-row append (paged_kv_cache.py:151-193), dense read + zero pad
    (batched_kv_cache.py:65-95), repeat_interleave (backend.py:47-48), padding
    mask (batched_kv_cache.py:97-102) and SDPA (backend.py:55-61).

    Rows are split into independent groups that run on ``executor``'s threads
    (each group pads to its own longest row, which changes no result).
    Returns ``[B, Hq, 1, D]`` float32."""
    b = q.shape[0]
    for r in range(b):
        append_only(key_cache, value_cache, layer, block_tables[r], int(starts[r]), k_new[r : r + 1], v_new[r : r + 1])
    lens = [int(s) + k_new.shape[2] for s in starts]
    group = q.shape[1] // key_cache.shape[2]

    def run(lo: int, hi: int):
        k, v = batch_read_pad(key_cache, value_cache, layer, block_tables[lo:hi], lens[lo:hi])
        mask = attention_mask(lens[lo:hi], q.shape[2])
        return lo, _sdpa_f32(q[lo:hi], repeat_kv(k, group), repeat_kv(v, group), mask)

    spans = [(i, min(i + rows_per_task, b)) for i in range(0, b, rows_per_task)]
    out = np.empty(q.shape, dtype=np.float32)
    results = executor.map(lambda s: run(*s), spans) if executor is not None else (run(*s) for s in spans)
    for lo, o in results:
        out[lo : lo + o.shape[0]] = o
    return out
