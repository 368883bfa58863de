"""Batched view over per-request paged caches for one decode step.

Interface of the reference's BatchKVCache / BatchLayerKV
(src/barellm/engine/batched_kv_cache.py:8-145).  The reference loops over rows
in Python for every layer (one append and one gather per row) and rebuilds
lengths and block tables on each call.  Here the batch resolves its requests
to arena rows once; per layer, lengths and capacity checks are numpy array
operations on the pool's length table, the step's metadata (arena rows,
pre-append and post-append lengths) reaches the device in one pinned copy the
first time any layer needs it and is shared by every layer of the step, and
the split-K decode plan built from it is shared the same way.  Appends and
reads are one kernel launch for the whole batch.
"""

from __future__ import annotations

from operator import attrgetter

import numpy as np
import torch

from . import ops
from .paged_kv_cache import PagedBatchKVMetadata, PagedKVCache, PagedKVCacheView, PagedLayerKV, check


_STORAGE = attrgetter("storage")
_REQUEST_ID = attrgetter("request_id")


class StepMeta:
    """Device metadata for one (pre-append lengths, new tokens) combination.

    With ``static_max_seq_len`` the device buffers are allocated once and
    ``refresh`` rewrites them in place (one pinned host-to-device copy), so a
    captured CUDA graph that reads them stays valid from step to step;
    ``max_seq_len`` is then the fixed bound the graph was captured with.

    ``renew`` reuses the object for the next step of the same batch: the
    device buffers are kept and the new lengths go in with one copy from a
    fresh pinned buffer (the pinned allocator does not hand that memory out
    again before the copy has run)."""

    def __init__(self, storage: PagedKVCache, rows: np.ndarray, starts: np.ndarray, new_tokens: int,
                 static_max_seq_len: int | None = None) -> None:
        self._pin = storage.device.type == "cuda"
        self._rows = rows
        host = self._fill(starts, new_tokens)
        self._dev = host.to(storage.device, non_blocking=True)
        self.rows, self.starts, self.seq_lens = self._dev.unbind(0)
        self.static = static_max_seq_len is not None
        self.max_seq_len = int(static_max_seq_len) if self.static else int(self.seq_lens_host.max())
        self.new_tokens = new_tokens
        self.version = 0  # bumped by renew
        self.plan_ws: torch.Tensor | None = None
        self.plan_heads = 0
        self.plan_token = -1

    def _fill(self, starts: np.ndarray, new_tokens: int) -> torch.Tensor:
        host = torch.empty((3, len(self._rows)), dtype=torch.int32, pin_memory=self._pin)
        h = host.numpy()
        h[0] = self._rows
        h[1] = starts
        np.add(starts, new_tokens, out=h[2], casting="unsafe")
        self._host = host
        self.seq_lens_host = h[2].astype(np.int64)
        return host

    def matches(self, starts: np.ndarray, new_tokens: int) -> bool:
        h = self._host.numpy()
        return new_tokens == self.new_tokens and np.array_equal(h[1], starts)

    def renew(self, starts: np.ndarray, new_tokens: int) -> None:
        """The next step's lengths into the same device buffers (same rows)."""
        self._dev.copy_(self._fill(starts, new_tokens), non_blocking=True)
        self.max_seq_len = int(self.seq_lens_host.max())
        self.new_tokens = new_tokens
        self.version += 1
        self.plan_ws = None  # the lengths changed: the plan must be rebuilt

    def stage(self, starts: np.ndarray, new_tokens: int) -> None:
        """Static mode, for graph replay: write the next step's lengths into the
        pinned host buffer only; the captured copy moves them to the device."""
        h = self._host.numpy()
        h[1] = starts
        h[2] = starts + new_tokens
        self.seq_lens_host = h[2].astype(np.int64)
        check(int(self.seq_lens_host.max()) <= self.max_seq_len, "sequence grew past the captured bound")

    def refresh(self, starts: np.ndarray, new_tokens: int) -> None:
        """Static mode: new lengths into the same device buffers (one copy)."""
        h = self._host.numpy()
        h[1] = starts
        h[2] = starts + new_tokens
        self.seq_lens_host = h[2].astype(np.int64)
        check(int(self.seq_lens_host.max()) <= self.max_seq_len, "sequence grew past the captured bound")
        self.new_tokens = new_tokens
        self._dev.copy_(self._host, non_blocking=True)
        self.plan_ws = None  # the lengths changed: the plan must be rebuilt


class BatchKVCache:
    """``static_max_seq_len``: keep one set of device metadata buffers for the
    life of this view (refreshed in place each step) so the decode step can be
    captured in a CUDA graph; lengths may not exceed the bound.

    Without it, a batch over the same requests as an earlier batch (the
    engine builds a new BatchKVCache every decode step) reuses that batch's
    device metadata buffers, renewed with the new lengths."""

    def __init__(self, caches: list[PagedKVCacheView], *, static_max_seq_len: int | None = None) -> None:
        check(len(caches) > 0, "batch cache cannot be empty")
        self.caches = caches
        self._meta: dict[tuple[bytes, int], tuple[StepMeta, int]] = {}
        self._static: StepMeta | None = None
        self._rowset = None
        first = getattr(caches[0], "storage", None)
        self.storage: PagedKVCache | None = None
        if (isinstance(first, PagedKVCache) and all(issubclass(t, PagedKVCacheView) for t in set(map(type, caches)))
                and set(map(_STORAGE, caches)) == {first}):
            self.storage = first
            self._rowset = first.row_set(tuple(map(_REQUEST_ID, caches)))
            self.rows = self._rowset.rows
            if static_max_seq_len is not None:
                zeros = np.zeros(len(caches), dtype=np.int64)
                self._static = StepMeta(first, self.rows, zeros, 0, static_max_seq_len=static_max_seq_len)

    def layer(self, layer_idx: int) -> "BatchLayerKV":
        if self.storage is not None and not 0 <= layer_idx < self.storage.num_layers:
            raise IndexError(f"Invalid layer index: {layer_idx}")
        return BatchLayerKV(None, owner=self, layer_idx=layer_idx)

    def step_meta(self, starts: np.ndarray, new_tokens: int) -> StepMeta:
        if self._static is not None:
            if not self._static.matches(starts, new_tokens):
                self._static.refresh(starts, new_tokens)
            return self._static
        key = (starts.tobytes(), new_tokens)
        hit = self._meta.get(key)
        if hit is not None and hit[0].version == hit[1]:
            return hit[0]
        rs = self._rowset
        shared = rs.meta
        if shared is None:
            meta = rs.meta = StepMeta(self.storage, self.rows, starts, new_tokens)
        elif hit is None and shared.matches(starts, new_tokens):
            meta = shared
        elif hit is None:
            shared.renew(starts, new_tokens)
            meta = shared
        else:
            # this batch's buffers were renewed by another batch over the same
            # requests since: keep a private copy for the rest of this step
            meta = StepMeta(self.storage, self.rows, starts, new_tokens)
        self._meta = {key: (meta, meta.version)}  # one live step per batch view
        return meta


class BatchLayerKV:
    """One layer of a BatchKVCache.  ``BatchLayerKV(layers)`` also accepts a
    list of PagedLayerKV of one layer, as the reference's constructor does."""

    def __init__(self, layers: list[PagedLayerKV] | None, owner: BatchKVCache | None = None,
                 layer_idx: int | None = None) -> None:
        if owner is None:
            check(layers is not None and len(layers) > 0, "batch cache cannot be empty")
            if not all(isinstance(l, PagedLayerKV) for l in layers):
                raise TypeError("paged metadata requires PagedLayerKV members")
            owner = BatchKVCache([PagedKVCacheView(l.storage, l.request_id) for l in layers])
            layer_idx = layers[0].layer_idx
            if any(l.layer_idx != layer_idx for l in layers):
                raise ValueError("paged batch layers must share storage and layout")
        self.owner = owner
        self.layer_idx = int(layer_idx)
        self._layers = layers

    # -- helpers -------------------------------------------------------------
    @property
    def layers(self) -> list:
        if self._layers is None:
            self._layers = [c.layer(self.layer_idx) for c in self.owner.caches]
        return self._layers

    def storage(self) -> PagedKVCache:
        """The single paged pool every member must share (TypeError otherwise)."""
        s = self.owner.storage
        if s is None:
            raise TypeError("paged metadata requires PagedLayerKV members sharing one PagedKVCache")
        return s

    def starts(self) -> np.ndarray:
        s = self.storage()
        return s.arena.lens[self.owner.rows, self.layer_idx]

    def meta(self, new_tokens: int) -> StepMeta:
        return self.owner.step_meta(self.starts(), new_tokens)

    @property
    def lengths(self) -> torch.Tensor:
        return torch.from_numpy(self.starts().copy())

    @property
    def seq_len(self) -> int:
        return int(self.starts().max())

    # -- reference interface ---------------------------------------------------
    def append(self, key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.append_only(key, value)
        return self.read()

    def _begin_append(self, key: torch.Tensor, value: torch.Tensor):
        b = len(self.owner.caches)
        check(key.shape[0] == b, "batch size must match number of caches")
        check(value.shape[0] == b, "batch size must match number of caches")
        s = self.storage()
        s.check_new_kv(key, value, batch=b)
        t = key.shape[2]
        rows = self.owner.rows
        starts = s.arena.lens[rows, self.layer_idx]
        ends = starts + t
        # ceil(end / bs) <= blocks  <=>  end <= blocks * bs
        check(bool((ends <= s.arena.used[rows] * s.block_size).all()), "request does not have enough allocated KV blocks")
        return s, rows, ends, self.owner.step_meta(starts, t)

    def append_only(self, key: torch.Tensor, value: torch.Tensor) -> StepMeta:
        """One scatter kernel for every row (reference: a Python loop of
        per-row appends, batched_kv_cache.py:40-63).  Returns the step metadata
        whose ``seq_lens`` are the post-append lengths."""
        s, rows, ends, meta = self._begin_append(key, value)
        ops.paged_append(s.key_cache, s.value_cache, self.layer_idx, s.arena.table, meta.starts, key, value,
                         row_ids=meta.rows, err=s.err)
        s.arena.lens[rows, self.layer_idx] = ends
        return meta

    def append_only_prepped(self, q: torch.Tensor, key: torch.Tensor, value: torch.Tensor, q_norm_weight,
                            k_norm_weight, cos, sin, eps: float) -> tuple[StepMeta, torch.Tensor]:
        """append_only of the QK-normalised, rotated key, with the same norm and
        rotation applied to ``q``, in one kernel (see
        ``ops.qk_norm_rope_append``).  Returns the step metadata and the
        prepared q."""
        s, rows, ends, meta = self._begin_append(key, value)
        q_out = ops.qk_norm_rope_append(q, key, value, q_norm_weight, k_norm_weight, cos, sin, eps, s.key_cache,
                                        s.value_cache, self.layer_idx, s.arena.table, meta.starts,
                                        row_ids=meta.rows, err=s.err)
        s.arena.lens[rows, self.layer_idx] = ends
        return meta, q_out

    def current_meta(self) -> StepMeta:
        """Metadata whose post-append lengths equal the current lengths."""
        cur = self.starts()
        st = self.owner._static
        if st is not None and np.array_equal(st.seq_lens_host, cur):
            return st
        for meta, version in self.owner._meta.values():
            if meta.version == version and np.array_equal(meta.seq_lens_host, cur):
                return meta
        return self.owner.step_meta(cur, 0)

    def read(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense zero-padded ``[B, H, Tmax, D]`` K and V (batched_kv_cache.py:65-95)."""
        check(bool((self.starts() > 0).all()), "KV cache is empty")
        s = self.storage()
        meta = self.current_meta()
        return ops.paged_gather(s.key_cache, s.value_cache, self.layer_idx, s.arena.table, meta.seq_lens,
                                meta.max_seq_len, row_ids=meta.rows, err=s.err)

    def attention_mask(self, q_len: int) -> torch.Tensor:
        """``[B, 1, q_len, Tmax]`` valid-key mask (batched_kv_cache.py:97-102)."""
        s = self.storage()
        lens = torch.from_numpy(self.starts().copy()).to(s.device)
        valid = torch.arange(int(lens.max()), device=s.device).unsqueeze(0) < lens.unsqueeze(1)
        return valid[:, None, None, :].expand(-1, 1, q_len, -1)

    def paged_metadata_post_append(self) -> PagedBatchKVMetadata:
        """Rectangular int32 block tables padded with -1 and int32 post-append
        lengths (batched_kv_cache.py:104-145), gathered from the arena."""
        s = self.storage()
        check(bool((self.starts() > 0).all()), "KV cache is empty")
        meta = self.current_meta()
        counts = s.arena.used[self.owner.rows]
        width = int(counts.max())
        tables = s.arena.table.index_select(0, meta.rows.long())[:, :width].clone()
        col = torch.arange(width, device=s.device).unsqueeze(0)
        limit = torch.from_numpy(counts.copy()).to(s.device).unsqueeze(1)
        tables.masked_fill_(col >= limit, -1)
        return PagedBatchKVMetadata(s.key_cache, s.value_cache, self.layer_idx, tables, meta.seq_lens.clone(),
                                    s.block_size)


class PackedBatchKVCache:
    """Several requests appending a ragged run of tokens each (batched,
    chunked prefill), packed on the token axis: row b's ``chunk_lens[b]`` new
    tokens are tokens ``offsets[b] .. offsets[b+1]`` of a ``[1, H, sum, D]``
    tensor.  The reference prefills one request per forward with an empty
    cache (src/barellm/engine/engine.py:187-310); this view lets one forward
    prefill many requests, each continuing from whatever its cache already
    holds (a chunk of a long prompt over its earlier chunks).

    Every layer of one forward appends the same runs, so the device metadata
    (arena rows, offsets, pre- and post-append lengths) is built once and
    shared by all layers."""

    def __init__(self, caches: list[PagedKVCacheView], chunk_lens: list[int]) -> None:
        check(len(caches) > 0 and len(caches) == len(chunk_lens), "one chunk length per request")
        check(all(n > 0 for n in chunk_lens), "K/V sequence length must be greater than zero")
        storage = caches[0].storage
        if not all(isinstance(c, PagedKVCacheView) and c.storage is storage for c in caches):
            raise TypeError("packed prefill requires PagedKVCacheView members sharing one PagedKVCache")
        self.caches = caches
        self.storage = storage
        pages = storage.request_pages
        self.rows = storage.rows_for(tuple(map(_REQUEST_ID, caches)))
        self.chunk_lens = np.asarray(chunk_lens, dtype=np.int64)
        self.total = int(self.chunk_lens.sum())
        self.max_chunk = int(self.chunk_lens.max())
        self._meta: PackedStepMeta | None = None

    def layer(self, layer_idx: int) -> "PackedBatchLayerKV":
        if not 0 <= layer_idx < self.storage.num_layers:
            raise IndexError(f"Invalid layer index: {layer_idx}")
        return PackedBatchLayerKV(self, layer_idx)

    def step_meta(self, starts: np.ndarray) -> "PackedStepMeta":
        if self._meta is None or not np.array_equal(self._meta.starts_host, starts):
            self._meta = PackedStepMeta(self.storage, self.rows, starts, self.chunk_lens)
        return self._meta


class PackedStepMeta:
    """Device metadata of one packed step: rows, pre-append lengths,
    post-append lengths and token offsets, moved in one pinned copy."""

    def __init__(self, storage: PagedKVCache, rows: np.ndarray, starts: np.ndarray, chunk_lens: np.ndarray) -> None:
        b = len(rows)
        host = torch.empty((4, b + 1), dtype=torch.int32, pin_memory=storage.device.type == "cuda")
        h = host.numpy()
        h[0, :b] = rows
        h[1, :b] = starts
        h[2, :b] = starts + chunk_lens
        h[3, 0] = 0
        h[3, 1:] = np.cumsum(chunk_lens)
        dev = host.to(storage.device, non_blocking=True)
        self._host, self._dev = host, dev
        self.rows, self.starts, self.seq_lens, self.offsets = dev[0, :b], dev[1, :b], dev[2, :b], dev[3]
        self.starts_host = np.array(starts, dtype=np.int64)
        self.max_chunk = int(chunk_lens.max())


class PackedBatchLayerKV:
    """One layer of a PackedBatchKVCache."""

    def __init__(self, owner: PackedBatchKVCache, layer_idx: int) -> None:
        self.owner = owner
        self.layer_idx = int(layer_idx)

    def _begin(self, key: torch.Tensor, value: torch.Tensor) -> tuple[PagedKVCache, np.ndarray, PackedStepMeta]:
        o = self.owner
        s = o.storage
        check(key.ndim == 4 and key.shape[0] == 1 and key.shape[2] == o.total,
              "packed K/V must have shape [1, H, sum of chunk lengths, D]")
        check(value.shape == key.shape, "K/V must have identical shape")
        s.check_new_kv(key, value, batch=1)
        starts = s.arena.lens[o.rows, self.layer_idx]
        ends = starts + o.chunk_lens
        need = (ends + s.block_size - 1) // s.block_size
        check(bool((need <= s.arena.used[o.rows]).all()), "request does not have enough allocated KV blocks")
        return s, ends, o.step_meta(starts)

    def append_only(self, key: torch.Tensor, value: torch.Tensor) -> PackedStepMeta:
        s, ends, meta = self._begin(key, value)
        ops.paged_append(s.key_cache, s.value_cache, self.layer_idx, s.arena.table, meta.starts, key, value,
                         row_ids=meta.rows, new_offsets=meta.offsets, max_new_tokens=meta.max_chunk, err=s.err)
        s.arena.lens[self.owner.rows, self.layer_idx] = ends
        return meta

    def append_only_prepped(self, q: torch.Tensor, key: torch.Tensor, value: torch.Tensor, q_norm_weight,
                            k_norm_weight, cos, sin, eps: float) -> tuple[PackedStepMeta, torch.Tensor]:
        s, ends, meta = self._begin(key, value)
        q_out = ops.qk_norm_rope_append(q, key, value, q_norm_weight, k_norm_weight, cos, sin, eps, s.key_cache,
                                        s.value_cache, self.layer_idx, s.arena.table, meta.starts,
                                        row_ids=meta.rows, new_offsets=meta.offsets, max_new_tokens=meta.max_chunk,
                                        err=s.err)
        s.arena.lens[self.owner.rows, self.layer_idx] = ends
        return meta, q_out
