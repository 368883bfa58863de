"""Batched view over per-request paged caches for one decode step.

Interface of the reference's BatchKVCache / BatchLayerKV
(src/barellm/engine/batched_kv_cache.py:8-145).  The reference loops over rows
in Python for every layer (one append and one gather per row) and rebuilds
lengths and block tables on each call.  Here a step's metadata -- arena row of
each request, pre-append lengths, post-append lengths -- goes to the device in
one pinned copy the first time any layer needs it and is shared by every
layer of the step (all layers of a request advance together); the split-K
decode plan built from it is shared the same way.  Appends and reads are one
kernel launch for the whole batch.
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops
from .paged_kv_cache import PagedBatchKVMetadata, PagedKVCache, PagedKVCacheView, PagedLayerKV, check


class StepMeta:
    """Device metadata for one (pre-append lengths, new tokens) combination."""

    def __init__(self, storage: PagedKVCache, rows: list[int], starts: list[int], new_tokens: int) -> None:
        b = len(rows)
        host = torch.empty((3, b), dtype=torch.int32).pin_memory()
        h = host.numpy()
        h[0] = rows
        h[1] = starts
        h[2] = np.asarray(starts, dtype=np.int64) + new_tokens
        dev = host.to(storage.device, non_blocking=True)
        self.rows, self.starts, self.seq_lens = dev[0], dev[1], dev[2]
        self.seq_lens_host = [s + new_tokens for s in starts]
        self.max_seq_len = max(self.seq_lens_host)
        self.new_tokens = new_tokens
        self.plan_ws: torch.Tensor | None = None
        self.plan_heads = 0
        self.plan_token = -1


class BatchKVCache:
    def __init__(self, caches: list[PagedKVCacheView]) -> None:
        check(len(caches) > 0, "batch cache cannot be empty")
        self.caches = caches
        self._meta: dict[tuple[tuple[int, ...], int], StepMeta] = {}

    def layer(self, layer_idx: int) -> "BatchLayerKV":
        return BatchLayerKV([cache.layer(layer_idx) for cache in self.caches], owner=self)

    def step_meta(self, storage: PagedKVCache, rows: list[int], starts: list[int], new_tokens: int) -> StepMeta:
        key = (tuple(starts), new_tokens)
        meta = self._meta.get(key)
        if meta is None:
            meta = StepMeta(storage, rows, starts, new_tokens)
            self._meta = {key: meta}  # one live step per batch view
        return meta


class BatchLayerKV:
    def __init__(self, layers: list[PagedLayerKV], owner: BatchKVCache | None = None) -> None:
        self.layers = layers
        self.owner = owner if owner is not None else BatchKVCache([PagedKVCacheView(l.storage, l.request_id) for l in layers])
        self._storage: PagedKVCache | None = None

    # -- helpers -------------------------------------------------------------
    def storage(self) -> PagedKVCache:
        """The single paged pool every member must share (TypeError otherwise)."""
        if self._storage is None:
            if not all(isinstance(l, PagedLayerKV) for l in self.layers):
                raise TypeError("paged metadata requires PagedLayerKV members")
            first = self.layers[0]
            if any(l.storage is not first.storage or l.layer_idx != first.layer_idx for l in self.layers[1:]):
                raise ValueError("paged batch layers must share storage and layout")
            self._storage = first.storage
        return self._storage

    def meta(self, new_tokens: int) -> StepMeta:
        s = self.storage()
        rows = [s.request_pages[l.request_id].row for l in self.layers]
        starts = [l.seq_len for l in self.layers]
        return self.owner.step_meta(s, rows, starts, new_tokens)

    @property
    def lengths(self) -> torch.Tensor:
        return torch.tensor([l.seq_len for l in self.layers], dtype=torch.long)

    @property
    def seq_len(self) -> int:
        return max(l.seq_len for l in self.layers)

    # -- reference interface ---------------------------------------------------
    def append(self, key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.append_only(key, value)
        return self.read()

    def append_only(self, key: torch.Tensor, value: torch.Tensor) -> StepMeta:
        """One scatter kernel for every row (reference: a Python loop of
        per-row appends, batched_kv_cache.py:40-63).  Returns the step metadata
        whose ``seq_lens`` are the post-append lengths."""
        check(key.shape[0] == len(self.layers), "batch size must match number of caches")
        check(value.shape[0] == len(self.layers), "batch size must match number of caches")
        s = self.storage()
        self.layers[0].check_new_kv(key, value, batch=len(self.layers))
        t = key.shape[2]
        for l in self.layers:
            l.check_capacity(t)
        meta = self.meta(t)
        ops.paged_append(s.key_cache, s.value_cache, self.layers[0].layer_idx, s.arena.table, meta.starts, key, value,
                         row_ids=meta.rows, err=s.err)
        for l in self.layers:
            l._request.layer_seq_lens[l.layer_idx] += t
        return meta

    def current_meta(self) -> StepMeta:
        """Metadata whose post-append lengths equal the current lengths."""
        for (starts, t), meta in self.owner._meta.items():
            if [a + t for a in starts] == [l.seq_len for l in self.layers]:
                return meta
        return self.meta(0)

    def read(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense zero-padded ``[B, H, Tmax, D]`` K and V (batched_kv_cache.py:65-95)."""
        check(all(l.seq_len > 0 for l in self.layers), "KV cache is empty")
        s = self.storage()
        meta = self.current_meta()
        return ops.paged_gather(s.key_cache, s.value_cache, self.layers[0].layer_idx, s.arena.table, meta.seq_lens,
                                meta.max_seq_len, row_ids=meta.rows, err=s.err)

    def attention_mask(self, q_len: int) -> torch.Tensor:
        """``[B, 1, q_len, Tmax]`` valid-key mask (batched_kv_cache.py:97-102)."""
        s = self.storage()
        lens = torch.tensor([l.seq_len for l in self.layers], dtype=torch.long, device=s.device)
        valid = torch.arange(int(lens.max()), device=s.device).unsqueeze(0) < lens.unsqueeze(1)
        return valid[:, None, None, :].expand(-1, 1, q_len, -1)

    def paged_metadata_post_append(self) -> PagedBatchKVMetadata:
        """Rectangular int32 block tables padded with -1 and int32 post-append
        lengths (batched_kv_cache.py:104-145), gathered from the arena."""
        s = self.storage()
        for l in self.layers:
            check(l.seq_len > 0, "KV cache is empty")
        meta = self.current_meta()
        counts = [len(s.request_pages[l.request_id].blocks) for l in self.layers]
        width = max(counts)
        tables = s.arena.table.index_select(0, meta.rows.long())[:, :width].clone()
        col = torch.arange(width, device=s.device).unsqueeze(0)
        limit = torch.tensor(counts, device=s.device).unsqueeze(1)
        tables.masked_fill_(col >= limit, -1)
        return PagedBatchKVMetadata(s.key_cache, s.value_cache, self.layers[0].layer_idx, tables, meta.seq_lens.clone(),
                                    s.block_size)
