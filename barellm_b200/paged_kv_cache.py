"""Paged K/V storage whose write and read paths run as CUDA kernels.

Interface of the reference's PagedKVCache / PagedKVCacheView / PagedLayerKV
(src/barellm/engine/paged_kv_cache.py:41-244): the same constructor, the same
``[L, P, Hkv, bs, D]`` ``key_cache`` / ``value_cache`` tensors, the same
per-request block lists and per-layer lengths, the same ``check()`` messages.

What changes underneath:
  * block tables live in one device-resident int32 arena (a row per live
    request, grown in place), instead of an int64 tensor rebuilt from a Python
    list on every growth (paged_kv_cache.py:86-99); a growth uploads only the
    new entries;
  * ``append_only`` is one slot-mapped scatter kernel (bl_paged_append) and
    ``read`` one gather kernel (bl_paged_gather).
The pool must live on a CUDA device; there is no CPU fallback.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import ops
from .block_pool import KVCacheBlock


def check(condition: bool, message: str) -> None:
    """The reference's argument check (src/barellm/utils.py:1-3)."""
    if not condition:
        raise ValueError(message)


class BlockTableArena:
    """Device-resident int32 block tables, one row per live request.

    Rows are recycled through a free list; a row's width grows (doubling, with
    one device copy) when a request outgrows it.  ``host`` mirrors the device
    table so a growth uploads only the entries that changed, asynchronously
    from pinned memory on the current stream."""

    def __init__(self, device: torch.device, rows: int = 64, width: int = 64, num_layers: int = 1) -> None:
        self.device = device
        self.host = np.full((rows, width), -1, dtype=np.int32)
        self.used = np.zeros(rows, dtype=np.int64)  # valid entries per row
        # per-row, per-layer cached lengths (host side); rows index the table
        self.lens = np.zeros((rows, num_layers), dtype=np.int64)
        self.table = torch.full((rows, width), -1, dtype=torch.int32, device=device)
        self._free_rows = list(range(rows - 1, -1, -1))

    @property
    def width(self) -> int:
        return self.host.shape[1]

    def _grow(self, rows: int | None = None, width: int | None = None) -> None:
        r0, w0 = self.host.shape
        r1, w1 = max(r0, rows or r0), max(w0, width or w0)
        host = np.full((r1, w1), -1, dtype=np.int32)
        host[:r0, :w0] = self.host
        table = torch.full((r1, w1), -1, dtype=torch.int32, device=self.device)
        table[:r0, :w0].copy_(self.table)
        self.host, self.table = host, table
        self.used = np.concatenate([self.used, np.zeros(r1 - r0, dtype=np.int64)])
        self.lens = np.concatenate([self.lens, np.zeros((r1 - r0, self.lens.shape[1]), dtype=np.int64)])
        self._free_rows = list(range(r1 - 1, r0 - 1, -1)) + self._free_rows

    def alloc_row(self) -> int:
        if not self._free_rows:
            self._grow(rows=2 * self.host.shape[0])
        row = self._free_rows.pop()
        self.lens[row] = 0
        return row

    def free_row(self, row: int) -> None:
        self.used[row] = 0
        self.lens[row] = 0
        self._free_rows.append(row)

    def set_row(self, row: int, block_ids: list[int]) -> None:
        n = len(block_ids)
        if n > self.width:
            w = self.width
            while w < n:
                w *= 2
            self._grow(width=w)
        new = np.asarray(block_ids, dtype=np.int32)
        old_n = int(self.used[row])
        common = min(old_n, n)
        diff = np.nonzero(self.host[row, :common] != new[:common])[0]
        start = int(diff[0]) if len(diff) else common
        if start < n:
            self.host[row, start:n] = new[start:]
            src = torch.from_numpy(self.host[row, start:n].copy())
            if self.device.type == "cuda":
                src = src.pin_memory()
            self.table[row, start:n].copy_(src, non_blocking=True)
        self.used[row] = n

    def row_view(self, row: int) -> torch.Tensor:
        return self.table[row, : int(self.used[row])]


@dataclass
class _RequestPages:
    blocks: list[KVCacheBlock]
    row: int
    arena: BlockTableArena = field(repr=False)

    @property
    def layer_seq_lens(self) -> np.ndarray:
        """Cached length per layer (a writable view into the arena's table)."""
        return self.arena.lens[self.row]

    @property
    def block_table(self) -> torch.Tensor:
        """The request's physical block ids (int32, on the pool's device)."""
        return self.arena.row_view(self.row)


@dataclass(frozen=True)
class PagedKVMetadata:
    """Read-only post-append view (paged_kv_cache.py:17-26)."""

    key_cache: torch.Tensor
    value_cache: torch.Tensor
    layer_idx: int
    block_table: torch.Tensor
    seq_len: int
    block_size: int


@dataclass(frozen=True)
class PagedBatchKVMetadata:
    """Rectangular device-resident batch metadata (paged_kv_cache.py:29-38)."""

    key_cache: torch.Tensor
    value_cache: torch.Tensor
    layer_idx: int
    block_tables: torch.Tensor
    seq_lens: torch.Tensor
    block_size: int


class _RowSet:
    """Arena rows of one request tuple, and that batch's reusable step metadata."""

    __slots__ = ("generation", "rows", "meta")

    def __init__(self, generation: int, rows: np.ndarray) -> None:
        self.generation = generation
        self.rows = rows
        self.meta = None


class PagedKVCache:
    """Paged K/V storage for one GPU (one BlockPool shard)."""

    def __init__(
        self,
        num_layers: int,
        max_blocks: int,
        num_kv_heads: int,
        block_size: int,
        head_dim: int,
        dtype: torch.dtype = torch.float32,
        device: torch.device | str = "cpu",
        *,
        max_requests: int = 64,
    ) -> None:
        check(num_layers > 0, "num_layers must be positive")
        check(max_blocks > 0, "max_blocks must be positive")
        check(num_kv_heads > 0, "num_kv_heads must be positive")
        check(block_size > 0, "block_size must be positive")
        check(head_dim > 0, "head_dim must be positive")
        check(max_blocks <= np.iinfo(np.int32).max, "physical block id does not fit in int32 metadata")
        self.num_layers = num_layers
        self.max_blocks = max_blocks
        self.num_kv_heads = num_kv_heads
        self.block_size = block_size
        self.head_dim = head_dim
        self.dtype = dtype
        shape = (num_layers, max_blocks, num_kv_heads, block_size, head_dim)
        self.key_cache = torch.empty(shape, dtype=dtype, device=device)
        self.value_cache = torch.empty_like(self.key_cache)
        self.device = self.key_cache.device
        self.request_pages: dict[str, _RequestPages] = {}
        self.arena = BlockTableArena(self.device, rows=max_requests, width=64, num_layers=num_layers)
        self._err = None
        self._generation = 0  # bumped whenever a request gains or loses its arena row
        self._rows_cache: dict[tuple, _RowSet] = {}

    # -- error word shared by this pool's kernels -------------------------
    @property
    def err(self) -> torch.Tensor | None:
        if self.device.type != "cuda":
            return None
        if self._err is None:
            self._err = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._err

    def check_device_errors(self) -> None:
        """Synchronises and raises if any kernel flagged an error (a bad block
        id, a table overrun, a timed-out wait) in this pool's error word; the
        word is cleared first."""
        if self._err is None:
            return
        code = int(self._err.item())
        if code:
            self._err.zero_()
            raise RuntimeError("paged-KV kernel reported " + ops.describe_device_error(code))

    def register_request(self, request_id: str, blocks: list[KVCacheBlock]) -> None:
        pages = self.request_pages.get(request_id)
        if pages is None:
            pages = _RequestPages(list(blocks), self.arena.alloc_row(), self.arena)
            self.request_pages[request_id] = pages
            self._generation += 1
        else:
            pages.blocks = list(blocks)
        self.arena.set_row(pages.row, [b.block_id for b in blocks])

    def check_new_kv(self, key: torch.Tensor, value: torch.Tensor, batch: int = 1) -> None:
        """The reference's append checks (paged_kv_cache.py:156-174)."""
        ks = key.shape
        if (len(ks) == 4 and value.shape == ks and ks[0] == batch and ks[1] == self.num_kv_heads and ks[2] > 0
                and ks[3] == self.head_dim and key.dtype is self.dtype and value.dtype is self.dtype
                and key.device == self.device and value.device == self.device):
            return
        check(key.ndim == 4 and value.ndim == 4, "K/V must have shape [B, H, T, D]")
        check(key.shape == value.shape, "K/V must have identical shape")
        check(key.shape[0] == batch, "PagedKVCache currently supports batch size 1")
        check(key.shape[1] == self.num_kv_heads, "KV-head count cannot change")
        check(key.shape[2] > 0, "K/V sequence length must be greater than zero")
        check(key.shape[3] == self.head_dim, "Head dimension cannot change")
        check(key.dtype == self.dtype, "K/V dtype cannot change")
        check(key.device == self.device, "K/V device cannot change")
        check(key.dtype == value.dtype, "K/V dtype must match")
        check(key.device == value.device, "K/V device must match")

    def unregister_request(self, request_id: str) -> None:
        pages = self.request_pages.pop(request_id, None)
        if pages is not None:
            self.arena.free_row(pages.row)
            self._generation += 1

    def row_set(self, request_ids: tuple) -> "_RowSet":
        """Arena rows of ``request_ids`` (a read-only int64 array) plus a slot
        for the batch's reusable step metadata.  A decode batch asks for the
        same requests step after step, so the answer is kept until a request
        is registered or removed."""
        hit = self._rows_cache.get(request_ids)
        if hit is not None and hit.generation == self._generation:
            return hit
        pages = self.request_pages
        try:
            rows = np.fromiter((pages[r].row for r in request_ids), dtype=np.int64, count=len(request_ids))
        except KeyError as exc:
            raise KeyError(f"Unknown request: {exc.args[0]}") from exc
        rows.flags.writeable = False
        if len(self._rows_cache) >= 16:
            self._rows_cache.clear()
        rs = self._rows_cache[request_ids] = _RowSet(self._generation, rows)
        return rs

    def rows_for(self, request_ids: tuple) -> np.ndarray:
        return self.row_set(request_ids).rows

    def get_cache(self, request_id: str) -> "PagedKVCacheView":
        if request_id not in self.request_pages:
            raise KeyError(f"Unknown request: {request_id}")
        return PagedKVCacheView(self, request_id)


class PagedKVCacheView:
    def __init__(self, storage: PagedKVCache, request_id: str) -> None:
        self.storage = storage
        self.request_id = request_id

    def layer(self, layer_idx: int) -> "PagedLayerKV":
        if not 0 <= layer_idx < self.storage.num_layers:
            raise IndexError(f"Invalid layer index: {layer_idx}")
        return PagedLayerKV(self.storage, self.request_id, layer_idx)


def _i32(values, device) -> torch.Tensor:
    """Small host int list -> device int32 tensor, async from pinned memory."""
    return torch.tensor(values, dtype=torch.int32).pin_memory().to(device, non_blocking=True)


class PagedLayerKV:
    def __init__(self, storage: PagedKVCache, request_id: str, layer_idx: int) -> None:
        self.storage = storage
        self.request_id = request_id
        self.layer_idx = layer_idx

    @property
    def _request(self) -> _RequestPages:
        try:
            return self.storage.request_pages[self.request_id]
        except KeyError as exc:
            raise KeyError(f"Unknown request: {self.request_id}") from exc

    @property
    def seq_len(self) -> int:
        return int(self._request.layer_seq_lens[self.layer_idx])

    def append(self, key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.append_only(key, value)
        return self.read()

    def check_new_kv(self, key: torch.Tensor, value: torch.Tensor, batch: int = 1) -> None:
        self.storage.check_new_kv(key, value, batch)

    def check_capacity(self, new_tokens: int) -> None:
        end = self.seq_len + new_tokens
        required = -(-end // self.storage.block_size)
        check(required <= len(self._request.blocks), "request does not have enough allocated KV blocks")

    def append_only(self, key: torch.Tensor, value: torch.Tensor) -> None:
        self.check_new_kv(key, value)
        self.check_capacity(key.shape[2])
        s = self.storage
        req = self._request
        start = int(req.layer_seq_lens[self.layer_idx])
        ops.paged_append(s.key_cache, s.value_cache, self.layer_idx, s.arena.table,
                         _i32([start], s.device), key, value, row_ids=_i32([req.row], s.device), err=s.err)
        req.layer_seq_lens[self.layer_idx] = start + key.shape[2]

    def append_only_prepped(self, q: torch.Tensor, key: torch.Tensor, value: torch.Tensor, q_norm_weight,
                            k_norm_weight, cos, sin, eps: float) -> torch.Tensor:
        """append_only of the QK-normalised, rotated key, with the same norm and
        rotation applied to ``q``, in one kernel; returns the prepared q."""
        self.check_new_kv(key, value)
        self.check_capacity(key.shape[2])
        s = self.storage
        req = self._request
        start = int(req.layer_seq_lens[self.layer_idx])
        q_out = ops.qk_norm_rope_append(q, key, value, q_norm_weight, k_norm_weight, cos, sin, eps, s.key_cache,
                                        s.value_cache, self.layer_idx, s.arena.table, _i32([start], s.device),
                                        row_ids=_i32([req.row], s.device), err=s.err)
        req.layer_seq_lens[self.layer_idx] = start + key.shape[2]
        return q_out

    def paged_metadata_post_append(self) -> PagedKVMetadata:
        check(self.seq_len > 0, "KV cache is empty")
        s = self.storage
        return PagedKVMetadata(s.key_cache, s.value_cache, self.layer_idx, self._request.block_table,
                               self.seq_len, s.block_size)

    def read(self) -> tuple[torch.Tensor, torch.Tensor]:
        check(self.seq_len > 0, "KV cache is empty")
        s = self.storage
        n = self.seq_len
        req = self._request
        return ops.paged_gather(s.key_cache, s.value_cache, self.layer_idx, s.arena.table, _i32([n], s.device), n,
                                row_ids=_i32([req.row], s.device), err=s.err)

    def attention_mask(self, q_len: int) -> torch.Tensor | None:
        del q_len
        return None
