"""The CUDA attention backend: ``AttentionBackend.attend`` over paged K/V.

Drop-in for the reference's backend seam (src/barellm/attention/backend.py:12-79):
``attend(q, new_k, new_v, layer_cache, group_size)`` appends the new K/V to
the layer cache and returns attention of ``q`` over the whole cached sequence,
``[B, Hq, q_len, D]``.  Where the reference appends, gathers every page into a
dense tensor, repeats it per query head and runs SDPA, this backend appends
with one scatter kernel and attends straight from the pages:

  * BatchLayerKV (batched decode, engine.py:458-488): one append kernel for
    the batch, then the split-K decode kernels for q_len == 1 (the plan is
    built once per step and reused by every layer), or the paged prefill
    kernel for q_len > 1;
  * PagedLayerKV (single-request prefill, engine.py:226-257, including a
    non-empty prefix = chunked prefill): append, then paged prefill with the
    bottom-right causal mask (equal to SDPA(is_causal=True) without a prefix);
  * PackedBatchLayerKV (batched chunked prefill: many requests' ragged chunks
    packed on the token axis): one packed append, one paged prefill;
  * None (uncached full forward): the new K/V are paged into a scratch pool
    and attended causally by the same prefill kernel.
There is no CPU path: a CPU tensor or an unknown cache type raises.
"""

from __future__ import annotations

from typing import Literal, Protocol

import torch

from . import ops
from .batched_kv_cache import BatchLayerKV, PackedBatchLayerKV
from .paged_kv_cache import PagedLayerKV, _i32, check

AttentionBackendName = Literal["auto", "sdpa", "triton", "cuda"]


def _paged_rows(layer_cache) -> list[PagedLayerKV] | None:
    """The member layers of a batched layer view that is not this package's
    (the reference's BatchLayerKV keeps them in ``.layers``), when every member
    is a PagedLayerKV of this package; else None."""
    rows = getattr(layer_cache, "layers", None)
    if isinstance(rows, list) and rows and all(isinstance(r, PagedLayerKV) for r in rows):
        return rows
    return None


class AttentionBackend(Protocol):
    def attend(self, q: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor, layer_cache,
               group_size: int) -> torch.Tensor: ...


class CudaPagedAttentionBackend:
    """Paged append + attention on sm_100a kernels."""

    def attend(self, q: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor, layer_cache,
               group_size: int) -> torch.Tensor:
        check(q.ndim == 4 and new_k.ndim == 4, "q/K/V must have shape [B, H, T, D]")
        check(q.shape[1] == new_k.shape[1] * group_size, "num_heads must divide evenly by num_kv_heads")
        if isinstance(layer_cache, BatchLayerKV):
            return self._batched(q, new_k, new_v, layer_cache)
        if isinstance(layer_cache, PagedLayerKV):
            return self._single(q, new_k, new_v, layer_cache)
        if isinstance(layer_cache, PackedBatchLayerKV):
            return self._packed_attend(q, layer_cache, layer_cache.append_only(new_k, new_v))
        if layer_cache is None:
            return self._uncached(q, new_k, new_v)
        rows = _paged_rows(layer_cache)
        if rows is not None:
            # the reference's own BatchLayerKV (batched_kv_cache.py:19-26) over
            # this package's paged layers: the engine's decode batch when only
            # PagedKVCache and the backend are swapped in
            return self._batched(q, new_k, new_v, BatchLayerKV(rows))
        raise TypeError(f"the cuda attention backend reads paged caches, not {type(layer_cache).__name__}")

    def attend_prepped(self, q: torch.Tensor, new_k: torch.Tensor, new_v: torch.Tensor, q_norm_weight: torch.Tensor,
                       k_norm_weight: torch.Tensor, eps: float, cos: torch.Tensor, sin: torch.Tensor, layer_cache,
                       group_size: int) -> torch.Tensor:
        """``attend`` for q / new_k straight out of the projections: the
        QK-RMSNorm and RoPE of the reference's attention
        (src/barellm/models/attention.py:161-169) run fused with the append
        (one kernel), then the same paged attention as ``attend``."""
        check(q.ndim == 4 and new_k.ndim == 4, "q/K/V must have shape [B, H, T, D]")
        check(q.shape[1] == new_k.shape[1] * group_size, "num_heads must divide evenly by num_kv_heads")
        if isinstance(layer_cache, BatchLayerKV):
            meta, qp = layer_cache.append_only_prepped(q, new_k, new_v, q_norm_weight, k_norm_weight, cos, sin, eps)
            return self._batched_attend(qp, layer_cache, meta)
        if isinstance(layer_cache, PagedLayerKV):
            check(q.shape[0] == 1, "PagedKVCache currently supports batch size 1")
            qp = layer_cache.append_only_prepped(q, new_k, new_v, q_norm_weight, k_norm_weight, cos, sin, eps)
            return self._single_attend(qp, layer_cache)
        if isinstance(layer_cache, PackedBatchLayerKV):
            meta, qp = layer_cache.append_only_prepped(q, new_k, new_v, q_norm_weight, k_norm_weight, cos, sin, eps)
            return self._packed_attend(qp, layer_cache, meta)
        raise TypeError("fused QK preparation needs a paged cache; use attend() with prepared q/k")

    def _batched(self, q, new_k, new_v, layer: BatchLayerKV) -> torch.Tensor:
        return self._batched_attend(q, layer, layer.append_only(new_k, new_v))

    def _batched_attend(self, q, layer: BatchLayerKV, meta) -> torch.Tensor:
        s = layer.storage()
        idx = layer.layer_idx
        b, hq, t, d = q.shape
        if t == 1:
            out = torch.empty((b, hq, 1, d), dtype=q.dtype, device=q.device)
            serial = ops.plan_serial(s.device)
            if meta.plan_ws is None or meta.plan_token != serial or meta.plan_heads != hq:
                # once per step (the plan depends only on the lengths, not the
                # layer): plan + attention + reduce in one call, into the shared
                # workspace that the step's later layers then reuse
                ws = ops.workspace(s.device, ops.decode_workspace_bytes(b, hq, d, s.block_size, meta.max_seq_len))
                ops.paged_decode(q, s.key_cache, s.value_cache, idx, s.arena.table, meta.seq_lens, meta.max_seq_len,
                                 out=out, row_ids=meta.rows, ws=ws, plan_ready=False, err=s.err)
                meta.plan_ws = ws
                meta.plan_token = ops.plan_serial(s.device)
                meta.plan_heads = hq
                return out
            ops.paged_decode(q, s.key_cache, s.value_cache, idx, s.arena.table, meta.seq_lens, meta.max_seq_len,
                             out=out, row_ids=meta.rows, ws=meta.plan_ws, plan_ready=True, err=s.err)
            return out
        return ops.paged_prefill(q, s.key_cache, s.value_cache, idx, s.arena.table, meta.seq_lens,
                                 row_ids=meta.rows, err=s.err)

    def _single(self, q, new_k, new_v, layer: PagedLayerKV) -> torch.Tensor:
        check(q.shape[0] == 1, "PagedKVCache currently supports batch size 1")
        layer.append_only(new_k, new_v)
        return self._single_attend(q, layer)

    def _single_attend(self, q, layer: PagedLayerKV) -> torch.Tensor:
        s = layer.storage
        n = layer.seq_len
        rows = _i32([layer._request.row], s.device)
        seq = _i32([n], s.device)
        if q.shape[2] == 1:
            out = ops.paged_decode(q, s.key_cache, s.value_cache, layer.layer_idx, s.arena.table, seq, n,
                                   row_ids=rows, err=s.err)
            return out.unsqueeze(2)
        return ops.paged_prefill(q, s.key_cache, s.value_cache, layer.layer_idx, s.arena.table, seq, row_ids=rows,
                                 err=s.err)

    def _packed_attend(self, q, layer: PackedBatchLayerKV, meta) -> torch.Tensor:
        """Chunked prefill of a packed batch: each row's chunk attends over its
        cached prefix and itself (bottom-right causal), one kernel."""
        s = layer.owner.storage
        return ops.paged_prefill(q, s.key_cache, s.value_cache, layer.layer_idx, s.arena.table, meta.seq_lens,
                                 q_offsets=meta.offsets, max_q_len=meta.max_chunk, row_ids=meta.rows, err=s.err)

    def _uncached(self, q, new_k, new_v) -> torch.Tensor:
        """Causal self-attention of a fresh sequence: page it into a scratch
        pool (block_size 16 when head_dim allows the tensor-core path) and run
        the prefill kernel with an empty prefix."""
        b, hkv, t, d = new_k.shape
        bs = 16
        nb = -(-t // bs)
        pool_shape = (1, b * nb, hkv, bs, d)
        kc = torch.empty(pool_shape, dtype=new_k.dtype, device=new_k.device)
        vc = torch.empty_like(kc)
        table = torch.arange(b * nb, dtype=torch.int32, device=new_k.device).view(b, nb)
        zeros = torch.zeros(b, dtype=torch.int32, device=new_k.device)
        ops.paged_append(kc, vc, 0, table, zeros, new_k, new_v)
        seq = torch.full((b,), t, dtype=torch.int32, device=new_k.device)
        return ops.paged_prefill(q, kc, vc, 0, table, seq)


def create_attention_backend(name: AttentionBackendName = "cuda", *, sdpa=None) -> AttentionBackend:
    """Backend factory mirroring the reference's (backend.py:64-79), for the
    one backend this package provides.  ``"cuda"`` and ``"auto"`` give the
    paged CUDA backend; ``"sdpa"`` is the reference's own portable backend and
    lives there."""
    del sdpa
    if name not in ("auto", "sdpa", "triton", "cuda"):
        raise ValueError(f"Unknown attention backend: {name!r}")
    if name == "triton":
        raise RuntimeError("The Triton attention backend is not implemented; use attention_backend='cuda'")
    if name == "sdpa":
        raise ValueError("the 'sdpa' backend is the reference's portable backend; barellm_b200 provides 'cuda'")
    return CudaPagedAttentionBackend()
