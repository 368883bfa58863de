"""KV-head-sharded decode across the GPUs of one node.

The reference decodes on one device (SDPAAttentionBackend.attend,
src/barellm/attention/backend.py:34-61).  Here the heads of one decode batch
are split across W GPUs instead of its requests: rank r keeps KV heads
[r*Hkv/W, (r+1)*Hkv/W) of every request in its own pool shard, and the query
heads that read them (query head h reads KV head h // G, the reference's
repeat_interleave grouping, src/barellm/attention/backend.py:46-49), so each
rank reads 1/W of the batch's K/V.  Every rank holds the same block tables.

The one exchange is the all-gather of the per-head outputs, and it is fused
into the decode kernels' epilogue: each output element is stored straight into
every rank's gathered buffer over NVLink (peer memory mapped with CUDA IPC,
no multicast), and a one-warp flag barrier closes the call
(``bl_paged_decode_allgather``).  :func:`gather_heads_collective` is the
unfused baseline -- decode, then an NCCL all-gather and a transpose copy.
"""

from __future__ import annotations

import torch

from . import _native as nat
from . import ops

_SIGNAL_BYTES = 256  # BL_MAX_RANKS int32 slots, padded
_HEADER_BYTES = 2 * _SIGNAL_BYTES  # signal pad, then this rank's epoch counter


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """KV heads [lo, hi) that rank ``rank`` of ``world`` owns."""
    if world < 1 or world > nat.BL_MAX_RANKS or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world} is not a valid head shard")
    if num_kv_heads % world:
        raise ValueError(f"num_kv_heads ({num_kv_heads}) must divide evenly across {world} GPUs")
    n = num_kv_heads // world
    return rank * n, (rank + 1) * n


def q_head_range(num_q_heads: int, num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Query heads [lo, hi) that read rank ``rank``'s KV heads."""
    if num_q_heads % num_kv_heads:
        raise ValueError("num_heads must divide evenly by num_kv_heads")
    g = num_q_heads // num_kv_heads
    lo, hi = kv_head_range(num_kv_heads, world, rank)
    return lo * g, hi * g


def _group_info(group) -> tuple[int, int]:
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


class HeadShardedDecode:
    """One rank's side of the KV-head-sharded decode of a fixed-size batch.

    Constructing it is a collective over ``group`` (every rank maps the
    others' output buffers, then all meet at a barrier).  :meth:`decode`
    takes this rank's query heads and pool shard and returns the gathered
    ``[batch, Hq, D]`` output.  The gathered buffers alternate (``buffers``
    of them), so a returned tensor stays valid until ``buffers - 1`` further
    calls have been made; every rank must make the same sequence of calls.

    Errors on the device (a bad block id, a barrier wait that timed out) go
    to a device error word: the caller's ``err`` when given, else one this
    object owns.  :meth:`check_device_errors` reads it (a device sync) and
    raises; :meth:`close` checks it as well.  A barrier time-out (a peer that
    did not finish the call within ``timeout_s``) is fatal to the call: its
    gathered output is undefined, and since this rank's epoch has moved on,
    the two-buffer guarantee no longer holds either -- close the object on
    every rank and build a new one (a collective) before decoding again.
    ``timeout_s`` bounds how far one rank's host may fall behind the others
    (first-call set-up, a collection pause); it is 10 s by default.
    """

    def __init__(
        self,
        batch: int,
        num_q_heads: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device,
        *,
        group=None,
        buffers: int = 2,
        timeout_s: float = 10.0,
    ):
        import torch.distributed as dist

        ops._check(buffers >= 2, "the gathered output needs at least two buffers")
        ops._check(dtype in ops.DTYPE_CODE, f"unsupported dtype {dtype}")
        self.world, self.rank = _group_info(group)
        self.group = group
        self.device = torch.device(device)
        self.batch, self.num_q_heads, self.head_dim, self.dtype = batch, num_q_heads, head_dim, dtype
        self.kv_heads = kv_head_range(num_kv_heads, self.world, self.rank)
        self.q_heads = q_head_range(num_q_heads, num_kv_heads, self.world, self.rank)
        esz = torch.empty((), dtype=dtype).element_size()
        self._elems = batch * num_q_heads * head_dim
        self._buf_bytes = -(-self._elems * esz // 256) * 256
        self.region = torch.zeros(_HEADER_BYTES + buffers * self._buf_bytes, dtype=torch.uint8, device=self.device)
        self._bases = [0] * self.world
        self._bases[self.rank] = self.region.data_ptr()
        if self.world > 1:
            handles: list[bytes | None] = [None] * self.world
            # over NCCL the object exchange stages through the current device
            with torch.cuda.device(self.device):
                dist.all_gather_object(handles, ops.ipc_export(self.region), group=group)
            for r in range(self.world):
                if r != self.rank:
                    self._bases[r] = ops.ipc_import(handles[r], self.device)
        # every signal pad is zero before any rank can signal into it
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=group)
        self.outs = [
            self.region[_HEADER_BYTES + k * self._buf_bytes:][: self._elems * esz].view(dtype)
            .view(batch, num_q_heads, head_dim)
            for k in range(buffers)
        ]
        self._next = 0
        g = nat.HeadGather()
        g.world, g.rank = self.world, self.rank
        for r in range(self.world):
            g.peer_signal[r] = self._bases[r]
        g.epoch = self.region.data_ptr() + _SIGNAL_BYTES
        g.head_offset = self.q_heads[0]
        g.timeout_ns = int(timeout_s * 1e9)
        self._g = g
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._closed = False

    def decode(
        self,
        q: torch.Tensor,
        key_cache: torch.Tensor,
        value_cache: torch.Tensor,
        layer: int,
        block_tables: torch.Tensor,
        seq_lens: torch.Tensor,
        max_seq_len: int,
        *,
        scale: float | None = None,
        row_ids: torch.Tensor | None = None,
        ws: torch.Tensor | None = None,
        plan_ready: bool = False,
        err: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Decode attention of this rank's heads, all-gathered into every
        rank's ``[batch, Hq, D]`` buffer; returns this rank's copy.

        ``q``: ``[batch, Hq/W, D]`` (or ``[batch, Hq/W, 1, D]``), this rank's
        query heads; ``key_cache`` / ``value_cache``: this rank's pool shard
        ``[L, P, Hkv/W, bs, D]``.  The scale defaults to 1/sqrt(D).
        ``err``: a device int32 error word; None uses this object's own."""
        if self._closed:
            raise RuntimeError("HeadShardedDecode is closed")
        if err is None:
            err = self.err
        q0, q1 = self.q_heads
        k = self._next
        out = self.outs[k]
        a, _, used_ws = ops._decode_args(q, key_cache, value_cache, layer, block_tables, seq_lens, max_seq_len,
                                         scale, out[:, q0:q1], row_ids, ws, plan_ready, err)
        off = _HEADER_BYTES + k * self._buf_bytes
        for r in range(self.world):
            self._g.peer_out[r] = self._bases[r] + off
        ops._raise_rc(nat.load().bl_paged_decode_allgather(a, self._g, ops._stream(self.device)))
        if not plan_ready:
            idx = ops._dev_index(self.device)
            if ops._WORKSPACES.get(idx) is used_ws:  # this call replaced the shared plan
                ops._PLAN_SERIAL[idx] = ops._PLAN_SERIAL.get(idx, 0) + 1
        self._next = (k + 1) % len(self.outs)
        return out

    def check_device_errors(self) -> None:
        """Raises RuntimeError if this object's device error word is set
        (waits for the device).  Errors sent to a caller's ``err`` word are
        the caller's to check."""
        word = int(self.err.item())
        if word:
            raise RuntimeError(ops.describe_device_error(word) + " in the head-sharded decode "
                               "(after a barrier time-out the gathered outputs are undefined)")

    def close(self) -> None:
        """Unmaps the other ranks' buffers (a collective: ends at a barrier),
        then raises if this object's device error word is set."""
        import torch.distributed as dist

        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for r in range(self.world):
            if r != self.rank and self._bases[r]:
                ops.ipc_close(self._bases[r])
                self._bases[r] = 0
        self._closed = True
        self.check_device_errors()


def gather_heads_collective(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """The unfused baseline: ``[B, Hq/W, D]`` on each rank -> ``[B, Hq, D]``
    on every rank through the process group's ``all_gather_into_tensor``
    (NCCL on GPUs) into a rank-major ``[W, B, Hq/W, D]`` buffer, then a
    transpose copy."""
    import torch.distributed as dist

    world, _ = _group_info(group)
    if world == 1:
        return out_local
    b, h, d = out_local.shape
    gathered = torch.empty((world * b, h, d), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(gathered, out_local.contiguous(), group=group)
    return gathered.view(world, b, h, d).permute(1, 0, 2, 3).reshape(b, world * h, d)
