"""Tensor-level wrappers over the C ABI (PyTorch is only the plumbing here).

Each function validates shapes the way the reference's ``check()`` does
(``ValueError`` with the reference's message where one exists,
src/barellm/utils.py:1-3) and then enqueues the CUDA kernels on the current
stream.  Nothing falls back to a CPU or ATen implementation: on a CPU tensor,
or without the built library, every call raises.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _native as nat

DTYPE_CODE = {torch.float32: nat.BL_F32, torch.float16: nat.BL_F16, torch.bfloat16: nat.BL_BF16}


class KernelError(RuntimeError):
    """A CUDA launch or driver call inside the library failed."""


def _check(cond: bool, message: str) -> None:
    if not cond:
        raise ValueError(message)


def describe_device_error(word: int) -> str:
    """Names the BL_DEVERR_* bits of a device error word."""
    names = [(nat.BL_DEVERR_BLOCK_ID, "block id outside the pool"), (nat.BL_DEVERR_TABLE, "block table overrun"),
             (nat.BL_DEVERR_TIMEOUT, "bounded wait timed out"),
             (nat.BL_DEVERR_WORKSPACE, "split-K workspace holds no matching plan")]
    found = [text for bit, text in names if word & bit]
    return f"device error word {word:#x} ({'; '.join(found) or 'unknown bits'})"


def _raise_rc(rc: int) -> None:
    if rc == nat.BL_OK:
        return
    msg = nat.last_error()
    if rc == nat.BL_ERR_LAUNCH:
        raise KernelError(msg)
    raise ValueError(msg)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The current CUDA stream of ``device`` as a raw handle (the fast
    accessor when this torch build has it)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"barellm_b200 kernels run on CUDA devices only; {name} is on {t.device}"
        )


def _int32_on(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    _check(t.dtype == torch.int32, f"{name} must be int32")
    _check(t.device == device, f"{name} must be on {device}")
    return t


def _paged_layer_checks(key_cache, value_cache, layer, block_tables, row_ids) -> None:
    """The pool / table checks one at a time, raising the first that fails."""
    _require_cuda(key_cache, "key_cache")
    _check(key_cache.ndim == 5, "K/V pool must have shape [L, P, H, S, D]")
    _check(key_cache.shape == value_cache.shape, "K/V pools must have identical shape")
    _check(key_cache.dtype == value_cache.dtype, "K/V dtype must match")
    _check(key_cache.device == value_cache.device, "K/V device must match")
    _check(key_cache.is_contiguous() and value_cache.is_contiguous(), "K/V pools must be contiguous")
    _check(key_cache.dtype in DTYPE_CODE, f"unsupported dtype {key_cache.dtype}")
    if not 0 <= layer < key_cache.shape[0]:
        raise IndexError(f"Invalid layer index: {layer}")
    _int32_on(block_tables, key_cache.device, "block_tables")
    _check(block_tables.ndim == 2 and block_tables.stride(1) == 1, "block_tables must be [rows, width] with unit inner stride")
    _check(block_tables.shape[1] > 0, "block_tables must have at least one column")
    if row_ids is not None:
        _int32_on(row_ids, key_cache.device, "row_ids")


def _paged_layer(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    row_ids: torch.Tensor | None,
) -> nat.PagedLayer:
    ks = key_cache.shape
    dev = key_cache.device
    dt = key_cache.dtype
    # every check in one expression (the common, valid case); on a failure
    # the step-by-step checks raise the specific error
    if not (len(ks) == 5 and value_cache.shape == ks and value_cache.dtype is dt and dt in DTYPE_CODE
            and value_cache.device == dev and key_cache.is_contiguous() and value_cache.is_contiguous()
            and 0 <= layer < ks[0] and block_tables.dtype is torch.int32 and block_tables.device == dev
            and block_tables.ndim == 2 and block_tables.stride(1) == 1 and block_tables.shape[1] > 0
            and (row_ids is None or (row_ids.dtype is torch.int32 and row_ids.device == dev))
            and key_cache.is_cuda):
        _paged_layer_checks(key_cache, value_cache, layer, block_tables, row_ids)
    return nat.PagedLayer(key_cache.data_ptr(), value_cache.data_ptr(), ks[0], ks[1], ks[2], ks[3], ks[4],
                          DTYPE_CODE[dt], layer, block_tables.data_ptr(), block_tables.stride(0),
                          block_tables.shape[1], None if row_ids is None else row_ids.data_ptr())


def _append_checks(key_cache, key, value, start_pos, new_offsets, max_new_tokens) -> None:
    """paged_append's input checks one at a time, raising the first that fails."""
    _check(key.ndim == 4 and value.ndim == 4, "K/V must have shape [B, H, T, D]")
    _check(key.shape == value.shape, "K/V must have identical shape")
    _check(key.shape[1] == key_cache.shape[2], "KV-head count cannot change")
    _check(key.shape[2] > 0, "K/V sequence length must be greater than zero")
    _check(key.shape[3] == key_cache.shape[4], "Head dimension cannot change")
    _check(key.dtype == key_cache.dtype, "K/V dtype cannot change")
    _check(key.device == key_cache.device, "K/V device cannot change")
    _check(key.dtype == value.dtype, "K/V dtype must match")
    _check(value.device == key_cache.device, "K/V device cannot change")
    _check(key.stride(3) == 1 and value.stride(3) == 1, "K/V head_dim must be contiguous")
    _int32_on(start_pos, key.device, "start_pos")
    batch = start_pos.shape[0]
    if new_offsets is None:
        _check(key.shape[0] == batch, "batch size must match number of caches")
    else:
        _int32_on(new_offsets, key.device, "new_offsets")
        _check(key.shape[0] == 1 and new_offsets.shape[0] == batch + 1, "packed K/V need [1, H, T, D] and [B+1] offsets")
        _check(max_new_tokens is not None and max_new_tokens > 0, "packed append needs max_new_tokens")


def paged_append(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    start_pos: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    row_ids: torch.Tensor | None = None,
    new_offsets: torch.Tensor | None = None,
    max_new_tokens: int | None = None,
    err: torch.Tensor | None = None,
) -> None:
    """Writes new K/V tokens straight into their pool slots.

    ``key``/``value``: ``[B, Hkv, T, D]`` (any strides, D contiguous); row b's
    tokens go to positions ``start_pos[b] ..``.  With ``new_offsets`` (``[B+1]``)
    the tokens are packed on the T axis of a ``[1, Hkv, sum T, D]`` tensor.
    Mirrors PagedLayerKV.append_only, src/barellm/engine/paged_kv_cache.py:151-193.
    """
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    ks = key.shape
    dev = key_cache.device
    batch = start_pos.shape[0]
    packed = new_offsets is not None
    if not (len(ks) == 4 and value.shape == ks and ks[1] == key_cache.shape[2] and ks[2] > 0
            and ks[3] == key_cache.shape[4] and key.dtype is key_cache.dtype and value.dtype is key.dtype
            and key.device == dev and value.device == dev and key.stride(3) == 1 and value.stride(3) == 1
            and start_pos.dtype is torch.int32 and start_pos.device == dev
            and (ks[0] == batch if not packed else
                 (new_offsets.dtype is torch.int32 and new_offsets.device == dev and ks[0] == 1
                  and new_offsets.shape[0] == batch + 1 and max_new_tokens is not None and max_new_tokens > 0))):
        _append_checks(key_cache, key, value, start_pos, new_offsets, max_new_tokens)
    ksd = key.stride()
    vsd = value.stride()
    # packed rows are addressed by new_offsets alone
    a = nat.AppendArgs(pl, key.data_ptr(), value.data_ptr(), 0 if packed else ksd[0], ksd[1], ksd[2],
                       0 if packed else vsd[0], vsd[1], vsd[2], start_pos.data_ptr(),
                       new_offsets.data_ptr() if packed else None, batch,
                       int(max_new_tokens) if packed else ks[2], None if err is None else err.data_ptr())
    _raise_rc(nat.load().bl_paged_append(a, _stream(key.device)))


def qk_norm_rope_append(
    q: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    eps: float,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    start_pos: torch.Tensor,
    *,
    row_ids: torch.Tensor | None = None,
    new_offsets: torch.Tensor | None = None,
    max_new_tokens: int | None = None,
    q_out: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """QK-RMSNorm + RoPE on q and k, then k and v appended to their pages, in
    one kernel; returns the normalised, rotated q (``[B, Hq, T, D]``).

    Equals ``apply_rope(q_norm(q), cos, sin)``, ``apply_rope(k_norm(k), cos,
    sin)`` and ``append_only(k, v)`` of the reference
    (src/barellm/models/attention.py:161-169, models/norm.py:14-21,
    models/rope.py:53-68, engine/paged_kv_cache.py:151-193), with the same
    roundings to the element type.  ``q``/``key``/``value``: ``[B, H, T, D]``
    (any strides, D contiguous), or packed ``[1, H, sum T, D]`` with
    ``new_offsets``.  ``cos``/``sin``: ``[B or 1, 1, T, D]`` as the reference's
    RotaryEmbedding returns them (packed: ``[1, 1, sum T, D]``).
    """
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    _check(q.ndim == 4 and key.ndim == 4 and value.ndim == 4, "q/K/V must have shape [B, H, T, D]")
    _check(key.shape == value.shape, "K/V must have identical shape")
    _check(key.shape[1] == key_cache.shape[2], "KV-head count cannot change")
    _check(key.shape[2] > 0, "K/V sequence length must be greater than zero")
    _check(key.shape[3] == key_cache.shape[4] and q.shape[3] == key.shape[3], "Head dimension cannot change")
    _check(q.shape[0] == key.shape[0] and q.shape[2] == key.shape[2], "q and K/V must cover the same tokens")
    _check(q.shape[1] % key.shape[1] == 0, "num_heads must divide evenly by num_kv_heads")
    for t, name in ((q, "q"), (key, "K"), (value, "V"), (q_norm_weight, "q_norm_weight"),
                    (k_norm_weight, "k_norm_weight"), (cos, "cos"), (sin, "sin")):
        _check(t.dtype == key_cache.dtype, f"{name} dtype must match the K/V pool")
        _check(t.device == key_cache.device, f"{name} must be on {key_cache.device}")
        _check(t.stride(-1) == 1, f"{name} must have a contiguous last dimension")
    d = key.shape[3]
    _check(q_norm_weight.shape == (d,) and k_norm_weight.shape == (d,), "norm weights must have shape [head_dim]")
    _check(cos.shape == sin.shape and cos.stride() == sin.stride(), "cos/sin must have identical shapes and strides")
    _check(cos.ndim == 4 and cos.shape[1] == 1 and cos.shape[2] == q.shape[2] and cos.shape[3] == d,
           "cos/sin must have shape [B or 1, 1, T, D]")
    _check(cos.shape[0] in (1, q.shape[0]), "cos/sin batch must be 1 or B")
    _int32_on(start_pos, key.device, "start_pos")
    batch = start_pos.shape[0]
    if new_offsets is None:
        _check(key.shape[0] == batch, "batch size must match number of caches")
        max_new = key.shape[2]
    else:
        _int32_on(new_offsets, key.device, "new_offsets")
        _check(key.shape[0] == 1 and new_offsets.shape[0] == batch + 1, "packed K/V need [1, H, T, D] and [B+1] offsets")
        _check(max_new_tokens is not None and max_new_tokens > 0, "packed append needs max_new_tokens")
        max_new = int(max_new_tokens)
    if q_out is None:
        q_out = torch.empty_like(q)  # q's memory layout when q is dense, else contiguous
    _check(q_out.shape == q.shape and q_out.stride(3) == 1 and q_out.dtype == q.dtype, "q_out must match q")
    a = nat.QkPrepArgs()
    a.kv = pl
    a.q_in, a.k_in, a.v_in, a.q_out = q.data_ptr(), key.data_ptr(), value.data_ptr(), q_out.data_ptr()
    a.q_in_stride_b, a.q_in_stride_h, a.q_in_stride_t = q.stride(0), q.stride(1), q.stride(2)
    a.k_in_stride_b, a.k_in_stride_h, a.k_in_stride_t = key.stride(0), key.stride(1), key.stride(2)
    a.v_in_stride_b, a.v_in_stride_h, a.v_in_stride_t = value.stride(0), value.stride(1), value.stride(2)
    a.q_out_stride_b, a.q_out_stride_h, a.q_out_stride_t = q_out.stride(0), q_out.stride(1), q_out.stride(2)
    a.q_norm_weight, a.k_norm_weight = q_norm_weight.data_ptr(), k_norm_weight.data_ptr()
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.rope_stride_b = cos.stride(0) if cos.shape[0] > 1 else 0
    a.rope_stride_t = cos.stride(2)
    a.eps = float(eps)
    a.num_q_heads = q.shape[1]
    a.start_pos = start_pos.data_ptr()
    a.new_offsets = _ptr(new_offsets)
    a.batch = batch
    a.max_new_tokens = max_new
    a.err = _ptr(err)
    _raise_rc(nat.load().bl_qk_norm_rope_append(a, _stream(key.device)))
    return q_out


def paged_gather(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    max_len: int,
    *,
    row_ids: torch.Tensor | None = None,
    out: tuple[torch.Tensor, torch.Tensor] | None = None,
    zero_fill: bool = True,
    err: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense ``[B, Hkv, max_len, D]`` copy of the cached tokens, zero padded.

    Mirrors PagedLayerKV.read + BatchLayerKV._pad
    (src/barellm/engine/paged_kv_cache.py:215-240, batched_kv_cache.py:80-95).
    """
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    _int32_on(seq_lens, key_cache.device, "seq_lens")
    _check(max_len > 0, "KV cache is empty")
    batch = seq_lens.shape[0]
    hkv, d = key_cache.shape[2], key_cache.shape[4]
    if out is None:
        shape = (batch, hkv, max_len, d)
        k_out = torch.empty(shape, dtype=key_cache.dtype, device=key_cache.device)
        v_out = torch.empty_like(k_out)
    else:
        k_out, v_out = out
        _check(k_out.shape == (batch, hkv, max_len, d) and v_out.shape == k_out.shape, "gather output shape mismatch")
        _check(k_out.stride() == v_out.stride() and k_out.stride(3) == 1, "gather outputs need identical strides, D contiguous")
    a = nat.GatherArgs()
    a.kv = pl
    a.seq_lens = seq_lens.data_ptr()
    a.batch = batch
    a.k_out = k_out.data_ptr()
    a.v_out = v_out.data_ptr()
    a.out_stride_b, a.out_stride_h, a.out_stride_t = k_out.stride(0), k_out.stride(1), k_out.stride(2)
    a.max_len = max_len
    a.zero_fill = 1 if zero_fill else 0
    a.err = _ptr(err)
    _raise_rc(nat.load().bl_paged_gather(a, _stream(key_cache.device)))
    return k_out, v_out


def decode_workspace_bytes(batch: int, num_q_heads: int, head_dim: int, block_size: int, max_seq_len: int) -> int:
    return int(nat.load().bl_paged_decode_workspace_bytes(batch, num_q_heads, head_dim, block_size, max_seq_len))


_WORKSPACES: dict[int, torch.Tensor] = {}
_PLAN_STUBS: dict[tuple, torch.Tensor] = {}
_PLAN_SERIAL: dict[int, int] = {}


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device scratch buffer for split-K decode (grown, never shrunk).

    Calls on one device share it, so decode calls must be ordered on a single
    stream (which the engine guarantees).  Growing it invalidates any plan it
    held."""
    idx = _dev_index(device)
    ws = _WORKSPACES.get(idx)
    if ws is None or ws.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        if ws is not None:
            size = max(size, 2 * ws.numel())
        ws = torch.empty(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _WORKSPACES[idx] = ws
        _PLAN_SERIAL[idx] = _PLAN_SERIAL.get(idx, 0) + 1
    return ws


def plan_serial(device: torch.device) -> int:
    """Changes whenever the shared workspace's plan is replaced."""
    return _PLAN_SERIAL.get(_dev_index(device), 0)


def _decode_checks(q, key_cache, seq_lens, out) -> None:
    """The decode input checks one at a time, raising the first that fails."""
    _require_cuda(q, "q")
    if q.ndim == 4:
        _check(q.shape[2] == 1, "decode takes one query token per request")
        q3 = q[:, :, 0, :]
    else:
        q3 = q
    _check(q3.ndim == 3, "q must be [B, Hq, D] or [B, Hq, 1, D]")
    _check(q3.dtype == key_cache.dtype and q3.device == key_cache.device, "q must match the K/V pool dtype and device")
    _check(q3.shape[2] == key_cache.shape[4], "Head dimension cannot change")
    _check(q3.stride(2) == 1, "q head_dim must be contiguous")
    _int32_on(seq_lens, q3.device, "seq_lens")
    batch, hq, d = q3.shape
    _check(seq_lens.shape[0] == batch, "batch size must match number of caches")
    _check(hq % key_cache.shape[2] == 0, "num_heads must divide evenly by num_kv_heads")
    if out is not None:
        out3 = out[:, :, 0, :] if out.ndim == 4 else out
        _check(out3.shape == (batch, hq, d) and out3.stride(2) == 1, "decode output must be [B, Hq, D], D contiguous")


def _decode_args(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    max_seq_len: int,
    scale: float | None,
    out: torch.Tensor | None,
    row_ids: torch.Tensor | None,
    ws: torch.Tensor | None,
    plan_ready: bool,
    err: torch.Tensor | None,
) -> tuple[nat.DecodeArgs, torch.Tensor, torch.Tensor]:
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    qs = q.shape
    qst = q.stride()
    nd = len(qs)
    # [B, Hq, 1, D] and [B, Hq, D] are read through their B / Hq strides
    if nd == 4:
        batch, hq, t1, d = qs
        qd = qst[3]
    else:
        batch, hq, d = qs if nd == 3 else (0, 0, 0)
        t1, qd = 1, qst[2] if nd == 3 else 0
    dev = key_cache.device
    if out is not None:
        os_, ost = out.shape, out.stride()
        out_ok = (os_ == (batch, hq, d) and ost[2] == 1) or (os_ == (batch, hq, 1, d) and ost[3] == 1)
    else:
        out_ok = True
    if not (nd in (3, 4) and t1 == 1 and q.dtype is key_cache.dtype and q.device == dev and d == key_cache.shape[4]
            and qd == 1 and seq_lens.dtype is torch.int32 and seq_lens.device == dev
            and seq_lens.shape[0] == batch and hq % key_cache.shape[2] == 0 and out_ok and q.is_cuda):
        _decode_checks(q, key_cache, seq_lens, out)
    if out is None:
        out = torch.empty((batch, hq, d), dtype=q.dtype, device=q.device)
    ost = out.stride()
    if ws is None:
        ws = workspace(q.device, decode_workspace_bytes(batch, hq, d, key_cache.shape[3], max_seq_len))
    a = nat.DecodeArgs(pl, q.data_ptr(), qst[0], qst[1], out.data_ptr(), ost[0], ost[1], seq_lens.data_ptr(), batch,
                       hq, 1.0 / math.sqrt(d) if scale is None else float(scale), ws.data_ptr(),
                       ws.numel() * ws.element_size(), max_seq_len, 1 if plan_ready else 0,
                       None if err is None else err.data_ptr())
    return a, out, ws


def paged_decode_plan(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    max_seq_len: int,
    num_q_heads: int,
    *,
    row_ids: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """Builds the split-K plan for ``seq_lens`` once; reusable by every layer."""
    batch = seq_lens.shape[0]
    d = key_cache.shape[4]
    # the plan reads no q / out: a broadcast [B, Hq, D] view of one cached
    # D-element row stands in for them
    key = (key_cache.device, key_cache.dtype, d)
    row = _PLAN_STUBS.get(key)
    if row is None:
        row = _PLAN_STUBS[key] = torch.zeros(d, dtype=key_cache.dtype, device=key_cache.device)
    q_shape = row.as_strided((batch, num_q_heads, d), (0, 0, 1))
    a, _, ws = _decode_args(q_shape, key_cache, value_cache, 0, block_tables, seq_lens, max_seq_len, None,
                            q_shape, row_ids, ws, False, err)
    _raise_rc(nat.load().bl_paged_decode_plan(a, _stream(key_cache.device)))
    idx = _dev_index(key_cache.device)
    if _WORKSPACES.get(idx) is ws:
        _PLAN_SERIAL[idx] = _PLAN_SERIAL.get(idx, 0) + 1
    return ws


def paged_decode(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    max_seq_len: int,
    *,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    row_ids: torch.Tensor | None = None,
    ws: torch.Tensor | None = None,
    plan_ready: bool = False,
    err: torch.Tensor | None = None,
    stage: str = "all",
) -> torch.Tensor:
    """One-token GQA attention over paged K/V, read in place; returns ``[B, Hq, D]``.

    ``stage``: "all" (plan unless ``plan_ready``, attention, reduce),
    "attention" (attention kernel only; needs ``plan_ready``) or "reduce"
    (split-K merge only).

    Equals the reference decode chain read -> _pad -> repeat_interleave ->
    attention_mask -> SDPA (src/barellm/attention/backend.py:34-61).
    ``seq_lens`` are post-append lengths (>= 1), ``max_seq_len`` a host-side
    upper bound used only to size the split-K workspace.
    """
    a, out, used_ws = _decode_args(q, key_cache, value_cache, layer, block_tables, seq_lens, max_seq_len, scale,
                                   out, row_ids, ws, plan_ready, err)
    lib = nat.load()
    if stage == "all":
        fn = lib.bl_paged_decode
    elif stage == "attention":
        fn = lib.bl_paged_decode_attention
    elif stage == "reduce":
        fn = lib.bl_paged_decode_reduce
    else:
        raise KeyError(stage)
    _raise_rc(fn(a, _stream(key_cache.device)))
    if not plan_ready and stage == "all":
        idx = _dev_index(key_cache.device)
        if _WORKSPACES.get(idx) is used_ws:  # this call replaced the shared plan
            _PLAN_SERIAL[idx] = _PLAN_SERIAL.get(idx, 0) + 1
    return out


def paged_decode_noalloc(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    max_seq_len: int,
    out: torch.Tensor,
    *,
    scale: float | None = None,
    row_ids: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode through ``bl_paged_decode_noalloc``: the split-K scratch is the
    library's built-in 16 MiB array, so neither this call nor the library
    allocates device memory (the caller passes ``out``).  For callers whose
    host framework owns all device memory or who must keep cudaMalloc off the
    decode loop.  Calls share the one array: order them on one stream."""
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    _require_cuda(q, "q")
    q3 = q[:, :, 0, :] if q.ndim == 4 else q
    out3 = out[:, :, 0, :] if out.ndim == 4 else out
    _check(q3.ndim == 3 and q3.stride(2) == 1, "q must be [B, Hq, D] or [B, Hq, 1, D], D contiguous")
    _check(q3.dtype == key_cache.dtype and q3.device == key_cache.device, "q must match the K/V pool dtype and device")
    _check(out3.shape == q3.shape and out3.stride(2) == 1 and out3.dtype == q3.dtype, "out must match q")
    _int32_on(seq_lens, q3.device, "seq_lens")
    a = nat.DecodeArgs()
    a.kv = pl
    a.q = q3.data_ptr()
    a.q_stride_b, a.q_stride_h = q3.stride(0), q3.stride(1)
    a.out = out3.data_ptr()
    a.out_stride_b, a.out_stride_h = out3.stride(0), out3.stride(1)
    a.seq_lens = seq_lens.data_ptr()
    a.batch, a.num_q_heads = q3.shape[0], q3.shape[1]
    a.scale = 1.0 / math.sqrt(q3.shape[2]) if scale is None else float(scale)
    a.max_seq_len = max_seq_len
    a.err = _ptr(err)
    _raise_rc(nat.load().bl_paged_decode_noalloc(a, _stream(q3.device)))
    return out


def ipc_export(t: torch.Tensor) -> bytes:
    """Handle (72 bytes) that lets another process of this node map ``t``'s
    memory with :func:`ipc_import` (CUDA IPC; ``t`` must stay alive)."""
    _require_cuda(t, "t")
    h = nat.IpcHandle()
    _raise_rc(nat.load().bl_ipc_export(t.data_ptr(), ctypes.byref(h)))
    return bytes(h)


def ipc_import(handle: bytes, device: torch.device) -> int:
    """Maps memory exported by another process into this one, for ``device``;
    returns the address that matches the exporter's tensor pointer."""
    _check(len(handle) == ctypes.sizeof(nat.IpcHandle), "not a bl_ipc_handle")
    h = nat.IpcHandle.from_buffer_copy(handle)
    ptr = ctypes.c_void_p()
    with torch.cuda.device(device):
        _raise_rc(nat.load().bl_ipc_import(ctypes.byref(h), ctypes.byref(ptr)))
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    """Unmaps an address returned by :func:`ipc_import`."""
    _raise_rc(nat.load().bl_ipc_close(ptr))


def paged_prefill(
    q: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    layer: int,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    q_offsets: torch.Tensor | None = None,
    max_q_len: int | None = None,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    row_ids: torch.Tensor | None = None,
    err: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal attention of new queries over prefix + themselves, read in place.

    ``q``: ``[B, Hq, T, D]`` (any strides, D contiguous), or ``[1, Hq, sum C, D]``
    packed with ``q_offsets`` ``[B+1]``.  ``seq_lens`` are the total lengths
    after the append; query i of a row with C queries sees keys
    ``0 .. seq_len - C + i``.  Returns a tensor shaped like ``q`` whose memory is
    ``[B, T, Hq, D]`` (so ``out.transpose(1, 2).reshape(B, T, -1)`` is free).
    """
    pl = _paged_layer(key_cache, value_cache, layer, block_tables, row_ids)
    _require_cuda(q, "q")
    _check(q.ndim == 4, "q must be [B, Hq, T, D]")
    _check(q.dtype == key_cache.dtype and q.device == key_cache.device, "q must match the K/V pool dtype and device")
    _check(q.shape[3] == key_cache.shape[4], "Head dimension cannot change")
    _check(q.shape[2] > 0, "K/V sequence length must be greater than zero")
    _check(q.stride(3) == 1, "q head_dim must be contiguous")
    _check(q.shape[1] % key_cache.shape[2] == 0, "num_heads must divide evenly by num_kv_heads")
    _int32_on(seq_lens, q.device, "seq_lens")
    batch = seq_lens.shape[0]
    if q_offsets is None:
        _check(q.shape[0] == batch, "batch size must match number of caches")
        mq = q.shape[2]
    else:
        _int32_on(q_offsets, q.device, "q_offsets")
        _check(q.shape[0] == 1 and q_offsets.shape[0] == batch + 1, "packed queries need [1, Hq, T, D] and [B+1] offsets")
        _check(max_q_len is not None and max_q_len > 0, "packed prefill needs max_q_len")
        mq = int(max_q_len)
    if out is None:
        b0, hq, t, d = q.shape
        out = torch.empty((b0, t, hq, d), dtype=q.dtype, device=q.device).transpose(1, 2)
    _check(out.shape == q.shape and out.stride(3) == 1, "prefill output must match q's shape, D contiguous")
    a = nat.PrefillArgs()
    a.kv = pl
    a.q = q.data_ptr()
    packed = q_offsets is not None  # packed rows are addressed by q_offsets alone
    a.q_stride_b, a.q_stride_h, a.q_stride_t = (0 if packed else q.stride(0)), q.stride(1), q.stride(2)
    a.out = out.data_ptr()
    a.out_stride_b, a.out_stride_h, a.out_stride_t = (0 if packed else out.stride(0)), out.stride(1), out.stride(2)
    a.q_offsets = _ptr(q_offsets)
    a.seq_lens = seq_lens.data_ptr()
    a.batch = batch
    a.num_q_heads = q.shape[1]
    a.max_q_len = mq
    a.scale = 1.0 / math.sqrt(q.shape[3]) if scale is None else float(scale)
    a.err = _ptr(err)
    _raise_rc(nat.load().bl_paged_prefill(a, _stream(q.device)))
    return out


def rms_norm(
    x: torch.Tensor,
    weight: torch.Tensor,
    eps: float,
    *,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    x_out: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm over the last axis in one kernel (decoder support around the
    attention path): ``rmsnorm(x) * weight`` with the reference's roundings
    (src/barellm/models/norm.py:14-21).  With ``residual`` it first forms
    ``x + residual`` (rounded to the element type, as a tensor add) and returns
    ``(x + residual, rmsnorm(x + residual) * weight)``.  Rows may be strided;
    the last axis must be contiguous."""
    _require_cuda(x, "x")
    h = x.shape[-1]
    _check(weight.shape == (h,) and weight.dtype == x.dtype and weight.device == x.device and weight.stride(0) == 1,
           "norm weight must be [hidden] of the input's dtype and device")
    _check(x.dtype in DTYPE_CODE, f"unsupported dtype {x.dtype}")
    _check(x.stride(-1) == 1, "x must have a contiguous last dimension")
    x2 = x.reshape(-1, h) if x.dim() != 2 else x
    _check(x2.stride(-1) == 1, "x rows must be addressable with one stride")
    rows = x2.shape[0]
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    o2 = out.view(-1, h)
    r2 = None
    xo2 = None
    if residual is not None:
        _check(residual.shape == x.shape and residual.dtype == x.dtype and residual.device == x.device,
               "residual must match x")
        r2 = residual.reshape(-1, h)
        _check(r2.stride(-1) == 1, "residual must have a contiguous last dimension")
        if x_out is None:
            x_out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        xo2 = x_out.view(-1, h)
    a = nat.RmsNormArgs(x2.data_ptr(), None if r2 is None else r2.data_ptr(), None if xo2 is None else xo2.data_ptr(),
                        o2.data_ptr(), weight.data_ptr(), rows, h, x2.stride(0), 0 if r2 is None else r2.stride(0),
                        0 if xo2 is None else xo2.stride(0), o2.stride(0), float(eps), DTYPE_CODE[x.dtype])
    _raise_rc(nat.load().bl_rms_norm(a, _stream(x.device)))
    return out if residual is None else (x_out, out)


def decode_path(dtype: torch.dtype, head_dim: int, block_size: int, num_q_heads: int, num_kv_heads: int) -> int:
    return int(nat.load().bl_decode_path(DTYPE_CODE[dtype], head_dim, block_size, num_q_heads, num_kv_heads))


def prefill_path(dtype: torch.dtype, head_dim: int, block_size: int, num_q_heads: int, num_kv_heads: int) -> int:
    return int(nat.load().bl_prefill_path(DTYPE_CODE[dtype], head_dim, block_size, num_q_heads, num_kv_heads))
