"""ctypes binding of the C ABI declared in ``include/barellm_b200.h``.

The structures below mirror the header field for field; ``tests/test_abi.py``
compiles a C probe against the header and checks every size and offset.
There is no fallback: if the shared library is missing the first call raises.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libbarellm_b200.so"

# return codes / dtype codes / device error bits (include/barellm_b200.h)
BL_OK = 0
BL_ERR_ARG = 1
BL_ERR_DTYPE = 2
BL_ERR_CAPACITY = 3
BL_ERR_LAUNCH = 4
BL_ERR_UNSUPPORTED = 5

BL_F32 = 0
BL_F16 = 1
BL_BF16 = 2

BL_DEVERR_BLOCK_ID = 1
BL_DEVERR_TABLE = 2
BL_DEVERR_TIMEOUT = 4
BL_DEVERR_WORKSPACE = 8

EXPORTED = (
    "bl_paged_append",
    "bl_qk_norm_rope_append",
    "bl_paged_gather",
    "bl_paged_decode_workspace_bytes",
    "bl_paged_decode_plan",
    "bl_paged_decode",
    "bl_paged_decode_attention",
    "bl_paged_decode_reduce",
    "bl_paged_decode_noalloc",
    "bl_paged_decode_allgather",
    "bl_ipc_export",
    "bl_ipc_import",
    "bl_ipc_close",
    "bl_paged_prefill",
    "bl_rms_norm",
    "bl_last_error",
    "bl_abi_version",
    "bl_decode_path",
    "bl_prefill_path",
)


class PagedLayer(Structure):
    _fields_ = [
        ("k_pool", c_void_p),
        ("v_pool", c_void_p),
        ("num_layers", c_int64),
        ("num_blocks", c_int64),
        ("num_kv_heads", c_int64),
        ("block_size", c_int64),
        ("head_dim", c_int64),
        ("dtype", c_int32),
        ("layer", c_int32),
        ("block_tables", c_void_p),
        ("bt_stride", c_int64),
        ("bt_width", c_int64),
        ("row_ids", c_void_p),
    ]


class AppendArgs(Structure):
    _fields_ = [
        ("kv", PagedLayer),
        ("k_new", c_void_p),
        ("v_new", c_void_p),
        ("new_stride_b", c_int64),
        ("new_stride_h", c_int64),
        ("new_stride_t", c_int64),
        ("v_stride_b", c_int64),
        ("v_stride_h", c_int64),
        ("v_stride_t", c_int64),
        ("start_pos", c_void_p),
        ("new_offsets", c_void_p),
        ("batch", c_int64),
        ("max_new_tokens", c_int64),
        ("err", c_void_p),
    ]


class GatherArgs(Structure):
    _fields_ = [
        ("kv", PagedLayer),
        ("seq_lens", c_void_p),
        ("batch", c_int64),
        ("k_out", c_void_p),
        ("v_out", c_void_p),
        ("out_stride_b", c_int64),
        ("out_stride_h", c_int64),
        ("out_stride_t", c_int64),
        ("max_len", c_int64),
        ("zero_fill", c_int32),
        ("err", c_void_p),
    ]


class DecodeArgs(Structure):
    _fields_ = [
        ("kv", PagedLayer),
        ("q", c_void_p),
        ("q_stride_b", c_int64),
        ("q_stride_h", c_int64),
        ("out", c_void_p),
        ("out_stride_b", c_int64),
        ("out_stride_h", c_int64),
        ("seq_lens", c_void_p),
        ("batch", c_int64),
        ("num_q_heads", c_int64),
        ("scale", c_float),
        ("workspace", c_void_p),
        ("workspace_bytes", c_size_t),
        ("max_seq_len", c_int64),
        ("plan_ready", c_int32),
        ("err", c_void_p),
    ]


BL_MAX_RANKS = 8


class HeadGather(Structure):
    _fields_ = [
        ("world", c_int32),
        ("rank", c_int32),
        ("peer_out", c_void_p * BL_MAX_RANKS),
        ("peer_signal", c_void_p * BL_MAX_RANKS),
        ("epoch", c_void_p),
        ("head_offset", c_int64),
        ("timeout_ns", c_int64),
    ]


class IpcHandle(Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64), ("offset", ctypes.c_uint64)]


class PrefillArgs(Structure):
    _fields_ = [
        ("kv", PagedLayer),
        ("q", c_void_p),
        ("q_stride_b", c_int64),
        ("q_stride_t", c_int64),
        ("q_stride_h", c_int64),
        ("out", c_void_p),
        ("out_stride_b", c_int64),
        ("out_stride_t", c_int64),
        ("out_stride_h", c_int64),
        ("q_offsets", c_void_p),
        ("seq_lens", c_void_p),
        ("batch", c_int64),
        ("num_q_heads", c_int64),
        ("max_q_len", c_int64),
        ("scale", c_float),
        ("err", c_void_p),
    ]


class QkPrepArgs(Structure):
    _fields_ = [
        ("kv", PagedLayer),
        ("q_in", c_void_p),
        ("q_in_stride_b", c_int64),
        ("q_in_stride_h", c_int64),
        ("q_in_stride_t", c_int64),
        ("k_in", c_void_p),
        ("k_in_stride_b", c_int64),
        ("k_in_stride_h", c_int64),
        ("k_in_stride_t", c_int64),
        ("v_in", c_void_p),
        ("v_in_stride_b", c_int64),
        ("v_in_stride_h", c_int64),
        ("v_in_stride_t", c_int64),
        ("q_out", c_void_p),
        ("q_out_stride_b", c_int64),
        ("q_out_stride_h", c_int64),
        ("q_out_stride_t", c_int64),
        ("q_norm_weight", c_void_p),
        ("k_norm_weight", c_void_p),
        ("cos", c_void_p),
        ("sin", c_void_p),
        ("rope_stride_b", c_int64),
        ("rope_stride_t", c_int64),
        ("eps", c_float),
        ("pad0", c_int32),
        ("num_q_heads", c_int64),
        ("start_pos", c_void_p),
        ("new_offsets", c_void_p),
        ("batch", c_int64),
        ("max_new_tokens", c_int64),
        ("err", c_void_p),
    ]


class RmsNormArgs(Structure):
    _fields_ = [
        ("x", c_void_p),
        ("residual", c_void_p),
        ("x_out", c_void_p),
        ("out", c_void_p),
        ("weight", c_void_p),
        ("rows", c_int64),
        ("hidden", c_int64),
        ("x_stride", c_int64),
        ("residual_stride", c_int64),
        ("x_out_stride", c_int64),
        ("out_stride", c_int64),
        ("eps", c_float),
        ("dtype", c_int32),
    ]


STRUCTS = {
    "bl_paged_layer": PagedLayer,
    "bl_qk_prep_args": QkPrepArgs,
    "bl_append_args": AppendArgs,
    "bl_gather_args": GatherArgs,
    "bl_decode_args": DecodeArgs,
    "bl_head_gather": HeadGather,
    "bl_ipc_handle": IpcHandle,
    "bl_prefill_args": PrefillArgs,
    "bl_rms_norm_args": RmsNormArgs,
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library (once) and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"barellm_b200 CUDA library not found at {LIB_PATH}; "
            "build it with `python -m barellm_b200.build`"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.bl_paged_append.argtypes = [POINTER(AppendArgs), c_void_p]
    lib.bl_paged_append.restype = c_int
    lib.bl_qk_norm_rope_append.argtypes = [POINTER(QkPrepArgs), c_void_p]
    lib.bl_qk_norm_rope_append.restype = c_int
    lib.bl_paged_gather.argtypes = [POINTER(GatherArgs), c_void_p]
    lib.bl_paged_gather.restype = c_int
    lib.bl_paged_decode_workspace_bytes.argtypes = [c_int64] * 5
    lib.bl_paged_decode_workspace_bytes.restype = c_size_t
    lib.bl_paged_decode_plan.argtypes = [POINTER(DecodeArgs), c_void_p]
    lib.bl_paged_decode_plan.restype = c_int
    for fn in (lib.bl_paged_decode, lib.bl_paged_decode_attention, lib.bl_paged_decode_reduce):
        fn.argtypes = [POINTER(DecodeArgs), c_void_p]
        fn.restype = c_int
    lib.bl_paged_decode_noalloc.argtypes = [POINTER(DecodeArgs), c_void_p]
    lib.bl_paged_decode_noalloc.restype = c_int
    lib.bl_paged_decode_allgather.argtypes = [POINTER(DecodeArgs), POINTER(HeadGather), c_void_p]
    lib.bl_paged_decode_allgather.restype = c_int
    lib.bl_ipc_export.argtypes = [c_void_p, POINTER(IpcHandle)]
    lib.bl_ipc_export.restype = c_int
    lib.bl_ipc_import.argtypes = [POINTER(IpcHandle), POINTER(c_void_p)]
    lib.bl_ipc_import.restype = c_int
    lib.bl_ipc_close.argtypes = [c_void_p]
    lib.bl_ipc_close.restype = c_int
    lib.bl_paged_prefill.argtypes = [POINTER(PrefillArgs), c_void_p]
    lib.bl_paged_prefill.restype = c_int
    lib.bl_rms_norm.argtypes = [POINTER(RmsNormArgs), c_void_p]
    lib.bl_rms_norm.restype = c_int
    lib.bl_last_error.argtypes = []
    lib.bl_last_error.restype = c_char_p
    lib.bl_abi_version.argtypes = []
    lib.bl_abi_version.restype = c_int
    lib.bl_decode_path.argtypes = [c_int32, c_int64, c_int64, c_int64, c_int64]
    lib.bl_decode_path.restype = c_int
    lib.bl_prefill_path.argtypes = [c_int32, c_int64, c_int64, c_int64, c_int64]
    lib.bl_prefill_path.restype = c_int
    _lib = lib
    return lib


def last_error() -> str:
    msg = load().bl_last_error()
    return msg.decode() if msg else ""
