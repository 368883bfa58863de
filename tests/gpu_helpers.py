"""Builds device-side paged pools from the seeded cases (GPU tests only)."""

from __future__ import annotations

import numpy as np
import torch

import cases
from barellm_b200 import ops

SENTINEL = -7.0


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to bfloat16 (nearest even), kept as float32."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def round_for(dtype: torch.dtype):
    if dtype == torch.float32:
        return lambda a: a
    return lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dtype).float().numpy()


def padded_tables(tables: list[np.ndarray], width: int | None = None) -> np.ndarray:
    w = width or max(len(x) for x in tables)
    out = np.full((len(tables), w), -1, dtype=np.int32)
    for i, x in enumerate(tables):
        out[i, : len(x)] = x
    return out


def to_dev(x: np.ndarray, dtype: torch.dtype, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).to(device)


class DecodeState:
    """Pool after a batched history append (packed, ragged) and a one-token
    append per request, both through the CUDA append kernel."""

    def __init__(self, case: cases.DecodeCase, dtype: torch.dtype, device):
        self.case = case
        self.dtype = dtype
        shape = (1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
        self.k_cache = torch.full(shape, SENTINEL, dtype=dtype, device=device)
        self.v_cache = torch.full(shape, SENTINEL, dtype=dtype, device=device)
        self.tables = case.block_tables()
        self.bt = torch.from_numpy(padded_tables(self.tables)).to(device)
        lens = [int(n) for n in case.lengths]
        offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        kh = to_dev(np.concatenate(case.k_hist, axis=2), dtype, device)
        vh = to_dev(np.concatenate(case.v_hist, axis=2), dtype, device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, torch.zeros(len(lens), dtype=torch.int32, device=device),
                         kh, vh, new_offsets=torch.from_numpy(offs).to(device), max_new_tokens=max(lens), err=self.err)
        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt,
                         torch.tensor(lens, dtype=torch.int32, device=device),
                         to_dev(case.k_new, dtype, device), to_dev(case.v_new, dtype, device), err=self.err)
        self.seq_lens_list = [n + 1 for n in lens]
        self.seq_lens = torch.tensor(self.seq_lens_list, dtype=torch.int32, device=device)
        self.q = to_dev(case.q, dtype, device)

    def decode(self, **kw) -> torch.Tensor:
        return ops.paged_decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens,
                                max(self.seq_lens_list), err=self.err, **kw)
