"""Fused QK-RMSNorm + RoPE + paged append (bl_qk_norm_rope_append) against the
reference's own QK-norm + RoPE outputs (golden fixtures) and its append
semantics.

Bars: float32 within 1e-5 of the reference; bf16 equal to the reference's
bf16 tensor-op chain except a rare element one bf16 step away (the mean
square's summation order), V copied bit-exactly, untouched slots unchanged."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import gpu_helpers as gh
from barellm_b200 import _native as nat
from barellm_b200 import ops
from oracle import paged_oracle as orc
from test_oracle_golden import assert_bf16_rope_close

pytestmark = pytest.mark.gpu

GOLDEN = cases.__file__.rsplit("/", 1)[0]
TAG = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f32"}  # fp16: the f32 tables, rounded


def golden(name):
    return np.load(f"{GOLDEN}/{name}.npz")


class PrepState:
    def __init__(self, case: cases.QkPrepCase, dtype: torch.dtype, device):
        self.case, self.dtype, self.device = case, dtype, device
        shape = (1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
        self.k_cache = torch.full(shape, gh.SENTINEL, dtype=dtype, device=device)
        self.v_cache = torch.full(shape, gh.SENTINEL, dtype=dtype, device=device)
        self.tables = case.block_tables()
        self.bt = torch.from_numpy(gh.padded_tables(self.tables)).to(device)
        self.starts = torch.tensor(case.starts, dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)

    def slots(self, cache: torch.Tensor) -> np.ndarray:
        """[B, Hkv, T, D] contents of the step's slots, read on the host."""
        c = cache.float().cpu().numpy()
        case = self.case
        out = np.zeros((case.batch, case.num_kv_heads, case.new_tokens, case.head_dim), dtype=np.float32)
        for b, bt in enumerate(self.tables):
            start = int(case.starts[b])
            k, _ = orc.read(c, c, 0, bt, start + case.new_tokens)
            out[b] = k[0, :, start:]
        return out


def run_case(name: str, dtype: torch.dtype, device, packed: bool = False):
    case = cases.qk_prep_case(name)
    g = golden(name)
    tag = TAG[dtype]
    st = PrepState(case, dtype, device)
    q = gh.to_dev(case.q, dtype, device)
    k = gh.to_dev(case.k, dtype, device)
    v = gh.to_dev(case.v, dtype, device)
    cos = gh.to_dev(g[f"cos_{tag}"], dtype, device)  # [B, 1, T, D]
    sin = gh.to_dev(g[f"sin_{tag}"], dtype, device)
    qw = gh.to_dev(g[f"q_weight_{tag}"], dtype, device)
    kw = gh.to_dev(g[f"k_weight_{tag}"], dtype, device)
    if not packed:
        # q as the model produces it: [B, T, H, D] memory viewed as [B, H, T, D]
        q = q.transpose(1, 2).contiguous().transpose(1, 2)
        q_out = ops.qk_norm_rope_append(q, k, v, qw, kw, cos, sin, case.eps, st.k_cache, st.v_cache, 0, st.bt,
                                        st.starts, err=st.err)
    else:
        t = case.new_tokens
        pack = lambda x: x.permute(1, 0, 2, 3).reshape(1, x.shape[1], -1, x.shape[3])  # noqa: E731
        offs = torch.arange(0, (case.batch + 1) * t, t, dtype=torch.int32, device=device)
        cos_p = cos.permute(1, 0, 2, 3).reshape(1, 1, -1, cos.shape[3])
        sin_p = sin.permute(1, 0, 2, 3).reshape(1, 1, -1, sin.shape[3])
        q_out = ops.qk_norm_rope_append(pack(q), pack(k), pack(v), qw, kw, cos_p, sin_p, case.eps, st.k_cache,
                                        st.v_cache, 0, st.bt, st.starts, new_offsets=offs, max_new_tokens=t,
                                        err=st.err)
        q_out = q_out.reshape(q.shape[1], case.batch, t, -1).permute(1, 0, 2, 3)
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    return case, g, st, q_out.float().cpu().numpy()


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("name", list(cases.QK_PREP_CASES))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_qk_prep_matches_reference(cuda, native_lib, name, dtype, packed):
    case, g, st, q_out = run_case(name, dtype, cuda, packed)
    tag = TAG[dtype]
    k_out = st.slots(st.k_cache)
    v_out = st.slots(st.v_cache)
    rnd = gh.round_for(dtype)
    np.testing.assert_array_equal(v_out, rnd(case.v))
    if dtype == torch.float32:
        np.testing.assert_allclose(q_out, g["q_out_f32"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(k_out, g["k_out_f32"], atol=1e-5, rtol=1e-5)
        return
    cos, sin = rnd(g[f"cos_{tag}"]), rnd(g[f"sin_{tag}"])
    for out, src, key in ((q_out, case.q, "q"), (k_out, case.k, "k")):
        w = rnd(g[f"{key}_weight_{tag}"])
        normed = orc.rms_norm(rnd(src), w, case.eps, rnd)
        # bf16: the reference's own output; fp16: the oracle with fp16 rounding
        want = g[f"{key}_out_bf16"] if dtype == torch.bfloat16 else orc.qk_norm_rope(rnd(src), w, cos, sin, case.eps, rnd)
        assert_bf16_rope_close(out, want, normed, cos, sin)


def test_qk_prep_leaves_other_slots_untouched(cuda, native_lib):
    case, g, st, _ = run_case("qk_prep_tiny", torch.float32, cuda)
    kc = st.k_cache.cpu().numpy()
    touched = np.zeros(kc.shape[:4], dtype=bool)
    for b, bt in enumerate(st.tables):
        for pos in range(int(case.starts[b]), int(case.starts[b]) + case.new_tokens):
            touched[0, bt[pos // case.block_size], :, pos % case.block_size] = True
    assert np.all(kc[~touched] == gh.SENTINEL)


def test_qk_prep_reports_a_short_block_table(cuda, native_lib):
    case = cases.qk_prep_case("qk_prep_tiny")
    st = PrepState(case, torch.float32, cuda)
    starts = torch.tensor([10, 15], dtype=torch.int32, device=cuda)  # positions in blocks 2 and 3
    bt = st.bt[:, :1].contiguous()  # one block wide
    q, k, v = (gh.to_dev(x, torch.float32, cuda) for x in (case.q, case.k, case.v))
    d = case.head_dim
    ones = torch.ones(d, device=cuda)
    cos = torch.ones((1, 1, case.new_tokens, d), device=cuda)
    ops.qk_norm_rope_append(q, k, v, ones, ones, cos, torch.zeros_like(cos), case.eps, st.k_cache, st.v_cache, 0,
                            bt, starts, err=st.err)
    torch.cuda.synchronize()
    assert int(st.err.item()) & nat.BL_DEVERR_TABLE
    assert np.all(st.k_cache.cpu().numpy() == gh.SENTINEL)  # nothing written through a missing table entry
