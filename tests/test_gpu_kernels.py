"""Parity of the CUDA kernels (called through the C ABI) with the oracle and
with the reference's golden outputs.

Bars: append and gather bit-exact; fp32 attention within 1e-5; bf16/fp16
attention within max-abs 2e-2 and mean-abs 2e-3 of the fp64 oracle evaluated
on the same (rounded) inputs, and of the reference's own bf16 CPU output."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import gpu_helpers as gh
from barellm_b200 import _native as nat
from barellm_b200 import ops
from oracle import paged_oracle as orc

pytestmark = pytest.mark.gpu

GOLDEN = cases.__file__.rsplit("/", 1)[0]
BF16_MAX, BF16_MEAN = 2e-2, 2e-3
F32_TOL = 1e-5


def golden(name):
    return np.load(f"{GOLDEN}/{name}.npz")


def assert_close_lowp(actual: np.ndarray, expected: np.ndarray):
    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    assert np.isfinite(actual).all()
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (float(err.max()), float(err.mean()))


# --------------------------------------------------------------------------
# append / gather (bit-exact)
# --------------------------------------------------------------------------
def test_storage_sequence_bit_exact(cuda, native_lib):
    g = golden("storage_sequence")
    kc = torch.full(g["key_cache"].shape, gh.SENTINEL, dtype=torch.float32, device=cuda)
    vc = torch.full_like(kc, gh.SENTINEL)
    tables = {rid: torch.from_numpy(g[f"table_{rid}"]).view(1, -1).to(cuda) for rid in ("A", "B")}
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    lens = {}
    for i, (rid, layer, start) in enumerate(zip(g["step_rid"], g["step_layer"], g["step_start"])):
        key = torch.from_numpy(g[f"step{i}_key"]).to(cuda)
        ops.paged_append(kc, vc, int(layer), tables[str(rid)], torch.tensor([int(start)], dtype=torch.int32, device=cuda),
                         key, key + 100, err=err)
        lens[(str(rid), int(layer))] = int(start) + key.shape[2]
    assert int(err.item()) == 0
    np.testing.assert_array_equal(kc.cpu().numpy(), g["key_cache"])
    np.testing.assert_array_equal(vc.cpu().numpy(), g["value_cache"])
    for rid, layer in (("A", 0), ("A", 1), ("B", 0)):
        n = lens[(rid, layer)]
        k, v = ops.paged_gather(kc, vc, layer, tables[rid], torch.tensor([n], dtype=torch.int32, device=cuda), n)
        np.testing.assert_array_equal(k.cpu().numpy(), g[f"read_{rid}{layer}_k"])
        np.testing.assert_array_equal(v.cpu().numpy(), g[f"read_{rid}{layer}_v"])


def test_batched_read_pads_with_zeros(cuda, native_lib):
    g = golden("batch_read")
    kc = torch.from_numpy(g["key_cache"]).to(cuda)
    vc = torch.from_numpy(g["value_cache"]).to(cuda)
    bt = torch.from_numpy(g["block_tables"]).to(cuda)
    lens = torch.from_numpy(g["lengths"]).to(cuda)
    for layer in range(2):
        k, v = ops.paged_gather(kc, vc, layer, bt, lens, int(g["lengths"].max()))
        np.testing.assert_array_equal(k.cpu().numpy(), g[f"k{layer}"])
        np.testing.assert_array_equal(v.cpu().numpy(), g[f"v{layer}"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_decode_append_bit_exact_vs_oracle(cuda, native_lib, dtype):
    case = cases.decode_case("decode_qwen06b_b4")
    st = gh.DecodeState(case, dtype, cuda)
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    rnd = gh.round_for(dtype)
    shape = tuple(st.k_cache.shape)
    kc = np.full(shape, gh.SENTINEL, dtype=np.float32)
    vc = np.full(shape, gh.SENTINEL, dtype=np.float32)
    for b, bt in enumerate(st.tables):
        n = orc.append_only(kc, vc, 0, bt, 0, rnd(case.k_hist[b]), rnd(case.v_hist[b]))
        orc.append_only(kc, vc, 0, bt, n, rnd(case.k_new[b : b + 1]), rnd(case.v_new[b : b + 1]))
    np.testing.assert_array_equal(st.k_cache.float().cpu().numpy(), kc)
    np.testing.assert_array_equal(st.v_cache.float().cpu().numpy(), vc)


def test_append_with_row_ids_and_strided_input(cuda, native_lib):
    """Rows are picked through row_ids from a larger table; the new tokens come
    from a transposed [B, T, H, D] buffer, as the model's k.view().transpose()."""
    rs = np.random.RandomState(5)
    P, H, bs, D = 40, 3, 4, 16
    kc = torch.zeros((2, P, H, bs, D), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    table = rs.permutation(P)[:30].reshape(6, 5).astype(np.int32)
    bt = torch.from_numpy(table).to(cuda)
    row_ids = torch.tensor([4, 1, 3], dtype=torch.int32, device=cuda)
    start = torch.tensor([0, 5, 11], dtype=torch.int32, device=cuda)
    raw = torch.randn(3, 7, H, D).to(torch.bfloat16).to(cuda)  # [B, T, H, D]
    k = raw.transpose(1, 2)
    ops.paged_append(kc, vc, 1, bt, start, k, k * 2, row_ids=row_ids)
    kn = np.zeros((2, P, H, bs, D), np.float32)
    vn = np.zeros_like(kn)
    for b, (r, s0) in enumerate(zip([4, 1, 3], [0, 5, 11])):
        kk = k[b : b + 1].float().cpu().numpy()
        orc.append_only(kn, vn, 1, table[r], s0, kk, kk * 2)
    np.testing.assert_array_equal(kc.float().cpu().numpy(), kn)
    np.testing.assert_array_equal(vc.float().cpu().numpy(), vn)


def test_bad_block_ids_set_the_error_word_without_faulting(cuda, native_lib):
    kc = torch.zeros((1, 8, 2, 4, 8), dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    bt = torch.tensor([[3, 99], [-1, 2]], dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    k = torch.ones((2, 2, 6, 8), dtype=torch.bfloat16, device=cuda)
    ops.paged_append(kc, vc, 0, bt, torch.zeros(2, dtype=torch.int32, device=cuda), k, k, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & nat.BL_DEVERR_BLOCK_ID
    # positions past the table width are flagged too
    err.zero_()
    ops.paged_append(kc, vc, 0, bt, torch.tensor([7, 0], dtype=torch.int32, device=cuda), k[:, :, :2], k[:, :, :2], err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & nat.BL_DEVERR_TABLE
    # in-range writes still landed: block 3 holds row 0's first four tokens
    assert kc[0, 3].float().sum().item() == 2 * 4 * 8


def test_decode_bad_block_id_reports_and_stays_finite(cuda, native_lib):
    case = cases.decode_case("decode_qwen06b_b4")
    st = gh.DecodeState(case, torch.bfloat16, cuda)
    bt = st.bt.clone()
    bt[0, 0] = case.num_blocks + 5
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_decode(st.q, st.k_cache, st.v_cache, 0, bt, st.seq_lens, max(st.seq_lens_list), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & nat.BL_DEVERR_BLOCK_ID


def test_host_side_argument_errors(cuda, native_lib):
    kc = torch.zeros((1, 8, 2, 4, 8), dtype=torch.bfloat16, device=cuda)
    bt = torch.zeros((1, 2), dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError, match="KV-head count cannot change"):
        ops.paged_append(kc, kc.clone(), 0, bt, torch.zeros(1, dtype=torch.int32, device=cuda),
                         torch.zeros((1, 3, 1, 8), dtype=torch.bfloat16, device=cuda),
                         torch.zeros((1, 3, 1, 8), dtype=torch.bfloat16, device=cuda))
    with pytest.raises(IndexError, match="Invalid layer index"):
        ops.paged_gather(kc, kc.clone(), 3, bt, torch.ones(1, dtype=torch.int32, device=cuda), 1)
    with pytest.raises(ValueError, match="int32"):
        ops.paged_gather(kc, kc.clone(), 0, bt.long(), torch.ones(1, dtype=torch.int32, device=cuda), 1)


# --------------------------------------------------------------------------
# decode attention
# --------------------------------------------------------------------------
@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_decode_matches_oracle_and_reference(cuda, native_lib, name, dtype):
    case = cases.decode_case(name)
    g = golden(name)
    st = gh.DecodeState(case, dtype, cuda)
    out = st.decode().float().cpu().numpy()
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    rnd = gh.round_for(dtype)
    kc = st.k_cache.float().cpu().numpy()
    vc = st.v_cache.float().cpu().numpy()
    ref = orc.decode_attention(rnd(case.q), kc, vc, 0, st.tables, st.seq_lens_list)[:, :, 0]
    if dtype == torch.float32:
        np.testing.assert_allclose(out, ref, atol=F32_TOL, rtol=F32_TOL)
        np.testing.assert_allclose(out, g["out_f32"][:, :, 0], atol=F32_TOL, rtol=F32_TOL)
    else:
        assert_close_lowp(out, ref)
        if dtype == torch.bfloat16:
            assert_close_lowp(out, g["out_bf16"][:, :, 0])


def test_decode_uses_the_tensor_core_path_at_qwen_shapes(native_lib):
    assert ops.decode_path(torch.bfloat16, 128, 16, 16, 8) == 1
    assert ops.decode_path(torch.bfloat16, 128, 16, 32, 8) == 1


@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (8, 8), (64, 8)])
def test_decode_large_batch_split_k(cuda, native_lib, hq, hkv):
    """32 rows with lengths U{128..2100} (up to five 512-token chunks) in bf16;
    every row checked against the fp64 oracle on the same stored values."""
    case = cases.make_decode_case(40 + hq, 32, hq, hkv, 128, 16, 8192, 128, 2100, scale=1.0 / np.sqrt(128))
    st = gh.DecodeState(case, torch.bfloat16, cuda)
    out = st.decode().float().cpu().numpy()
    torch.cuda.synchronize()
    assert int(st.err.item()) == 0
    kd, vd = ops.paged_gather(st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
    kd, vd = kd.float().cpu().numpy(), vd.float().cpu().numpy()
    rows_k = [kd[b, :, :n] for b, n in enumerate(st.seq_lens_list)]
    rows_v = [vd[b, :, :n] for b, n in enumerate(st.seq_lens_list)]
    ref = orc.decode_attention_rows(st.q.float().cpu().numpy()[:, :, 0], rows_k, rows_v)
    assert_close_lowp(out, ref)


def test_decode_is_batch_invariant(cuda, native_lib):
    """A row's output is bit-identical alone and inside a batch (the split-K
    layout depends only on the row's own length)."""
    case = cases.make_decode_case(77, 12, 32, 8, 128, 16, 4096, 100, 3000)
    st = gh.DecodeState(case, torch.bfloat16, cuda)
    full = st.decode()
    for b in (0, 5, 11):
        alone = ops.paged_decode(st.q[b : b + 1], st.k_cache, st.v_cache, 0, st.bt[b : b + 1], st.seq_lens[b : b + 1],
                                 st.seq_lens_list[b])
        assert torch.equal(alone, full[b : b + 1])


def test_decode_plan_reuse_across_layers(cuda, native_lib):
    """One plan serves every layer: plan_ready=True gives identical results."""
    case = cases.make_decode_case(3, 9, 16, 8, 128, 16, 2048, 1, 2000)
    st = gh.DecodeState(case, torch.bfloat16, cuda)
    first = st.decode()
    ws = ops.paged_decode_plan(st.k_cache, st.v_cache, st.bt, st.seq_lens, max(st.seq_lens_list), 16)
    again = st.decode(ws=ws, plan_ready=True)
    assert torch.equal(first, again)


# --------------------------------------------------------------------------
# prefill attention
# --------------------------------------------------------------------------
def prefill_state(case: cases.PrefillCase, dtype, device):
    shape = (1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
    kc = torch.full(shape, gh.SENTINEL, dtype=dtype, device=device)
    vc = torch.full(shape, gh.SENTINEL, dtype=dtype, device=device)
    table = case.block_table()
    bt = torch.from_numpy(table.astype(np.int32)).view(1, -1).to(device)
    n = 0
    if case.prefix:
        ops.paged_append(kc, vc, 0, bt, torch.tensor([0], dtype=torch.int32, device=device),
                         gh.to_dev(case.k_prefix, dtype, device), gh.to_dev(case.v_prefix, dtype, device))
        n = case.prefix
    ops.paged_append(kc, vc, 0, bt, torch.tensor([n], dtype=torch.int32, device=device),
                     gh.to_dev(case.k_chunk, dtype, device), gh.to_dev(case.v_chunk, dtype, device))
    return kc, vc, table, bt, case.prefix + case.chunk


@pytest.mark.parametrize("name", list(cases.PREFILL_CASES))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_prefill_matches_oracle_and_reference(cuda, native_lib, name, dtype):
    case = cases.prefill_case(name)
    g = golden(name)
    kc, vc, table, bt, total = prefill_state(case, dtype, cuda)
    q = gh.to_dev(case.q, dtype, cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(q, kc, vc, 0, bt, torch.tensor([total], dtype=torch.int32, device=cuda), err=err)
    out = out.float().cpu().numpy()
    assert int(err.item()) == 0
    rnd = gh.round_for(dtype)
    ref = orc.prefill_attention(rnd(case.q), kc.float().cpu().numpy(), vc.float().cpu().numpy(), 0, table, total)
    if dtype == torch.float32:
        np.testing.assert_allclose(out, ref, atol=F32_TOL, rtol=F32_TOL)
        np.testing.assert_allclose(out, g["out_f32"], atol=F32_TOL, rtol=F32_TOL)
    else:
        assert_close_lowp(out, ref)
        if dtype == torch.bfloat16:
            assert_close_lowp(out, g["out_bf16"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 8), (8, 8), (64, 8)])
def test_packed_chunked_prefill_many_requests(cuda, native_lib, hq, hkv, dtype):
    """Several requests with different prefixes and chunk lengths packed into
    one call (q_offsets), tensor-core path; each row vs the fp64 oracle."""
    rs = np.random.RandomState(hq)
    specs = [(0, 45), (37, 130), (300, 17), (16, 200), (513, 64)]
    bs, D, P = 16, 128, 512
    kc = torch.full((1, P, hkv, bs, D), gh.SENTINEL, dtype=dtype, device=cuda)
    vc = torch.full_like(kc, gh.SENTINEL)
    free = list(rs.permutation(P))
    tables, qs, lens = [], [], []
    for prefix, chunk in specs:
        total = prefix + chunk
        tables.append(np.array([free.pop() for _ in range((total + bs - 1) // bs)], dtype=np.int32))
        lens.append(total)
    bt = torch.from_numpy(gh.padded_tables(tables)).to(cuda)
    for b, (prefix, chunk) in enumerate(specs):
        k = torch.randn(1, hkv, prefix + chunk, D).to(dtype).to(cuda)
        v = torch.randn(1, hkv, prefix + chunk, D).to(dtype).to(cuda)
        ops.paged_append(kc, vc, 0, bt[b : b + 1], torch.tensor([0], dtype=torch.int32, device=cuda), k, v)
        qs.append(torch.randn(1, hq, chunk, D).to(dtype).to(cuda))
    q = torch.cat(qs, dim=2)
    offs = torch.tensor(np.concatenate([[0], np.cumsum([c for _, c in specs])]), dtype=torch.int32, device=cuda)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(q, kc, vc, 0, bt, seq, q_offsets=offs, max_q_len=max(c for _, c in specs))
    out = out.float().cpu().numpy()
    kcn, vcn = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    o = 0
    for b, (prefix, chunk) in enumerate(specs):
        qb = q[:, :, o : o + chunk].float().cpu().numpy()
        ref = orc.prefill_attention(qb, kcn, vcn, 0, tables[b], prefix + chunk)
        assert_close_lowp(out[:, :, o : o + chunk], ref)
        o += chunk


@pytest.mark.parametrize("pad", [2, 8])
def test_packed_prefill_strided_q_and_out_match_contiguous(cuda, native_lib, pad):
    """q and out as views of [1, T, Hq, D + pad] buffers.  pad = 2 gives rows
    that do not start on 16-byte boundaries (the kernel loads q and stores the
    output element-wise); pad = 8 keeps 16-byte rows with non-default strides
    (vector paths).  Either way the arithmetic is the same, so the output must
    equal the contiguous call bit for bit."""
    rs = np.random.RandomState(11)
    specs = [(0, 45), (37, 130), (300, 17), (16, 200), (513, 64)]
    hq, hkv, bs, D, P, dtype = 32, 8, 16, 128, 512, torch.bfloat16
    kc = torch.full((1, P, hkv, bs, D), gh.SENTINEL, dtype=dtype, device=cuda)
    vc = torch.full_like(kc, gh.SENTINEL)
    free = list(rs.permutation(P))
    tables, lens = [], []
    for prefix, chunk in specs:
        total = prefix + chunk
        tables.append(np.array([free.pop() for _ in range((total + bs - 1) // bs)], dtype=np.int32))
        lens.append(total)
    bt = torch.from_numpy(gh.padded_tables(tables)).to(cuda)
    gen = torch.Generator().manual_seed(11)
    for b, (prefix, chunk) in enumerate(specs):
        k = torch.randn(1, hkv, prefix + chunk, D, generator=gen).to(dtype).to(cuda)
        v = torch.randn(1, hkv, prefix + chunk, D, generator=gen).to(dtype).to(cuda)
        ops.paged_append(kc, vc, 0, bt[b : b + 1], torch.tensor([0], dtype=torch.int32, device=cuda), k, v)
    T = sum(c for _, c in specs)
    q = torch.randn(1, T, hq, D, generator=gen).to(dtype).to(cuda).transpose(1, 2)
    offs = torch.tensor(np.concatenate([[0], np.cumsum([c for _, c in specs])]), dtype=torch.int32, device=cuda)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    mq = max(c for _, c in specs)
    want = ops.paged_prefill(q, kc, vc, 0, bt, seq, q_offsets=offs, max_q_len=mq)
    qbuf = torch.zeros(1, T, hq, D + pad, dtype=dtype, device=cuda)
    qbuf[..., :D] = q.transpose(1, 2)
    obuf = torch.full((1, T, hq, D + pad), float("nan"), dtype=dtype, device=cuda)
    got = ops.paged_prefill(qbuf[..., :D].transpose(1, 2), kc, vc, 0, bt, seq, q_offsets=offs, max_q_len=mq,
                            out=obuf[..., :D].transpose(1, 2))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.isnan(obuf[..., D:]).all()  # nothing written past each row


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_stale_nan_slots_never_reach_the_outputs(cuda, native_lib, dtype):
    """The pool starts as NaN everywhere (the reference never clears freed
    blocks, so a reused slot may hold any bit pattern).  Rows end inside their
    last page (and one exactly on a page boundary); prefill and decode read
    those pages in place, and no stale byte may reach an output: P = 0 does
    not cancel a NaN in P V, so stale V slots must never be loaded."""
    rs = np.random.RandomState(7)
    specs = [(0, 45), (37, 130), (300, 17), (16, 200), (513, 64), (100, 28)]
    hq, hkv, bs, D, P = 32, 8, 16, 128, 512
    kc = torch.full((1, P, hkv, bs, D), float("nan"), dtype=dtype, device=cuda)
    vc = torch.full_like(kc, float("nan"))
    free = list(rs.permutation(P))
    tables, qs, lens = [], [], []
    for prefix, chunk in specs:
        total = prefix + chunk
        tables.append(np.array([free.pop() for _ in range((total + bs - 1) // bs)], dtype=np.int32))
        lens.append(total)
    bt = torch.from_numpy(gh.padded_tables(tables)).to(cuda)
    gen = torch.Generator().manual_seed(7)
    for b, (prefix, chunk) in enumerate(specs):
        k = torch.randn(1, hkv, prefix + chunk, D, generator=gen).to(dtype).to(cuda)
        v = torch.randn(1, hkv, prefix + chunk, D, generator=gen).to(dtype).to(cuda)
        ops.paged_append(kc, vc, 0, bt[b : b + 1], torch.tensor([0], dtype=torch.int32, device=cuda), k, v)
        qs.append(torch.randn(1, hq, chunk, D, generator=gen).to(dtype).to(cuda))
    q = torch.cat(qs, dim=2)
    offs = torch.tensor(np.concatenate([[0], np.cumsum([c for _, c in specs])]), dtype=torch.int32, device=cuda)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(q, kc, vc, 0, bt, seq, q_offsets=offs, max_q_len=max(c for _, c in specs), err=err)
    qd = torch.randn(len(specs), hq, 1, D, generator=gen).to(dtype).to(cuda)
    dec = ops.paged_decode(qd, kc, vc, 0, bt, seq, max(lens), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    out, dec = out.float().cpu().numpy(), dec.float().cpu().numpy()
    assert np.isfinite(out).all() and np.isfinite(dec).all()
    kcn, vcn = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    o = 0
    for b, (prefix, chunk) in enumerate(specs):
        qb = q[:, :, o : o + chunk].float().cpu().numpy()
        assert_close_lowp(out[:, :, o : o + chunk], orc.prefill_attention(qb, kcn, vcn, 0, tables[b], prefix + chunk))
        o += chunk
    assert_close_lowp(dec, orc.decode_attention(qd.float().cpu().numpy(), kcn, vcn, 0, tables, lens)[:, :, 0])
