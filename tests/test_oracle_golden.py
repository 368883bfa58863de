"""Pins the CPU oracle to the reference: every oracle function reproduces the
golden vectors that tests/golden/make_golden.py recorded from the reference's
own classes.  Copies must match exactly; fp32 attention within 1e-5."""

from __future__ import annotations

import numpy as np
import pytest

import cases
from oracle import paged_oracle as orc

GOLDEN = cases.__file__.rsplit("/", 1)[0]
SENTINEL = -7.0


def load(name: str):
    return np.load(f"{GOLDEN}/{name}.npz")


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 -> float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def build_decode_pool(case: cases.DecodeCase, round_fn=None):
    """Oracle pool after every request's history and new token are appended."""
    rnd = round_fn or (lambda a: a)
    shape = (1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
    kc = np.full(shape, SENTINEL, dtype=np.float32)
    vc = np.full(shape, SENTINEL, dtype=np.float32)
    tables = case.block_tables()
    lens = []
    for b, bt in enumerate(tables):
        n = orc.append_only(kc, vc, 0, bt, 0, rnd(case.k_hist[b]), rnd(case.v_hist[b]))
        n = orc.append_only(kc, vc, 0, bt, n, rnd(case.k_new[b : b + 1]), rnd(case.v_new[b : b + 1]))
        lens.append(n)
    return kc, vc, tables, lens


def test_storage_sequence_matches_reference():
    g = load("storage_sequence")
    kc = np.full(g["key_cache"].shape, SENTINEL, dtype=np.float32)
    vc = np.full_like(kc, SENTINEL)
    tables = {"A": g["table_A"], "B": g["table_B"]}
    lens = {}
    for i, (rid, layer, start) in enumerate(zip(g["step_rid"], g["step_layer"], g["step_start"])):
        key = g[f"step{i}_key"]
        assert lens.get((str(rid), int(layer)), 0) == int(start)
        # the growth step registers a longer table; earlier steps only used its prefix
        lens[(str(rid), int(layer))] = orc.append_only(kc, vc, int(layer), tables[str(rid)], int(start), key, key + 100)
    np.testing.assert_array_equal(kc, g["key_cache"])
    np.testing.assert_array_equal(vc, g["value_cache"])
    for rid, layer in (("A", 0), ("A", 1), ("B", 0)):
        k, v = orc.read(kc, vc, layer, tables[rid], lens[(rid, layer)])
        np.testing.assert_array_equal(k, g[f"read_{rid}{layer}_k"])
        np.testing.assert_array_equal(v, g[f"read_{rid}{layer}_v"])


def test_batch_read_pad_and_mask_match_reference():
    g = load("batch_read")
    lengths = [int(x) for x in g["lengths"]]
    tables = [row[row >= 0] for row in g["block_tables"]]
    kc = np.full(g["key_cache"].shape, SENTINEL, dtype=np.float32)
    vc = np.full_like(kc, SENTINEL)
    for i, (bt, n) in enumerate(zip(tables, lengths)):
        for layer in range(2):
            orc.append_only(kc, vc, layer, bt, 0, cases.pattern_tensor(i, layer, n, 2, 3, 0.0),
                            cases.pattern_tensor(i, layer, n, 2, 3, 0.5))
    np.testing.assert_array_equal(kc, g["key_cache"])
    for layer in range(2):
        k, v = orc.batch_read_pad(kc, vc, layer, tables, lengths)
        np.testing.assert_array_equal(k, g[f"k{layer}"])
        np.testing.assert_array_equal(v, g[f"v{layer}"])
        np.testing.assert_array_equal(orc.attention_mask(lengths, 1), g[f"mask{layer}"])


@pytest.mark.parametrize("name", list(cases.DECODE_CASES))
def test_decode_oracle_matches_reference(name):
    g = load(name)
    case = cases.decode_case(name)
    assert np.isclose(case.checksum(), float(g["checksum"]), rtol=1e-12), "seeded inputs drifted"
    kc, vc, tables, lens = build_decode_pool(case)
    assert lens == list(g["seq_lens"])
    np.testing.assert_array_equal(cases_tables(tables), g["block_tables"])
    out = orc.decode_attention(case.q, kc, vc, 0, tables, lens)
    np.testing.assert_allclose(out, g["out_f32"], atol=1e-5, rtol=1e-5)
    # the reference's own bf16 CPU run agrees with the fp64 oracle on bf16 inputs
    kc16, vc16, _, _ = build_decode_pool(case, bf16_round)
    out16 = orc.decode_attention(bf16_round(case.q), kc16, vc16, 0, tables, lens)
    err = np.abs(out16 - g["out_bf16"])
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (err.max(), err.mean())


def cases_tables(tables):
    width = max(len(x) for x in tables)
    out = np.full((len(tables), width), -1, dtype=np.int32)
    for i, x in enumerate(tables):
        out[i, : len(x)] = x
    return out


@pytest.mark.parametrize("name", list(cases.PREFILL_CASES))
def test_prefill_oracle_matches_reference(name):
    g = load(name)
    case = cases.prefill_case(name)
    assert np.isclose(case.checksum(), float(g["checksum"]), rtol=1e-12)
    shape = (1, case.num_blocks, case.num_kv_heads, case.block_size, case.head_dim)
    kc = np.full(shape, SENTINEL, dtype=np.float32)
    vc = np.full(shape, SENTINEL, dtype=np.float32)
    bt = case.block_table()
    np.testing.assert_array_equal(bt, g["block_table"])
    n = 0
    if case.prefix:
        n = orc.append_only(kc, vc, 0, bt, 0, case.k_prefix, case.v_prefix)
    n = orc.append_only(kc, vc, 0, bt, n, case.k_chunk, case.v_chunk)
    out = orc.prefill_attention(case.q, kc, vc, 0, bt, n)
    np.testing.assert_allclose(out, g["out_f32"], atol=1e-5, rtol=1e-5)


def test_oracle_rejects_insufficient_blocks():
    kc = np.zeros((1, 4, 2, 2, 3), dtype=np.float32)
    with pytest.raises(ValueError, match="enough allocated"):
        orc.append_only(kc, kc.copy(), 0, np.array([1]), 0, np.ones((1, 2, 3, 3), np.float32),
                        np.ones((1, 2, 3, 3), np.float32))


def test_bottom_right_mask_reduces_to_causal_without_prefix():
    m = orc.causal_mask_bottom_right(5, 5)
    np.testing.assert_array_equal(m, np.tril(np.ones((5, 5), dtype=bool)))
    m = orc.causal_mask_bottom_right(2, 5)
    np.testing.assert_array_equal(m, [[1, 1, 1, 1, 0], [1, 1, 1, 1, 1]])


def test_decode_rows_helper_matches_padded_oracle():
    case = cases.decode_case("decode_tiny_gqa")
    kc, vc, tables, lens = build_decode_pool(case)
    out = orc.decode_attention(case.q, kc, vc, 0, tables, lens)[:, :, 0]
    rows_k = [orc.read(kc, vc, 0, bt, n)[0][0] for bt, n in zip(tables, lens)]
    rows_v = [orc.read(kc, vc, 0, bt, n)[1][0] for bt, n in zip(tables, lens)]
    np.testing.assert_allclose(orc.decode_attention_rows(case.q[:, :, 0], rows_k, rows_v), out, atol=1e-12)


@pytest.mark.parametrize("name", list(cases.QK_PREP_CASES))
def test_qk_norm_rope_oracle_matches_reference(name):
    g = load(name)
    case = cases.qk_prep_case(name)
    assert np.isclose(case.checksum(), float(g["checksum"]), rtol=1e-12), "seeded inputs drifted"
    # float32: the float64 restatement on the reference's own cos/sin tables
    q32 = orc.qk_norm_rope(case.q, g["q_weight_f32"], g["cos_f32"], g["sin_f32"], case.eps)
    k32 = orc.qk_norm_rope(case.k, g["k_weight_f32"], g["cos_f32"], g["sin_f32"], case.eps)
    np.testing.assert_allclose(q32, g["q_out_f32"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(k32, g["k_out_f32"], atol=1e-5, rtol=1e-5)
    # bf16: the same steps with each tensor op's rounding; the mean square's
    # summation order may move a rare normalised element by one bf16 step,
    # which RoPE carries as one step of x * cos or rotate_half(x) * sin
    for src, key in ((case.q, "q"), (case.k, "k")):
        rnd = lambda a: bf16_round(a.astype(np.float32))  # noqa: E731
        out = orc.qk_norm_rope(bf16_round(src), g[f"{key}_weight_bf16"], g["cos_bf16"], g["sin_bf16"], case.eps,
                               round_fn=rnd)
        ref = g[f"{key}_out_bf16"]
        assert_bf16_rope_close(out, ref, orc.rms_norm(bf16_round(src), g[f"{key}_weight_bf16"], case.eps, rnd),
                               g["cos_bf16"], g["sin_bf16"])


def assert_bf16_rope_close(out, ref, normed, cos, sin):
    """All but a rare element equal; the rest within one bf16 step of the RoPE
    products they came from."""
    exact = np.mean(out == ref)
    step = 2.0 ** -7 * (np.abs(normed * cos) + np.abs(orc.rotate_half(normed) * sin) + np.abs(ref)) + 1e-30
    assert exact >= 0.99 and np.all(np.abs(out - ref) <= step), (exact, np.max(np.abs(out - ref)))
