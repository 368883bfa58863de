"""Parity at the benchmark workloads' full sizes.

The fp64 oracle is too slow to check every row of these workloads, so they
are checked through properties that hold at any size, plus a few whole rows
against the oracle:

  * append -> gather is the identity, bit for bit, over the whole batch
    (64 requests of U{128..4096} tokens in a shuffled 65536-block pool), with
    zeros past each row's length;
  * with V constant per (request, KV head) every attention output equals that
    constant (the softmax weights sum to one), within one bf16 step;
  * with K = 0 every key gets the same weight, so decode returns the mean of V
    over the row's keys and chunked prefill returns, for query row i, the mean
    of V over keys 0 .. prefix + i (the causal mask at full size); stale slots
    past each row's length hold a large sentinel, so a key read past the
    length shows;
  * a row decoded alone equals the same row inside the full batch, bit for bit;
  * a few whole rows (the longest included) against the fp64 oracle, within
    max-abs 2e-2 / mean-abs 2e-3.

Workloads: batched decode at Qwen3-0.6B attention shapes (B 64, lengths
U{128..4096}), long-context decode at Qwen3-8B shapes (B 256, lengths
log-uniform 1k..32k, ~9.6 GB of K/V), and packed chunked prefill at Qwen3-8B
shapes (32 requests, prefix U{0..8192}, chunk U{512..2048}).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from barellm_b200 import ops
from oracle import paged_oracle as orc

pytestmark = pytest.mark.gpu

BS, D = 16, 128
STALE = 64.0  # value of every pool slot no request owns
BF16_MAX, BF16_MEAN = 2e-2, 2e-3
ONE_STEP = 2.0**-7  # one bf16 step, relative


def shuffled_tables(lens: list[int], pool_blocks: int, seed: int) -> list[np.ndarray]:
    perm = np.random.RandomState(seed).permutation(pool_blocks)
    out, at = [], 0
    for n in lens:
        k = -(-n // BS)
        out.append(perm[at : at + k].astype(np.int32))
        at += k
    assert at <= pool_blocks
    return out


def padded(tables: list[np.ndarray], device) -> torch.Tensor:
    bt = np.full((len(tables), max(len(t) for t in tables)), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, : len(t)] = t
    return torch.from_numpy(bt).to(device)


def pool_rows(cache: torch.Tensor, table: np.ndarray, n: int) -> torch.Tensor:
    """``[Hkv, n, D]`` of one request read with torch indexing (the reference's
    read), independent of the gather kernel."""
    pos = torch.arange(n, device=cache.device)
    pages = torch.from_numpy(table).to(cache.device).long()[pos // BS]
    return cache[0, pages, :, pos % BS, :].permute(1, 0, 2)


def mark_stale(cache: torch.Tensor, tables: list[np.ndarray], lens: list[int]) -> None:
    """Slots past each row's length inside its last page get the sentinel."""
    for t, n in zip(tables, lens):
        if n % BS:
            cache[0, int(t[-1]), :, n % BS :, :] = STALE


def assert_constant(out: torch.Tensor, want: torch.Tensor) -> None:
    err = (out.float() - want.float()).abs()
    assert torch.isfinite(out.float()).all()
    bound = ONE_STEP * want.float().abs() + 1e-6
    assert bool((err <= bound).all()), float((err - bound).max())


def assert_close(actual: np.ndarray, expected: np.ndarray) -> None:
    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    assert np.isfinite(actual).all()
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (float(err.max()), float(err.mean()))


# --------------------------------------------------------------------------
# batched decode, Qwen3-0.6B attention shapes
# --------------------------------------------------------------------------
@pytest.fixture(scope="module")
def decode_b64(cuda, native_lib):
    hkv, pool_blocks = 8, 65536
    lens = [int(x) for x in np.random.RandomState(1234).randint(128, 4097, size=64)]
    tables = shuffled_tables(lens, pool_blocks, 99)
    bt = padded(tables, cuda)
    shape = (1, pool_blocks, hkv, BS, D)
    kc = torch.full(shape, STALE, dtype=torch.bfloat16, device=cuda)
    vc = torch.full(shape, STALE, dtype=torch.bfloat16, device=cuda)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    total = sum(lens)
    k = torch.randn((1, hkv, total, D), generator=gen, device=cuda).to(torch.bfloat16)
    v = torch.randn((1, hkv, total, D), generator=gen, device=cuda).to(torch.bfloat16)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_append(kc, vc, 0, bt, torch.zeros(64, dtype=torch.int32, device=cuda), k, v,
                     new_offsets=torch.from_numpy(offs).to(cuda), max_new_tokens=max(lens), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return dict(lens=lens, tables=tables, bt=bt, kc=kc, vc=vc, k=k, v=v, offs=offs, hkv=hkv)


def test_append_gather_roundtrip_full_batch(cuda, decode_b64):
    w = decode_b64
    lens, offs = w["lens"], w["offs"]
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    ko, vo = ops.paged_gather(w["kc"], w["vc"], 0, w["bt"], seq, max(lens))
    for b, n in enumerate(lens):
        assert torch.equal(ko[b, :, :n], w["k"][0, :, offs[b] : offs[b] + n])
        assert torch.equal(vo[b, :, :n], w["v"][0, :, offs[b] : offs[b] + n])
        assert not ko[b, :, n:].any() and not vo[b, :, n:].any()


def test_decode_constant_v_full_batch(cuda, decode_b64):
    w = decode_b64
    hq, hkv, g = 16, w["hkv"], 2
    lens, tables = w["lens"], w["tables"]
    gen = torch.Generator(device=cuda)
    gen.manual_seed(6)
    c = torch.randn((64, hkv), generator=gen, device=cuda).to(torch.bfloat16)
    vc = torch.full_like(w["vc"], STALE)
    for b, t in enumerate(tables):
        vc[0, torch.from_numpy(t).to(cuda).long()] = c[b][:, None, None]
    mark_stale(vc, tables, lens)
    q = (torch.randn((64, hq, D), generator=gen, device=cuda) / math.sqrt(D)).to(torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = ops.paged_decode(q, w["kc"], vc, 0, w["bt"], seq, max(lens))
    want = c.repeat_interleave(g, dim=1)[:, :, None].expand(-1, -1, D)
    assert_constant(out, want)


def test_decode_uniform_keys_average_v_full_batch(cuda, decode_b64):
    w = decode_b64
    hq, hkv, g = 16, w["hkv"], 2
    lens, tables = w["lens"], w["tables"]
    kc = torch.zeros_like(w["kc"])
    gen = torch.Generator(device=cuda)
    gen.manual_seed(7)
    q = torch.randn((64, hq, D), generator=gen, device=cuda).to(torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = ops.paged_decode(q, kc, w["vc"], 0, w["bt"], seq, max(lens)).float()
    for b, n in enumerate(lens):
        mean = pool_rows(w["vc"], tables[b], n).float().mean(dim=1)  # [Hkv, D]
        want = mean.repeat_interleave(g, dim=0)
        assert (out[b] - want).abs().max().item() <= 2e-3 + ONE_STEP * want.abs().max().item()


# --------------------------------------------------------------------------
# long-context decode, Qwen3-8B attention shapes
# --------------------------------------------------------------------------
@pytest.fixture(scope="module")
def decode_long(cuda, native_lib):
    hq, hkv = 32, 8
    x = np.exp(np.random.RandomState(1234).uniform(np.log(1024), np.log(32768), size=256))
    lens = [int(n) for n in np.round(x)]
    pool_blocks = sum(-(-n // BS) for n in lens) + 1024
    tables = shuffled_tables(lens, pool_blocks, 17)
    bt = padded(tables, cuda)
    shape = (1, pool_blocks, hkv, BS, D)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(8)
    kc = torch.empty(shape, dtype=torch.bfloat16, device=cuda)
    vc = torch.empty(shape, dtype=torch.bfloat16, device=cuda)
    kc.normal_(generator=gen)
    vc.normal_(generator=gen)
    mark_stale(kc, tables, lens)
    mark_stale(vc, tables, lens)
    q = torch.randn((256, hq, D), generator=gen, device=cuda).to(torch.bfloat16)
    seq = torch.tensor(lens, dtype=torch.int32, device=cuda)
    return dict(lens=lens, tables=tables, bt=bt, kc=kc, vc=vc, q=q, seq=seq, hq=hq, hkv=hkv)


def test_long_decode_rows_vs_oracle(cuda, decode_long):
    w = decode_long
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.paged_decode(w["q"], w["kc"], w["vc"], 0, w["bt"], w["seq"], max(w["lens"]), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    lens = w["lens"]
    rows = sorted({int(np.argmax(lens)), int(np.argmin(lens)), 100})
    q = w["q"][rows].float().cpu().numpy()
    ks = [pool_rows(w["kc"], w["tables"][b], lens[b]).float().cpu().numpy() for b in rows]
    vs = [pool_rows(w["vc"], w["tables"][b], lens[b]).float().cpu().numpy() for b in rows]
    ref = orc.decode_attention_rows(q, ks, vs)
    assert_close(out[rows].float().cpu().numpy(), ref)


def test_long_decode_rows_are_batch_invariant(cuda, decode_long):
    w = decode_long
    full = ops.paged_decode(w["q"], w["kc"], w["vc"], 0, w["bt"], w["seq"], max(w["lens"]))
    lens = w["lens"]
    for b in sorted({int(np.argmax(lens)), int(np.argmin(lens)), 7, 200}):
        alone = ops.paged_decode(w["q"][b : b + 1], w["kc"], w["vc"], 0, w["bt"][b : b + 1], w["seq"][b : b + 1],
                                 lens[b])
        assert torch.equal(alone, full[b : b + 1])


def test_long_decode_constant_v(cuda, decode_long):
    w = decode_long
    hkv, g = w["hkv"], w["hq"] // w["hkv"]
    gen = torch.Generator(device=cuda)
    gen.manual_seed(9)
    c = torch.randn((256, hkv), generator=gen, device=cuda).to(torch.bfloat16)
    per_block = torch.zeros((w["vc"].shape[1], hkv), dtype=torch.bfloat16, device=cuda)
    for b, t in enumerate(w["tables"]):
        per_block[torch.from_numpy(t).to(cuda).long()] = c[b]
    vc = per_block[None, :, :, None, None].expand_as(w["vc"]).contiguous()
    mark_stale(vc, w["tables"], w["lens"])
    out = ops.paged_decode(w["q"], w["kc"], vc, 0, w["bt"], w["seq"], max(w["lens"]))
    del vc
    want = c.repeat_interleave(g, dim=1)[:, :, None].expand(-1, -1, D)
    assert_constant(out, want)


# --------------------------------------------------------------------------
# packed chunked prefill, Qwen3-8B attention shapes
# --------------------------------------------------------------------------
@pytest.fixture(scope="module")
def prefill_chunks(cuda, native_lib):
    hq, hkv, pool_blocks = 32, 8, 65536
    rs = np.random.RandomState(4321)
    prefix = [int(x) for x in rs.randint(0, 8193, size=32)]
    chunk = [int(x) for x in rs.randint(512, 2049, size=32)]
    totals = [p + c for p, c in zip(prefix, chunk)]
    tables = shuffled_tables(totals, pool_blocks, 23)
    bt = padded(tables, cuda)
    q_offs = torch.tensor(np.concatenate([[0], np.cumsum(chunk)]), dtype=torch.int32, device=cuda)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(10)
    q = torch.randn((1, sum(chunk), hq, D), generator=gen, device=cuda).to(torch.bfloat16).transpose(1, 2)
    return dict(prefix=prefix, chunk=chunk, totals=totals, tables=tables, bt=bt, q_offs=q_offs, q=q, hq=hq,
                hkv=hkv, pool_blocks=pool_blocks)


def fill_prefill_pool(w: dict, cuda, k_fn, v_fn):
    """Pool whose rows hold prefix + chunk tokens with K/V from k_fn / v_fn
    (``[1, Hkv, n, D]`` per request), appended as packed runs."""
    hkv = w["hkv"]
    shape = (1, w["pool_blocks"], hkv, BS, D)
    kc = torch.full(shape, STALE, dtype=torch.bfloat16, device=cuda)
    vc = torch.full(shape, STALE, dtype=torch.bfloat16, device=cuda)
    ks = torch.cat([k_fn(b, n) for b, n in enumerate(w["totals"])], dim=2)
    vs = torch.cat([v_fn(b, n) for b, n in enumerate(w["totals"])], dim=2)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(w["totals"])]), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ops.paged_append(kc, vc, 0, w["bt"], torch.zeros(32, dtype=torch.int32, device=cuda), ks, vs, new_offsets=offs,
                     max_new_tokens=max(w["totals"]), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return kc, vc


def run_prefill(w: dict, kc, vc, cuda) -> torch.Tensor:
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    seq = torch.tensor(w["totals"], dtype=torch.int32, device=cuda)
    out = ops.paged_prefill(w["q"], kc, vc, 0, w["bt"], seq, q_offsets=w["q_offs"], max_q_len=max(w["chunk"]), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out  # [1, Hq, sum C, D]


def test_prefill_rows_vs_oracle_full_workload(cuda, prefill_chunks):
    w = prefill_chunks
    gen = torch.Generator(device=cuda)
    gen.manual_seed(11)
    kc, vc = fill_prefill_pool(
        w, cuda,
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16),
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16))
    out = run_prefill(w, kc, vc, cuda)
    offs = w["q_offs"].cpu().numpy()
    for b in sorted({int(np.argmax(w["totals"])), int(np.argmin(w["totals"])), 5}):
        p, c = w["prefix"][b], w["chunk"][b]
        k = pool_rows(kc, w["tables"][b], p + c).float().cpu().numpy()[None]
        v = pool_rows(vc, w["tables"][b], p + c).float().cpu().numpy()[None]
        qb = w["q"][:, :, offs[b] : offs[b + 1]].float().cpu().numpy()
        ob = out[:, :, offs[b] : offs[b + 1]].float().cpu().numpy()
        # the last 8 query rows attend over all p + c keys (bottom-right mask)
        ref = orc.sdpa(qb[:, :, c - 8 :], orc.repeat_kv(k, 4), orc.repeat_kv(v, 4),
                       attn_mask=orc.causal_mask_bottom_right(8, p + c)[None, None])
        assert_close(ob[:, :, c - 8 :], ref)
        # the first 8 query rows see keys 0 .. p + i only
        ref = orc.sdpa(qb[:, :, :8], orc.repeat_kv(k[:, :, : p + 8], 4), orc.repeat_kv(v[:, :, : p + 8], 4),
                       attn_mask=orc.causal_mask_bottom_right(8, p + 8)[None, None])
        assert_close(ob[:, :, :8], ref)


def test_prefill_repeat_launches_bitwise_identical_full_workload(cuda, prefill_chunks):
    """The MMA issuer queues S_X behind the P V that reads P_X from S_X's own
    TMEM columns without waiting for it (a thread's MMAs run in issue order).
    Were that overwrite ever to overtake the read, outputs would change from
    launch to launch; every launch of the full workload must give the same
    bits."""
    w = prefill_chunks
    gen = torch.Generator(device=cuda)
    gen.manual_seed(14)
    kc, vc = fill_prefill_pool(
        w, cuda,
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16),
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16))
    first = run_prefill(w, kc, vc, cuda).clone()
    assert torch.isfinite(first).all()
    for _ in range(7):
        assert torch.equal(run_prefill(w, kc, vc, cuda), first)


def test_prefill_constant_v_full_workload(cuda, prefill_chunks):
    w = prefill_chunks
    gen = torch.Generator(device=cuda)
    gen.manual_seed(12)
    c = torch.randn((32, w["hkv"]), generator=gen, device=cuda).to(torch.bfloat16)
    kc, vc = fill_prefill_pool(
        w, cuda,
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16),
        lambda b, n: c[b][None, :, None, None].expand(1, w["hkv"], n, D))
    out = run_prefill(w, kc, vc, cuda)
    offs = w["q_offs"].cpu().numpy()
    for b in range(32):
        want = c[b].repeat_interleave(w["hq"] // w["hkv"])[None, :, None, None]
        assert_constant(out[:, :, offs[b] : offs[b + 1]], want.expand(1, -1, w["chunk"][b], D))


def test_prefill_uniform_keys_causal_mean_full_workload(cuda, prefill_chunks):
    """K = 0: query row i of a chunk averages V over keys 0 .. prefix + i."""
    w = prefill_chunks
    gen = torch.Generator(device=cuda)
    gen.manual_seed(13)
    kc, vc = fill_prefill_pool(
        w, cuda,
        lambda b, n: torch.zeros((1, w["hkv"], n, D), dtype=torch.bfloat16, device=cuda),
        lambda b, n: torch.randn((1, w["hkv"], n, D), generator=gen, device=cuda).to(torch.bfloat16))
    out = run_prefill(w, kc, vc, cuda).float()
    offs = w["q_offs"].cpu().numpy()
    g = w["hq"] // w["hkv"]
    for b in range(32):
        p, c = w["prefix"][b], w["chunk"][b]
        v = pool_rows(vc, w["tables"][b], p + c).double()  # [Hkv, p + c, D]
        csum = v.cumsum(dim=1)[:, p:]  # sums over keys 0 .. p + i
        mean = (csum / torch.arange(p + 1, p + c + 1, device=cuda, dtype=torch.float64)[None, :, None]).float()
        want = mean.repeat_interleave(g, dim=0)
        got = out[0, :, offs[b] : offs[b + 1]]
        assert (got - want).abs().max().item() <= 2e-3 + ONE_STEP * want.abs().max().item(), b
