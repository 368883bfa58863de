"""The reference arm of bench.py (``--impl reference``) on host cores: for
every workload kind it prints one JSON line with the contract's keys, the
metric and unit of the GPU arm, ``impl: reference``, a ``cpu_baseline`` that
describes the run and an ``e2e`` object with no host<->device bytes.  Tiny
copies of each workload keep this to seconds; the numbers are not checked."""

from __future__ import annotations

import json
import types

import pytest

import bench

BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}

TINY = {
    # name in WORKLOADS -> overrides that shrink it
    "decode_qwen06b_b64": dict(batch=3, len_lo=20, len_hi=60),
    "decode_qwen8b_long": dict(batch=3, len_lo=20, len_hi=60),
    "decode_qwen8b_long_heads": dict(batch=3, len_lo=20, len_hi=60),
    "prefill_qwen8b": dict(batch=2, prefix_lo=0, prefix_hi=40, chunk_lo=16, chunk_hi=24),
    "append_qwen8b_chunks": dict(batch=2, prefix_lo=0, prefix_hi=40, chunk_lo=16, chunk_hi=24),
    "qkprep_qwen8b_chunks": dict(batch=2, prefix_lo=0, prefix_hi=40, chunk_lo=16, chunk_hi=24),
    "gather_qwen06b_b64": dict(batch=3, len_lo=20, len_hi=60),
}
GPU_METRIC = {
    "decode_qwen06b_b64": ("paged-decode KV read GB/s", "GB/s"),
    "decode_qwen8b_long": ("paged-decode KV read GB/s", "GB/s"),
    "decode_qwen8b_long_heads": ("paged-decode KV read GB/s", "GB/s"),
    "prefill_qwen8b": ("paged chunked-prefill attention TFLOP/s", "TFLOP/s"),
}


@pytest.mark.parametrize("name", sorted(TINY))
def test_reference_arm_prints_the_contract_line(name, monkeypatch, capsys):
    wl = dict(bench.WORKLOADS[name], **TINY[name])
    monkeypatch.setitem(bench.WORKLOADS, name, wl)
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    args = types.SimpleNamespace(steps=1, warmup=3, gpus=1, cpu_seconds=0.0)
    kind = wl.get("kind")
    if kind == "prefill":
        bench.run_reference_prefill(args, name)
    elif kind == "copy":
        bench.run_reference_copy(args, name)
    else:
        bench.run_reference(args, name)
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    res = json.loads(lines[0])
    assert BASE_KEYS <= set(res)
    assert res["impl"] == "reference" and res["n_gpus"] == 1 and res["steps"] == 1 and res["warmup"] == 3
    assert res["value"] > 0 and res["higher_is_better"] is True
    assert res["config"]["workload"] == name
    cpu = res["cpu_baseline"]
    assert cpu["value"] == res["value"] and cpu["unit"] == res["unit"] and cpu["cores"] >= 1
    assert cpu["kind"] in ("port", "reference") and cpu["sample"]
    if wl.get("kind") not in ("prefill", "copy"):
        # the decode arms run the reference's own classes when its installed copy imports
        assert cpu["kind"] == ("reference" if bench.reference_package() is not None else "port")
    assert res["e2e"] == {"value": res["value"], "unit": res["unit"], "h2d_bytes_per_step": 0,
                          "d2h_bytes_per_step": 0}
    if name in GPU_METRIC:
        assert (res["metric"], res["unit"]) == GPU_METRIC[name]


def test_reference_arm_is_silent_on_other_ranks(monkeypatch, capsys):
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    args = types.SimpleNamespace(steps=1, warmup=3, gpus=2, cpu_seconds=0.0)
    bench.run_reference(args, "decode_qwen06b_b64")
    bench.run_reference_prefill(args, "prefill_qwen8b")
    bench.run_reference_copy(args, "gather_qwen06b_b64")
    assert capsys.readouterr().out == ""


def test_reference_chain_computes_what_the_oracle_computes():
    """The CPU baseline's reference chain (the reference's BatchKVCache +
    SDPAAttentionBackend on its PagedKVCache) gives, step after step, the
    oracle's decode attention over the same histories: the baseline times the
    same computation the GPU arm is checked against."""
    ref = bench.reference_package()
    if ref is None:
        pytest.skip("the reference's installed copy (baseline/_ref) is not present")
    import numpy as np

    from oracle import paged_oracle as orc

    wl = dict(bench.WORKLOADS["decode_qwen8b_long"], batch=3)
    lens = [37, 5, 80]
    chain = bench.RefDecodeChain(ref, wl, lens, 3)
    for step in range(2):
        layer = ref.BatchKVCache(chain.views).layer(0)
        out = chain.backend.attend(chain.q, chain.k_new, chain.v_new, layer, chain.group)
        k_rows, v_rows = [], []
        for view in chain.views:
            k, v = view.layer(0).read()
            k_rows.append(k[0].numpy())
            v_rows.append(v[0].numpy())
        assert [k.shape[1] for k in k_rows] == [n + step + 1 for n in lens]
        want = orc.decode_attention_rows(chain.q[:, :, 0].numpy(), k_rows, v_rows)
        np.testing.assert_allclose(out[:, :, 0].numpy(), want, atol=1e-5, rtol=1e-5)
