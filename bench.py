#!/usr/bin/env python
"""Paged-decode benchmark: append + split-K decode attention, read in place.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]   (default decode_qwen8b_long; see WORKLOADS:
                    decode_qwen06b_b64, decode_qwen8b_long_heads, prefill_qwen8b,
                    append_qwen8b_chunks, qkprep_qwen8b_chunks, gather_qwen06b_b64,
                    e2e_qwen06b, refengine_qwen06b)

One step is one pass of the hot path over one batch: the one-token K/V append
of every request, the split-K plan, the decode attention kernel and the
split-K reduce (4 kernels, replayed as one CUDA graph, each starting early
through programmatic dependent launch).  Default workload: long-context
batched paged decode at Qwen3-8B attention shapes (32 q / 8 kv heads,
head_dim 128, block_size 16), bf16, one batch of 256 requests with history
lengths log-uniform in 1k..32k, each GPU's blocks shuffled across a ~150 GB
pool, Q/K/V ~ N(0,1).  Multi-GPU runs one process per GPU (torchrun), each
with its own BlockPool shard: the 256 requests are placed whole onto the GPUs
(longest first onto the least-loaded shard, barellm_b200.placement), so the
total work is fixed as N grows (strong scaling) and there is no collective on
the data path.

Metric: algorithmic K/V bytes read per second (sum over GPUs), bytes =
sum_b len_b * Hkv * D * 2 (K+V) * 2 B  +  q and output bytes.

``--impl reference`` times the reference's own decode chain (BatchKVCache
over its PagedKVCache: per-row append, dense gather + pad to the batch's
longest row, repeat_interleave, padding mask, SDPA through
SDPAAttentionBackend.attend) from the installed reference package on this
host's cores, on a bounded sample of the same workload; without the installed
package it falls back to the float32 numpy restatement of that chain.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from barellm_b200.placement import place_requests  # noqa: E402

WORKLOADS = {
    # batched paged decode at Qwen3-0.6B attention shapes, 64 requests per GPU
    # (weak scaling: every GPU decodes a batch with the same 64 lengths)
    "decode_qwen06b_b64": dict(hq=16, hkv=8, d=128, bs=16, batch=64, len_lo=128, len_hi=4096, log_uniform=False,
                               pool_blocks=65536, shard_batch=False, scale=1 / math.sqrt(128)),
    # long-context decode at Qwen3-8B attention shapes (the headline workload):
    # one batch of 256 requests placed across the GPUs, lengths log-uniform
    # 1k..32k, ~150 GB KV pool per GPU
    "decode_qwen8b_long": dict(hq=32, hkv=8, d=128, bs=16, batch=256, len_lo=1024, len_hi=32768, log_uniform=True,
                               pool_bytes=150e9, shard_batch=True, scale=1.0),
    # the same long-context batch with its KV heads (not its requests) split
    # across the GPUs: every GPU reads 1/N of every request's K/V and the
    # per-head outputs are all-gathered by the decode kernels' own stores
    "decode_qwen8b_long_heads": dict(kind="heads", hq=32, hkv=8, d=128, bs=16, batch=256, len_lo=1024,
                                     len_hi=32768, log_uniform=True, shard_batch=False, scale=1.0,
                                     scaling="strong"),
    # paged chunked prefill at Qwen3-8B attention shapes: 32 requests, each a
    # paged prefix of U{0..8192} tokens plus a new chunk of U{512..2048}
    "prefill_qwen8b": dict(kind="prefill", hq=32, hkv=8, d=128, bs=16, batch=32, prefix_lo=0, prefix_hi=8192,
                           chunk_lo=512, chunk_hi=2048, pool_blocks=65536, shard_batch=True),
    # K/V copies on their own (HBM-bound): the chunk append of the prefill
    # workload (packed ragged chunks into fresh pages after each prefix), the
    # same chunks through the fused QK-RMSNorm + RoPE + append kernel, and the
    # dense zero-padded read of the decode workload's pages
    "append_qwen8b_chunks": dict(kind="copy", op="append", hq=32, hkv=8, d=128, bs=16, batch=32, prefix_lo=0,
                                 prefix_hi=8192, chunk_lo=512, chunk_hi=2048, pool_blocks=65536, shard_batch=True),
    "qkprep_qwen8b_chunks": dict(kind="copy", op="qkprep", hq=32, hkv=8, d=128, bs=16, batch=32, prefix_lo=0,
                                 prefix_hi=8192, chunk_lo=512, chunk_hi=2048, pool_blocks=65536, shard_batch=True),
    "gather_qwen06b_b64": dict(kind="copy", op="gather", hq=16, hkv=8, d=128, bs=16, batch=64, len_lo=128,
                               len_hi=4096, log_uniform=False, pool_blocks=65536, shard_batch=False,
                               scale=1 / math.sqrt(128)),
    # end to end: Qwen3-0.6B architecture, random bf16 weights, 128 requests of
    # random token ids (prompts U{64..2048}) placed across the GPUs, greedy
    # decoding of 256 new tokens through the paged engine
    "e2e_qwen06b": dict(kind="e2e", batch=128, prompt_lo=64, prompt_hi=2048, new_tokens=256, shard_batch=True),
    # the reference's own Engine + Scheduler + KVCacheManager + BlockPool and
    # its Qwen3 model (Qwen3-0.6B architecture, random bf16 weights) on one
    # GPU, run twice: on its own "sdpa" backend with its PagedKVCache, and
    # with this package's PagedKVCache and CUDA backend swapped in
    "refengine_qwen06b": dict(kind="refengine", batch=32, prompt_lo=64, prompt_hi=2048, new_tokens=64,
                              max_batch=32),
}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks(key: str = "hbm_gbs") -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())[key]), "measured"
    return PEAKS_FALLBACK[key], "fallback"


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def request_lengths(wl: dict, seed: int) -> np.ndarray:
    rs = np.random.RandomState(seed)
    if wl["log_uniform"]:
        x = np.exp(rs.uniform(np.log(wl["len_lo"]), np.log(wl["len_hi"]), size=wl["batch"]))
        return np.round(x).astype(np.int64)
    return rs.randint(wl["len_lo"], wl["len_hi"] + 1, size=wl["batch"]).astype(np.int64)


class DecodeWorkload:
    """Device-resident state of one GPU's share of the workload."""

    def __init__(self, wl: dict, rank: int, world: int, device: torch.device, seed: int = 1234):
        from barellm_b200 import ops

        self.wl = wl
        self.device = device
        if wl["shard_batch"]:
            # strong scaling: one global batch, whole requests placed on the GPUs
            all_lens = request_lengths(wl, seed)
            self.request_ids = place_requests(all_lens, world)[rank]
            lens = all_lens[self.request_ids]
        else:
            # weak scaling: every GPU decodes a batch with the same lengths
            lens = request_lengths(wl, seed)
            self.request_ids = list(range(len(lens)))
        seed_r = seed + 7919 * (rank + 1)
        self.lens = [int(x) for x in lens]
        b = len(self.lens)
        self.batch = b
        hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
        if "pool_blocks" in wl:
            pool_blocks = wl["pool_blocks"]
        else:
            pool_blocks = int(wl["pool_bytes"] // (hkv * bs * d * 2 * 2))
        self.pool_blocks = pool_blocks
        rs = np.random.RandomState(seed_r)
        free = list(rs.permutation(pool_blocks))
        need = [-(-(n + 1) // bs) for n in self.lens]
        tables = [[int(free.pop()) for _ in range(k)] for k in need]
        width = max(need)
        bt = np.full((b, width), -1, dtype=np.int32)
        for i, t in enumerate(tables):
            bt[i, : len(t)] = t
        self.tables_np = tables
        self.bt = torch.from_numpy(bt).to(device)
        shape = (1, pool_blocks, hkv, bs, d)
        self.k_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        self.v_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed_r)
        sc = wl["scale"]
        # history: packed ragged appends, a few hundred MB at a time
        starts_all = torch.zeros(b, dtype=torch.int32, device=device)
        lo = 0
        while lo < b:
            hi, tok = lo, 0
            while hi < b and (tok + self.lens[hi]) * hkv * d * 2 <= (1 << 30):
                tok += self.lens[hi]
                hi += 1
            hi = max(hi, lo + 1)
            n = sum(self.lens[lo:hi])
            kh = (torch.randn((1, hkv, n, d), generator=gen, device=device) * sc).to(torch.bfloat16)
            vh = (torch.randn((1, hkv, n, d), generator=gen, device=device) * sc).to(torch.bfloat16)
            offs = torch.tensor(np.concatenate([[0], np.cumsum(self.lens[lo:hi])]), dtype=torch.int32, device=device)
            ops.paged_append(self.k_cache, self.v_cache, 0, self.bt[lo:hi], starts_all[lo:hi], kh, vh,
                             new_offsets=offs, max_new_tokens=max(self.lens[lo:hi]))
            del kh, vh
            lo = hi
        self.q = (torch.randn((b, hq, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.k_new = (torch.randn((b, hkv, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.v_new = (torch.randn((b, hkv, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.starts = torch.tensor(self.lens, dtype=torch.int32, device=device)
        self.seq_lens_host = [n + 1 for n in self.lens]
        self.seq_lens = torch.tensor(self.seq_lens_host, dtype=torch.int32, device=device)
        self.max_seq = max(self.seq_lens_host)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.out = torch.empty((b, hq, d), dtype=torch.bfloat16, device=device)
        self.ws = ops.workspace(device, ops.decode_workspace_bytes(b, hq, d, bs, self.max_seq))
        torch.cuda.synchronize(device)

    def decode_bytes(self, seq_lens: list[int] | None = None) -> int:
        wl = self.wl
        lens = self.seq_lens_host if seq_lens is None else seq_lens
        kv = sum(lens) * wl["hkv"] * wl["d"] * 2 * 2
        qo = 2 * len(lens) * wl["hq"] * wl["d"] * 2
        return kv + qo

    def step(self) -> None:
        """append -> plan -> attention -> reduce (4 kernel launches; plan,
        attention and reduce start early through programmatic dependent launch)."""
        from barellm_b200 import ops

        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, self.starts, self.k_new, self.v_new, err=self.err)
        ops.paged_decode_plan(self.k_cache, self.v_cache, self.bt, self.seq_lens, self.max_seq, self.wl["hq"],
                              ws=self.ws, err=self.err)
        self.attention()
        ops.paged_decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, self.max_seq, out=self.out,
                         ws=self.ws, plan_ready=True, err=self.err, stage="reduce")

    def attention(self) -> None:
        from barellm_b200 import ops

        ops.paged_decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, self.max_seq, out=self.out,
                         ws=self.ws, plan_ready=True, err=self.err, stage="attention")


# ---------------------------------------------------------------------------
# clocks (NVML, sampled on a thread during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "sw_power_cap": 0x4,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[tuple[int, int, int]] = []
        self.period = period_s
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[device_index]) if vis else device_index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def sample(self):
        if not self.ok:
            return
        n = self.nvml
        try:
            sm = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
            get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or n.nvmlDeviceGetCurrentClocksThrottleReasons
            reasons = get(self.h)
            util = n.nvmlDeviceGetUtilizationRates(self.h).gpu
            self.samples.append((sm, reasons, util))
        except Exception:  # noqa: BLE001
            pass

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()
        self.sample()

    def summary(self) -> dict:
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        loaded = [s for s in self.samples if s[2] > 0] or self.samples
        reasons = sorted({k for _, r, _ in self.samples for k, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# distributed helpers
# ---------------------------------------------------------------------------
def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def allreduce(x: float, op: str, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int, device) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier(device_ids=[device.index])


# ---------------------------------------------------------------------------
# measurements
# ---------------------------------------------------------------------------
def time_steps(fn, steps: int, device) -> float:
    """ms for `steps` calls of fn, CUDA events on the current stream."""
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize(device)
    return s.elapsed_time(e)


def traffic_from_profile(kernel: str, workload: str, algorithmic_bytes: float | None = None
                         ) -> tuple[float | None, str | None]:
    """DRAM bytes per launch of ``kernel`` from its committed ncu summary.  A
    summary captured on a smaller case of the workload (the full one is too
    large to capture) gives traffic / algorithmic bytes, applied to this
    launch's algorithmic bytes."""
    p = ROOT / "profiles" / f"{kernel}.{workload}.json"
    if p.exists():
        d = json.loads(p.read_text())
        if d.get("traffic_ratio") is not None and algorithmic_bytes is not None:
            return round(d["traffic_ratio"] * algorithmic_bytes), d.get("note")
        return d.get("dram_bytes_per_launch"), d.get("note")
    return None, None


def e2e_measure(wl: dict, work: DecodeWorkload, steps: int, warmup: int, device) -> dict:
    """The same metric through the public API (PagedKVCache + BatchKVCache +
    CudaPagedAttentionBackend.attend) with host-resident inputs: each step
    copies q / k / v from pinned host memory (one copy of a packed buffer),
    appends + attends, and copies the output back."""
    from barellm_b200 import BatchKVCache, BlockPool, CudaPagedAttentionBackend, KVCacheManager, PagedKVCache, ops

    hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
    b = work.batch
    total_steps = 2 * steps + warmup  # the timed steps, the warm-up and the host-issue timing
    need = sum(-(-(n + total_steps + 1) // bs) for n in work.lens)
    pool_blocks = min(work.pool_blocks, int(need * 1.05) + 64)
    kv = PagedKVCache(1, pool_blocks, hkv, bs, d, dtype=torch.bfloat16, device=device, max_requests=b)
    pool = BlockPool(pool_blocks)
    pool.free_ids = [int(x) for x in np.random.RandomState(99).permutation(pool_blocks)]
    mgr = KVCacheManager(bs, pool, kv)

    class Req:
        def __init__(self, i, n):
            self.id = f"req{i}"
            self.seq_len = n

    reqs = [Req(i, n + total_steps + 1) for i, n in enumerate(work.lens)]
    for r in reqs:
        assert mgr.allocate_request(r)
    views = [mgr.get_cache(r) for r in reqs]
    # history: copy each row's pages from the device-resident workload
    for i, vw in enumerate(views):
        n = work.lens[i]
        kd, vd = ops.paged_gather(work.k_cache, work.v_cache, 0, work.bt[i : i + 1],
                                  torch.tensor([n], dtype=torch.int32, device=device), n)
        vw.layer(0).append_only(kd, vd)
        del kd, vd
    backend = CudaPagedAttentionBackend()
    # the step's q, k and v side by side in one pinned host buffer, so one
    # host-to-device copy brings them all; the device tensors are views
    nq, nk = work.q.numel(), work.k_new.numel()
    in_h = torch.cat([work.q.reshape(-1), work.k_new.reshape(-1), work.v_new.reshape(-1)]).cpu().pin_memory()
    in_d = torch.empty_like(in_h, device=device)
    q_d = in_d[:nq].view(work.q.shape)
    k_d = in_d[nq : nq + nk].view(work.k_new.shape)
    v_d = in_d[nq + nk :].view(work.v_new.shape)
    out_h = torch.empty((b, hq, 1, d), dtype=torch.bfloat16).pin_memory()
    seq_hist: list[list[int]] = []

    def one():
        in_d.copy_(in_h, non_blocking=True)
        layer = BatchKVCache(views).layer(0)
        out = backend.attend(q_d, k_d, v_d, layer, hq // hkv)
        seq_hist.append(layer.starts().tolist())
        out_h.copy_(out, non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize(device)
    seq_hist.clear()
    ms = time_steps(one, steps, device)
    kv.check_device_errors()
    nbytes = sum(work.decode_bytes(s) for s in seq_hist)
    h2d = in_h.numel() * 2 + 3 * b * 4
    d2h = out_h.numel() * 2
    # the host's own time to issue a step (outside the timed region): when it
    # is close to the device step, the public-API step is host-bound
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    host_ms = (time.perf_counter() - t0) * 1e3 / steps
    torch.cuda.synchronize(device)
    return {"ms": ms, "bytes": nbytes, "h2d": h2d, "d2h": d2h, "host_issue_ms": host_ms}


def cpu_sample_state(wl: dict, lens: list[int], seed: int = 5):
    """Host float32 pages for a few requests (the first rows of the workload,
    same lengths), in a compact shuffled pool; Q/K/V from a seeded numpy RNG."""
    from oracle import paged_oracle as orc

    hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
    rs = np.random.RandomState(seed)
    need = [-(-(n + 1) // bs) for n in lens]
    perm = list(rs.permutation(sum(need)))
    tables = [np.array([perm.pop() for _ in range(k)]) for k in need]
    shape = (1, sum(need), hkv, bs, d)
    kc = np.zeros(shape, dtype=np.float32)
    vc = np.zeros(shape, dtype=np.float32)
    sc = np.float32(wl["scale"])
    for t, n in zip(tables, lens):
        k = rs.standard_normal((1, hkv, n, d)).astype(np.float32) * sc
        v = rs.standard_normal((1, hkv, n, d)).astype(np.float32) * sc
        orc.append_only(kc, vc, 0, t, 0, k, v)
    b = len(lens)
    q = rs.standard_normal((b, hq, 1, d)).astype(np.float32) * sc
    kn = rs.standard_normal((b, hkv, 1, d)).astype(np.float32) * sc
    vn = rs.standard_normal((b, hkv, 1, d)).astype(np.float32) * sc
    return kc, vc, tables, np.array(lens), q, kn, vn


def cpu_sample_lens(lens: list[int], max_rows: int, max_tokens: int) -> list[int]:
    """The first rows of the workload, up to max_rows rows / max_tokens tokens (>= 1 row)."""
    out: list[int] = []
    for n in lens[:max_rows]:
        if out and sum(out) + n > max_tokens:
            break
        out.append(n)
    return out


def cpu_bytes(wl: dict, lens) -> int:
    """Same algorithmic byte count as the GPU arm (bf16 elements)."""
    return sum(n + 1 for n in lens) * wl["hkv"] * wl["d"] * 2 * 2 + 2 * len(lens) * wl["hq"] * wl["d"] * 2


def cpu_run(wl: dict, lens: list[int], seconds: float, min_runs: int, threads: int):
    """Times the reference chain on host cores; returns (GB/s, runs, sec/run)."""
    from oracle import paged_oracle as orc

    kc, vc, tables, lens_a, q, kn, vn = cpu_sample_state(wl, lens)
    nbytes = cpu_bytes(wl, lens)
    with ThreadPoolExecutor(threads) as ex:
        orc.decode_step_cpu(kc, vc, 0, tables, lens_a, q, kn, vn, executor=ex)  # warm-up
        t0 = time.perf_counter()
        runs = 0
        while runs < min_runs or time.perf_counter() - t0 < seconds:
            orc.decode_step_cpu(kc, vc, 0, tables, lens_a, q, kn, vn, executor=ex)
            runs += 1
        el = time.perf_counter() - t0
    return nbytes * runs / el / 1e9, runs, el / runs


# ---------------------------------------------------------------------------
# the reference's own CPU decode chain (installed copy of the reference)
# ---------------------------------------------------------------------------
def reference_package():
    """The reference's modules from its installed copy (baseline/_ref), or None."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "barellm" / "engine" / "batched_kv_cache.py").exists():
        return None
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    try:
        from barellm.attention.backend import SDPAAttentionBackend
        from barellm.engine.batched_kv_cache import BatchKVCache
        from barellm.engine.block_pool import BlockPool
        from barellm.engine.kv_cache_manager import KVCacheManager
        from barellm.engine.paged_kv_cache import PagedKVCache
    except ImportError:
        return None
    import types

    return types.SimpleNamespace(SDPAAttentionBackend=SDPAAttentionBackend, BatchKVCache=BatchKVCache,
                                 BlockPool=BlockPool, KVCacheManager=KVCacheManager, PagedKVCache=PagedKVCache)


class RefDecodeChain:
    """One layer of the reference's batched decode on host cores, float32 (its
    CPU dtype): ``BatchKVCache(views).layer(0)`` and
    ``SDPAAttentionBackend().attend(q, k_new, v_new, layer, group)`` -- the
    calls Engine._decode -> GroupedQueryAttention.forward make per layer
    (src/barellm/engine/engine.py:458-488, src/barellm/models/attention.py:171-178):
    per-row append_only, dense read + zero pad to the batch's longest row,
    repeat_interleave, padding mask, SDPA.  Every step appends one more token
    per row, as decoding does.  Blocks come from the reference's BlockPool
    (free list shuffled by the seed) through its KVCacheManager."""

    def __init__(self, ref, wl: dict, lens: list[int], max_steps: int, seed: int = 5) -> None:
        hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
        self.wl, self.ref, self.group = wl, ref, hq // hkv
        gen = torch.Generator().manual_seed(seed)
        total = [n + max_steps + 1 for n in lens]
        blocks = sum(-(-t // bs) for t in total)
        self.kv = ref.PagedKVCache(num_layers=1, max_blocks=blocks, num_kv_heads=hkv, block_size=bs, head_dim=d,
                                   dtype=torch.float32, device="cpu")
        pool = ref.BlockPool(blocks)
        pool.free_ids = [int(x) for x in np.random.RandomState(seed).permutation(blocks)]
        mgr = ref.KVCacheManager(bs, pool, self.kv)

        class _Req:
            def __init__(self, rid: str, n: int) -> None:
                self.id, self.seq_len = rid, n

        reqs = [_Req(f"r{i}", t) for i, t in enumerate(total)]
        for r in reqs:
            if not mgr.allocate_request(r):
                raise RuntimeError("reference block pool too small")
        self.views = [mgr.get_cache(r) for r in reqs]
        sc = wl["scale"]
        for view, n in zip(self.views, lens):
            k = torch.randn((1, hkv, n, d), generator=gen) * sc
            v = torch.randn((1, hkv, n, d), generator=gen) * sc
            view.layer(0).append_only(k, v)
        b = len(lens)
        self.q = torch.randn((b, hq, 1, d), generator=gen) * sc
        self.k_new = torch.randn((b, hkv, 1, d), generator=gen) * sc
        self.v_new = torch.randn((b, hkv, 1, d), generator=gen) * sc
        self.backend = ref.SDPAAttentionBackend()

    def step(self) -> int:
        """One decode step; returns its algorithmic bytes (bf16 element count,
        the same accounting as the GPU arm)."""
        layer = self.ref.BatchKVCache(self.views).layer(0)
        self.backend.attend(self.q, self.k_new, self.v_new, layer, self.group)
        return cpu_bytes(self.wl, [v.layer(0).seq_len - 1 for v in self.views])


def ref_sample_rows(ref, wl: dict, lens: list[int], step_budget_s: float, max_rows: int = 16,
                    max_padded_tokens: int = 65536) -> list[int]:
    """The first rows of the workload (at least one) whose reference decode
    step should take about ``step_budget_s``: one row is timed, and a sample
    of n rows costs about n x (its longest row) as much per padded token (the
    reference pads every row to the batch's longest)."""
    probe = RefDecodeChain(ref, wl, lens[:1], 2)
    probe.step()
    t0 = time.perf_counter()
    probe.step()
    per_padded = (time.perf_counter() - t0) / max(lens[0], 1)
    del probe
    n = 1
    while n < min(max_rows, len(lens)):
        m = n + 1
        padded = m * max(lens[:m])
        if padded > max_padded_tokens or padded * per_padded > step_budget_s:
            break
        n = m
    return lens[:n]


def ref_cpu_run(ref, wl: dict, lens: list[int], seconds: float, min_runs: int, threads: int):
    """Times the reference's own decode chain; returns (GB/s, runs, sec/run)."""
    torch.set_num_threads(threads)
    max_runs = max(min_runs, 1) + 2000  # the pool holds this many appended tokens per row
    chain = RefDecodeChain(ref, wl, lens, max_runs)
    with torch.inference_mode():
        chain.step()  # warm-up
        t0 = time.perf_counter()
        runs, nbytes = 0, 0
        while runs < min_runs or time.perf_counter() - t0 < seconds:
            nbytes += chain.step()
            runs += 1
            if runs + 1 >= max_runs:
                break
        el = time.perf_counter() - t0
    return nbytes / el / 1e9, runs, el / runs


def decode_oracle_check(work, out: torch.Tensor, n_rows: int = 3) -> dict:
    """Checks rows of a decode output against the float64 oracle: the
    shortest, the longest and a middle row of this GPU's batch, their K/V read
    back from the pool (bf16 element values).  Raises on a mismatch beyond the
    bf16 bars (max-abs 2e-2, mean-abs 2e-3)."""
    from barellm_b200 import ops
    from oracle import paged_oracle as orc

    lens = work.seq_lens_host
    order = sorted(range(len(lens)), key=lambda i: lens[i])
    rows = sorted({order[0], order[-1], order[len(order) // 2]})[:n_rows]
    k_rows, v_rows = [], []
    for i in rows:
        n = lens[i]
        kd, vd = ops.paged_gather(work.k_cache, work.v_cache, 0, work.bt[i : i + 1],
                                  torch.tensor([n], dtype=torch.int32, device=work.device), n)
        k_rows.append(kd[0].float().cpu().numpy())
        v_rows.append(vd[0].float().cpu().numpy())
        del kd, vd
    q = work.q[rows, :, 0].float().cpu().numpy()
    want = orc.decode_attention_rows(q, k_rows, v_rows)
    got = out[rows].float().cpu().numpy()
    err = np.abs(got - want)
    res = {"rows": [int(r) for r in rows], "row_lengths": [int(lens[r]) for r in rows],
           "max_abs": float(err.max()), "mean_abs": float(err.mean()), "bars": "max-abs 2e-2, mean-abs 2e-3"}
    if not (np.isfinite(got).all() and err.max() <= 2e-2 and err.mean() <= 2e-3):
        raise RuntimeError(f"decode output differs from the oracle: {res}")
    return res


def gather_floats(vals: list[float], world: int, device) -> list[list[float]]:
    """Every rank's values (all ranks take part), outside any timed region."""
    if world == 1:
        return [list(vals)]
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device=device)
    out = torch.empty((world, len(vals)), dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(out, t)
    return out.tolist()


def cpu_baselines(wl: dict, lens: list[int], batch: int, seconds: float) -> tuple[dict, dict]:
    """The N=1 rank-0 CPU baselines: the reference's own chain (when its
    installed copy imports) and the numpy restatement of it."""
    threads = os.cpu_count() or 1
    ref = reference_package()
    primary = None
    if ref is not None:
        rlens = ref_sample_rows(ref, wl, lens, step_budget_s=2.0)
        gbs, runs, per = ref_cpu_run(ref, wl, rlens, seconds=seconds, min_runs=1, threads=threads)
        primary = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "reference",
                   "sample": f"{len(rlens)} of {batch} requests ({sum(rlens)} cached tokens, padded to "
                             f"{max(rlens)}), {runs} decode steps of {per:.3f} s: the reference's "
                             "BatchKVCache + SDPAAttentionBackend.attend on its PagedKVCache, float32, "
                             f"torch.set_num_threads({threads})"}
    plens = cpu_sample_lens(lens, 8, 20000)
    gbs, runs, per = cpu_run(wl, plens, seconds=seconds / 2 if primary else seconds, min_runs=1, threads=threads)
    port = {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{len(plens)} of {batch} requests ({sum(plens)} cached tokens), {runs} runs of {per:.3f} s, "
                      "float32 numpy restatement of the reference decode chain, threaded over rows (each group of "
                      "rows padded to its own longest)"}
    return (primary or port), (port if primary else None)


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def run_ours(args, wl_name: str) -> None:
    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    wl = WORKLOADS[wl_name]
    work = DecodeWorkload(wl, rank, world, device)
    steps, warmup = args.steps, args.warmup

    # one step as a CUDA graph (4 launches)
    work.step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            work.step()
    torch.cuda.current_stream(device).wait_stream(stream)
    sampler = ClockSampler(local)
    barrier(world, device)
    with sampler:
        # warm-up right before the timed region, so the GPU never idles
        # (and drops its clocks) between the two
        for _ in range(warmup):
            graph.replay()
        ms = time_steps(graph.replay, steps, device)
    barrier(world, device)
    if int(work.err.item()):
        raise RuntimeError(f"device error word {int(work.err.item())}")
    ms_max = allreduce(ms, "max", world, device)
    bytes_step = allreduce(float(work.decode_bytes()), "sum", world, device)
    value = bytes_step * steps / (ms_max / 1e3) / 1e9
    per_gpu = gather_floats([float(work.decode_bytes()), ms / steps, float(work.batch)], world, device)

    # the timed graph's output, checked against the oracle (not timed; every
    # replay appends the same token at the same position, so the output is
    # that of one step)
    oracle_check = decode_oracle_check(work, work.out)

    # dominant kernel alone: the decode attention kernel, eager launches
    for _ in range(3):
        work.attention()
    att_ms = time_steps(work.attention, max(steps, 20), device) / max(steps, 20)
    hbm_peak, peak_src = load_peaks()
    att_bytes = work.decode_bytes()
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    traffic, traffic_note = traffic_from_profile("decode_tc_kernel", wl_name, att_bytes)
    del graph

    # end to end through the public API with host buffers
    work_lens = list(work.lens)
    e2e = e2e_measure(wl, work, steps, warmup, device)
    e2e_ms = allreduce(e2e["ms"], "max", world, device)
    e2e_bytes = allreduce(float(e2e["bytes"]), "sum", world, device)
    e2e_value = e2e_bytes / (e2e_ms / 1e3) / 1e9

    cpu, cpu_port = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, cpu_port = cpu_baselines(wl, work_lens, work.batch, args.cpu_seconds)

    if rank == 0:
        kv_bytes = [int(r[0]) for r in per_gpu]
        res = {
            "metric": "paged-decode KV read GB/s",
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": ms_max / steps,
            "higher_is_better": True,
            "scaling": "strong" if wl["shard_batch"] else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": wl_name,
                "model_shapes": f"{wl['hq']}q/{wl['hkv']}kv heads, head_dim {wl['d']}, block_size {wl['bs']}",
                "requests_per_gpu": work.batch if not wl["shard_batch"] else None,
                "requests_total": wl["batch"] if wl["shard_batch"] else wl["batch"] * world,
                "lengths": f"{'log-uniform' if wl['log_uniform'] else 'uniform'} {wl['len_lo']}..{wl['len_hi']}",
                "pool_blocks_per_gpu": work.pool_blocks,
                "kv_bytes_per_step_per_gpu": work.decode_bytes(),
                "step": "append + plan + decode attention + split-K reduce, one CUDA graph",
                "parallelism": (f"dp{world} by request: one batch placed whole-request onto the GPUs' BlockPool "
                                "shards, longest first onto the least-loaded" if wl["shard_batch"] else
                                f"dp{world} by request: every GPU decodes its own batch with the same lengths"),
                "l2": "inputs larger than L2 (K/V per step >> 126 MB)",
            },
            "hbm_frac_per_gpu": round(value / world / hbm_peak, 4),
            "per_gpu": {
                "requests": [int(r[2]) for r in per_gpu],
                "kv_bytes_per_step": kv_bytes,
                "step_ms": [round(r[1], 5) for r in per_gpu],
                "bytes_imbalance_max_over_mean": round(max(kv_bytes) / (sum(kv_bytes) / len(kv_bytes)), 4),
                "note": "value = bytes of all GPUs / the slowest GPU's time; the imbalance bounds the strong-scaling "
                        "efficiency from above",
            },
            "oracle_check": oracle_check,
            "roofline": {
                "kernel": "decode_tc_kernel",
                "bound": "hbm",
                "achieved": round(achieved, 2),
                "peak": hbm_peak,
                "peak_source": f"{peak_src} hbm_gbs (copy)",
                "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "traffic": traffic,
                "traffic_note": traffic_note,
                "algorithmic_bytes_per_launch": att_bytes,
                "launch_ms": att_ms,
            },
            "cpu_baseline": cpu,
            "cpu_baseline_port": cpu_port,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e_ms / steps,
                    "host_issue_ms_per_step": round(e2e["host_issue_ms"], 4),
                    "path": "PagedKVCache + BatchKVCache + CudaPagedAttentionBackend.attend, pinned host I/O"},
            "gpu_launches": 4 * steps,
            "clocks": sampler.summary(),
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_reference(args, wl_name: str) -> None:
    """The reference's CPU decode chain, on host cores, bounded per step: its
    own classes from the installed copy when they import (else the numpy
    restatement), on the first rows of the same workload."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[wl_name]
    seed = 1234
    all_lens = [int(x) for x in request_lengths(wl, seed)]
    threads = os.cpu_count() or 1
    # size the per-step sample so the whole run stays within ~2 minutes
    budget = 120.0 / max(args.steps + args.warmup, 1)
    ref = reference_package()
    if ref is not None:
        torch.set_num_threads(threads)
        lens = ref_sample_rows(ref, wl, all_lens, step_budget_s=budget)
        chain = RefDecodeChain(ref, wl, lens, args.steps + args.warmup + 1)
        with torch.inference_mode():
            for _ in range(args.warmup):
                chain.step()
            t0 = time.perf_counter()
            nbytes = sum(chain.step() for _ in range(args.steps))
            el = time.perf_counter() - t0
        kind = "reference"
        sample = (f"{len(lens)} of {len(all_lens)} requests per step ({sum(lens)} cached tokens, padded to "
                  f"{max(lens)}): the reference's BatchKVCache + SDPAAttentionBackend.attend on its PagedKVCache "
                  f"(installed copy), float32, torch.set_num_threads({threads})")
        dtype = "f32"
    else:
        cand = cpu_sample_lens(all_lens, 8, 20000)
        _, _, per_row = cpu_run(wl, cand[:1], seconds=0.0, min_runs=1, threads=threads)
        n_rows = int(max(1, min(len(cand), budget / max(per_row, 1e-6))))
        lens = cand[:n_rows]
        from oracle import paged_oracle as orc

        kc, vc, tables, lens_a, q, kn, vn = cpu_sample_state(wl, lens)
        nbytes = cpu_bytes(wl, lens) * args.steps
        with ThreadPoolExecutor(threads) as ex:
            for _ in range(args.warmup):
                orc.decode_step_cpu(kc, vc, 0, tables, lens_a, q, kn, vn, executor=ex)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                orc.decode_step_cpu(kc, vc, 0, tables, lens_a, q, kn, vn, executor=ex)
            el = time.perf_counter() - t0
        kind = "port"
        sample = (f"{n_rows} of {len(all_lens)} requests per step ({sum(lens)} cached tokens), float32 numpy "
                  "restatement of the reference decode chain (append, gather + pad, repeat_interleave, mask, SDPA), "
                  "threaded over rows (the reference's installed copy was not found)")
        dtype = "f32"
    value = nbytes / el / 1e9
    res = {
        "metric": "paged-decode KV read GB/s",
        "value": round(value, 4),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": wl.get("scaling", "strong" if wl["shard_batch"] else "weak"),
        "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic",
        "config": {"workload": wl_name, "lengths": f"{wl['len_lo']}..{wl['len_hi']}",
                   "bytes": "same algorithmic accounting as the GPU arm (bf16 element count of the K/V read)"},
        "impl": "reference",
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


# ---------------------------------------------------------------------------
# KV-head-sharded decode
# ---------------------------------------------------------------------------
class HeadShardWorkload:
    """One GPU's head shard of a decode batch: every request, but only KV heads
    [r*Hkv/N, (r+1)*Hkv/N) in this GPU's pool (and the query heads that read
    them).  Block tables are the same on every GPU."""

    def __init__(self, wl: dict, rank: int, world: int, device: torch.device, seed: int = 1234):
        from barellm_b200 import head_shard as hs
        from barellm_b200 import ops

        self.wl, self.device, self.world = wl, device, world
        self.lens = [int(x) for x in request_lengths(wl, seed)]
        b = self.batch = len(self.lens)
        hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
        self.kv0, self.kv1 = hs.kv_head_range(hkv, world, rank)
        self.q0, self.q1 = hs.q_head_range(hq, hkv, world, rank)
        hkv_l, hq_l = self.kv1 - self.kv0, self.q1 - self.q0
        rs = np.random.RandomState(seed)
        need = [-(-(n + 1) // bs) for n in self.lens]
        self.pool_blocks = int(sum(need) * 1.25) + 64
        free = list(rs.permutation(self.pool_blocks))
        tables = [[int(free.pop()) for _ in range(k)] for k in need]
        bt = np.full((b, max(need)), -1, dtype=np.int32)
        for i, t in enumerate(tables):
            bt[i, : len(t)] = t
        self.bt = torch.from_numpy(bt).to(device)
        shape = (1, self.pool_blocks, hkv_l, bs, d)
        self.k_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        self.v_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + 7919 * (rank + 1))
        sc = wl["scale"]
        zeros = torch.zeros(b, dtype=torch.int32, device=device)
        lo = 0
        while lo < b:
            hi, tok = lo, 0
            while hi < b and (tok + self.lens[hi]) * hkv_l * d * 2 <= (1 << 30):
                tok += self.lens[hi]
                hi += 1
            hi = max(hi, lo + 1)
            n = sum(self.lens[lo:hi])
            kh = (torch.randn((1, hkv_l, n, d), generator=gen, device=device) * sc).to(torch.bfloat16)
            vh = (torch.randn((1, hkv_l, n, d), generator=gen, device=device) * sc).to(torch.bfloat16)
            offs = torch.tensor(np.concatenate([[0], np.cumsum(self.lens[lo:hi])]), dtype=torch.int32, device=device)
            ops.paged_append(self.k_cache, self.v_cache, 0, self.bt[lo:hi], zeros[lo:hi], kh, vh,
                             new_offsets=offs, max_new_tokens=max(self.lens[lo:hi]))
            del kh, vh
            lo = hi
        self.q = (torch.randn((b, hq_l, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.k_new = (torch.randn((b, hkv_l, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.v_new = (torch.randn((b, hkv_l, 1, d), generator=gen, device=device) * sc).to(torch.bfloat16)
        self.starts = torch.tensor(self.lens, dtype=torch.int32, device=device)
        self.seq_lens_host = [n + 1 for n in self.lens]
        self.seq_lens = torch.tensor(self.seq_lens_host, dtype=torch.int32, device=device)
        self.max_seq = max(self.seq_lens_host)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.out_local = torch.empty((b, hq_l, d), dtype=torch.bfloat16, device=device)
        self.ws = ops.workspace(device, ops.decode_workspace_bytes(b, hq_l, d, bs, self.max_seq))
        self.shard = hs.HeadShardedDecode(b, hq, hkv, d, torch.bfloat16, device)
        torch.cuda.synchronize(device)

    def local_bytes(self) -> int:
        """This GPU's algorithmic bytes: its heads' K/V of every row, its q
        heads and their outputs."""
        wl = self.wl
        hkv_l, hq_l = self.kv1 - self.kv0, self.q1 - self.q0
        return sum(self.seq_lens_host) * hkv_l * wl["d"] * 2 * 2 + 2 * self.batch * hq_l * wl["d"] * 2

    def step(self) -> torch.Tensor:
        """append -> plan -> attention -> reduce (outputs stored into every
        GPU's gathered buffer) -> completion barrier: 5 launches."""
        from barellm_b200 import ops

        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, self.starts, self.k_new, self.v_new, err=self.err)
        return self.shard.decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, self.max_seq,
                                 ws=self.ws, err=self.err)

    def step_collective(self) -> torch.Tensor:
        """The unfused baseline: the same append and decode into a local
        buffer, then the all-gather through NCCL and a transpose copy."""
        from barellm_b200 import head_shard as hs
        from barellm_b200 import ops

        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, self.starts, self.k_new, self.v_new, err=self.err)
        ops.paged_decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, self.max_seq,
                         out=self.out_local, ws=self.ws, err=self.err)
        return hs.gather_heads_collective(self.out_local)

    def attention(self) -> None:
        from barellm_b200 import ops

        ops.paged_decode(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, self.max_seq,
                         out=self.out_local, ws=self.ws, plan_ready=True, err=self.err, stage="attention")


def capture(fn, device) -> torch.cuda.CUDAGraph:
    fn()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            fn()
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    return graph


def run_heads(args, wl_name: str) -> None:
    from barellm_b200 import ops

    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    wl = WORKLOADS[wl_name]
    work = HeadShardWorkload(wl, rank, world, device)
    steps, warmup = args.steps, args.warmup
    hq, d = wl["hq"], wl["d"]

    graph = capture(work.step, device)
    sampler = ClockSampler(local)
    barrier(world, device)
    with sampler:
        for _ in range(warmup):
            graph.replay()
        ms = time_steps(graph.replay, steps, device)
    barrier(world, device)
    if int(work.err.item()):
        raise RuntimeError(f"device error word {int(work.err.item())}")
    ms_max = allreduce(ms, "max", world, device)
    bytes_step = allreduce(float(work.local_bytes()), "sum", world, device)
    value = bytes_step * steps / (ms_max / 1e3) / 1e9
    del graph

    # the unfused baseline: decode, then NCCL all-gather + transpose (graph
    # captured when there is something to gather)
    coll_graph = capture(work.step_collective, device) if world > 1 else None
    run_coll = coll_graph.replay if coll_graph is not None else work.step_collective
    barrier(world, device)
    for _ in range(warmup):
        run_coll()
    coll_ms = time_steps(run_coll, steps, device)
    barrier(world, device)
    coll_ms_max = allreduce(coll_ms, "max", world, device)
    # the graph holds NCCL work: release it (the bound replay method too)
    # before the process group is destroyed
    del run_coll, coll_graph
    torch.cuda.synchronize(device)

    # dominant kernel alone: this GPU's decode attention kernel
    for _ in range(3):
        work.attention()
    n_att = max(steps, 20)
    att_ms = time_steps(work.attention, n_att, device) / n_att
    hbm_peak, peak_src = load_peaks()
    att_bytes = work.local_bytes()
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    traffic, traffic_note = traffic_from_profile("decode_tc_kernel", "decode_qwen8b_long", att_bytes)

    # end to end through the public API: this GPU's q / new K / new V heads
    # from pinned host memory, append + sharded decode, the gathered
    # [B, Hq, D] output back to the host
    nq, nk = work.q.numel(), work.k_new.numel()
    in_h = torch.cat([work.q.reshape(-1), work.k_new.reshape(-1), work.v_new.reshape(-1)]).cpu().pin_memory()
    in_d = torch.empty_like(in_h, device=device)  # one copy brings q, k and v; views below
    q_d = in_d[:nq].view(work.q.shape)
    k_d = in_d[nq : nq + nk].view(work.k_new.shape)
    v_d = in_d[nq + nk :].view(work.v_new.shape)
    out_h = torch.empty((work.batch, hq, d), dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        in_d.copy_(in_h, non_blocking=True)
        ops.paged_append(work.k_cache, work.v_cache, 0, work.bt, work.starts, k_d, v_d, err=work.err)
        out = work.shard.decode(q_d, work.k_cache, work.v_cache, 0, work.bt, work.seq_lens, work.max_seq,
                                ws=work.ws, err=work.err)
        out_h.copy_(out, non_blocking=True)

    barrier(world, device)
    for _ in range(warmup):
        e2e_step()
    e2e_ms = time_steps(e2e_step, steps, device)
    barrier(world, device)
    e2e_ms_max = allreduce(e2e_ms, "max", world, device)
    e2e_value = bytes_step * steps / (e2e_ms_max / 1e3) / 1e9
    if int(work.err.item()):
        raise RuntimeError(f"device error word {int(work.err.item())}")

    cpu, cpu_port = None, None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu, cpu_port = cpu_baselines(wl, list(work.lens), work.batch, args.cpu_seconds)
    work.shard.close()
    if rank == 0:
        res = {
            "metric": "paged-decode KV read GB/s",
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": ms_max / steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": wl_name,
                "model_shapes": f"{hq}q/{wl['hkv']}kv heads, head_dim {d}, block_size {wl['bs']}",
                "requests_total": work.batch,
                "lengths": f"log-uniform {wl['len_lo']}..{wl['len_hi']}",
                "kv_heads_per_gpu": work.kv1 - work.kv0,
                "pool_blocks_per_gpu": work.pool_blocks,
                "kv_bytes_per_step_per_gpu": work.local_bytes(),
                "step": "append + plan + decode attention + split-K reduce (outputs stored into every GPU's "
                        "gathered buffer) + completion barrier, one CUDA graph",
                "parallelism": f"kv-head shards x{world}, all-gather fused into the decode epilogue (peer stores)",
                "l2": "inputs larger than L2 (K/V per step per GPU >> 126 MB)",
            },
            "hbm_frac_per_gpu": round(value / world / hbm_peak, 4),
            "collective_baseline": {
                "value": round(bytes_step * steps / (coll_ms_max / 1e3) / 1e9, 2),
                "ms_per_step": coll_ms_max / steps,
                "path": "same decode into a local buffer, then all_gather_into_tensor (NCCL) + transpose copy"
                        + (", one CUDA graph" if world > 1 else " (nothing to gather at one GPU)"),
            },
            "roofline": {
                "kernel": "decode_tc_kernel",
                "bound": "hbm",
                "achieved": round(achieved, 2),
                "peak": hbm_peak,
                "peak_source": f"{peak_src} hbm_gbs (copy)",
                "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "traffic": traffic,
                "traffic_note": traffic_note,
                "algorithmic_bytes_per_launch": att_bytes,
                "launch_ms": att_ms,
            },
            "cpu_baseline": cpu,
            "cpu_baseline_port": cpu_port,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": in_h.numel() * 2,
                    "d2h_bytes_per_step": out_h.numel() * 2, "ms_per_step": e2e_ms_max / steps,
                    "path": "ops.paged_append + HeadShardedDecode.decode, pinned host I/O per GPU"},
            "gpu_launches": 5 * steps,
            "clocks": sampler.summary(),
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# chunked prefill
# ---------------------------------------------------------------------------
def prefill_lengths(wl: dict, seed: int) -> tuple[np.ndarray, np.ndarray]:
    rs = np.random.RandomState(seed)
    prefix = rs.randint(wl["prefix_lo"], wl["prefix_hi"] + 1, size=wl["batch"]).astype(np.int64)
    chunk = rs.randint(wl["chunk_lo"], wl["chunk_hi"] + 1, size=wl["batch"]).astype(np.int64)
    return prefix, chunk


def prefill_flops(hq: int, d: int, prefix, chunk) -> float:
    """4 * Hq * D * (C*P + C(C+1)/2) per request: Q.K^T and P.V over the causal keys."""
    return float(sum(4 * hq * d * (c * p + c * (c + 1) / 2) for p, c in zip(prefix, chunk)))


class PrefillWorkload:
    """One GPU's share of the chunked-prefill workload, device resident."""

    def __init__(self, wl: dict, rank: int, world: int, device: torch.device, seed: int = 4321):
        from barellm_b200 import ops

        self.wl = wl
        self.device = device
        prefix_all, chunk_all = prefill_lengths(wl, seed)
        mine = place_requests(prefix_all + chunk_all, world)[rank]
        self.prefix = [int(prefix_all[i]) for i in mine]
        self.chunk = [int(chunk_all[i]) for i in mine]
        b = len(mine)
        self.batch = b
        hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
        self.pool_blocks = wl["pool_blocks"]
        rs = np.random.RandomState(seed + rank)
        free = list(rs.permutation(self.pool_blocks))
        totals = [p + c for p, c in zip(self.prefix, self.chunk)]
        tables = [[int(free.pop()) for _ in range(-(-n // bs))] for n in totals]
        bt = np.full((b, max(len(t) for t in tables)), -1, dtype=np.int32)
        for i, t in enumerate(tables):
            bt[i, : len(t)] = t
        self.bt = torch.from_numpy(bt).to(device)
        shape = (1, self.pool_blocks, hkv, bs, d)
        self.k_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        self.v_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed + rank)
        zeros = torch.zeros(b, dtype=torch.int32, device=device)
        if sum(self.prefix):
            n = sum(self.prefix)
            kh = torch.randn((1, hkv, n, d), generator=gen, device=device).to(torch.bfloat16)
            vh = torch.randn((1, hkv, n, d), generator=gen, device=device).to(torch.bfloat16)
            offs = torch.tensor(np.concatenate([[0], np.cumsum(self.prefix)]), dtype=torch.int32, device=device)
            ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, zeros, kh, vh, new_offsets=offs,
                             max_new_tokens=max(max(self.prefix), 1))
            del kh, vh
        nc = sum(self.chunk)
        # q as the model produces it: [1, T, Hq, D] memory viewed as [1, Hq, T, D]
        self.q = torch.randn((1, nc, hq, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
        self.k_new = torch.randn((1, nc, hkv, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
        self.v_new = torch.randn((1, nc, hkv, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
        self.q_offs = torch.tensor(np.concatenate([[0], np.cumsum(self.chunk)]), dtype=torch.int32, device=device)
        self.starts = torch.tensor(self.prefix, dtype=torch.int32, device=device)
        self.seq_lens = torch.tensor(totals, dtype=torch.int32, device=device)
        self.out = torch.empty((1, nc, hq, d), dtype=torch.bfloat16, device=device).transpose(1, 2)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.flops = prefill_flops(hq, d, self.prefix, self.chunk)
        torch.cuda.synchronize(device)

    def append(self) -> None:
        from barellm_b200 import ops

        ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, self.starts, self.k_new, self.v_new,
                         new_offsets=self.q_offs, max_new_tokens=max(self.chunk), err=self.err)

    def attention(self) -> None:
        from barellm_b200 import ops

        ops.paged_prefill(self.q, self.k_cache, self.v_cache, 0, self.bt, self.seq_lens, q_offsets=self.q_offs,
                          max_q_len=max(self.chunk), out=self.out, err=self.err)

    def step(self) -> None:
        self.append()
        self.attention()


def prefill_e2e(wl: dict, work: PrefillWorkload, steps: int, warmup: int, device) -> dict:
    """Chunked prefill through the public API, one request at a time as the
    engine's prefill does: pinned host chunk -> PagedLayerKV attend -> host."""
    from barellm_b200 import BlockPool, CudaPagedAttentionBackend, KVCacheManager, PagedKVCache, ops

    hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
    totals = [p + c for p, c in zip(work.prefix, work.chunk)]
    need = sum(-(-n // bs) for n in totals)
    kv = PagedKVCache(1, need + 64, hkv, bs, d, dtype=torch.bfloat16, device=device, max_requests=work.batch)
    pool = BlockPool(need + 64)
    pool.free_ids = [int(x) for x in np.random.RandomState(7).permutation(need + 64)]
    mgr = KVCacheManager(bs, pool, kv)

    class Req:
        def __init__(self, i, n):
            self.id, self.seq_len = f"p{i}", n

    layers = []
    for i, (p, n) in enumerate(zip(work.prefix, totals)):
        r = Req(i, n)
        assert mgr.allocate_request(r)
        layer = mgr.get_cache(r).layer(0)
        if p:
            kd, vd = ops.paged_gather(work.k_cache, work.v_cache, 0, work.bt[i : i + 1],
                                      torch.tensor([p], dtype=torch.int32, device=device), p)
            layer.append_only(kd, vd)
        layers.append(layer)
    offs = [0] + list(np.cumsum(work.chunk))
    host = [(work.q[:, :, offs[i] : offs[i + 1]].transpose(1, 2).contiguous().cpu().pin_memory(),
             work.k_new[:, :, offs[i] : offs[i + 1]].transpose(1, 2).contiguous().cpu().pin_memory(),
             work.v_new[:, :, offs[i] : offs[i + 1]].transpose(1, 2).contiguous().cpu().pin_memory())
            for i in range(work.batch)]
    dev = [(torch.empty_like(q, device=device), torch.empty_like(k, device=device), torch.empty_like(v, device=device))
           for q, k, v in host]
    outs_h = [torch.empty((1, c, hq, d), dtype=torch.bfloat16).pin_memory() for c in work.chunk]
    backend = CudaPagedAttentionBackend()

    def one():
        for i, layer in enumerate(layers):
            layer._request.layer_seq_lens[0] = work.prefix[i]  # re-prefill the same chunk each step
            qd, kd, vd = dev[i]
            qd.copy_(host[i][0], non_blocking=True)
            kd.copy_(host[i][1], non_blocking=True)
            vd.copy_(host[i][2], non_blocking=True)
            out = backend.attend(qd.transpose(1, 2), kd.transpose(1, 2), vd.transpose(1, 2), layer, hq // hkv)
            outs_h[i].copy_(out.transpose(1, 2), non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize(device)
    ms = time_steps(one, steps, device)
    kv.check_device_errors()
    h2d = sum((q.numel() + k.numel() + v.numel()) * 2 for q, k, v in host)
    return {"ms": ms, "h2d": h2d, "d2h": sum(o.numel() * 2 for o in outs_h)}


def run_prefill(args, wl_name: str) -> None:
    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    wl = WORKLOADS[wl_name]
    work = PrefillWorkload(wl, rank, world, device)
    steps, warmup = args.steps, args.warmup
    work.step()
    torch.cuda.synchronize(device)
    sampler = ClockSampler(local)
    barrier(world, device)
    with sampler:
        for _ in range(warmup):
            work.step()
        ms = time_steps(work.step, steps, device)
    barrier(world, device)
    if int(work.err.item()):
        raise RuntimeError(f"device error word {int(work.err.item())}")
    ms_max = allreduce(ms, "max", world, device)
    flops_all = allreduce(work.flops, "sum", world, device)
    value = flops_all * steps / (ms_max / 1e3) / 1e12
    att_ms = time_steps(work.attention, max(steps, 5), device) / max(steps, 5)
    peak, peak_src = load_peaks("bf16_tflops")
    achieved = work.flops / (att_ms / 1e3) / 1e12
    traffic, traffic_note = traffic_from_profile("prefill_tc_kernel", wl_name)
    e2e = prefill_e2e(wl, work, steps, warmup, device)
    e2e_ms = allreduce(e2e["ms"], "max", world, device)
    e2e_value = flops_all * steps / (e2e_ms / 1e3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = prefill_cpu(wl, work.prefix[0], min(work.chunk[0], 256), args.cpu_seconds)
    if rank == 0:
        res = {
            "metric": "paged chunked-prefill attention TFLOP/s",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": ms_max / steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {
                "workload": wl_name,
                "model_shapes": f"{wl['hq']}q/{wl['hkv']}kv heads, head_dim {wl['d']}, block_size {wl['bs']}",
                "requests_total": wl["batch"],
                "prefix": f"uniform {wl['prefix_lo']}..{wl['prefix_hi']}",
                "chunk": f"uniform {wl['chunk_lo']}..{wl['chunk_hi']}",
                "flops_per_step_per_gpu": work.flops,
                "step": "packed chunk append + paged prefill attention (bottom-right causal)",
                "parallelism": f"dp{world} by request",
                "l2": "K/V re-read per query tile; working set > L2",
            },
            "roofline": {"kernel": "prefill_tc_kernel", "bound": "tensor", "achieved": round(achieved, 2),
                         "peak": peak, "peak_source": f"{peak_src} bf16_tflops (cuBLAS burst)", "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_note": traffic_note,
                         "launch_ms": att_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e_ms / steps,
                    "path": "PagedKVCache + CudaPagedAttentionBackend.attend per request (engine prefill path)"},
            "gpu_launches": 2 * steps,
            "clocks": sampler.summary(),
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def prefill_cpu(wl: dict, prefix: int, chunk: int, seconds: float, runs_min: int = 1, warmup: int = 1) -> dict:
    """The reference's read + repeat_interleave + masked SDPA for one request
    (float32 numpy), timed on the host."""
    from oracle import paged_oracle as orc

    hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
    rs = np.random.RandomState(3)
    n = prefix + chunk
    nb = -(-n // bs)
    kc = np.zeros((1, nb, hkv, bs, d), np.float32)
    vc = np.zeros_like(kc)
    table = rs.permutation(nb)
    orc.append_only(kc, vc, 0, table, 0, rs.standard_normal((1, hkv, n, d)).astype(np.float32),
                    rs.standard_normal((1, hkv, n, d)).astype(np.float32))
    q = rs.standard_normal((1, hq, chunk, d)).astype(np.float32)
    g = hq // hkv

    def run():
        k, v = orc.read(kc, vc, 0, table, n)
        mask = orc.causal_mask_bottom_right(chunk, n)[None, None]
        return orc._sdpa_f32(q, orc.repeat_kv(k, g), orc.repeat_kv(v, g), mask)

    for _ in range(warmup):
        run()
    t0 = time.perf_counter()
    runs = 0
    while runs < runs_min or time.perf_counter() - t0 < seconds:
        run()
        runs += 1
    el = (time.perf_counter() - t0) / runs
    fl = prefill_flops(hq, d, [prefix], [chunk])
    return {"value": round(fl / el / 1e12, 6), "unit": "TFLOP/s", "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"one request, prefix {prefix} + chunk {chunk}, {runs} runs of {el:.3f} s, float32 numpy"}


def run_reference_prefill(args, wl_name: str) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[wl_name]
    prefix, chunk = prefill_lengths(wl, 4321)
    budget = 120.0 / max(args.steps + args.warmup, 1)
    c = 256
    while True:  # shrink the sampled chunk until one step fits the per-step budget
        probe = prefill_cpu(wl, int(prefix[0]), c, 0.0)
        per = float(probe["sample"].split(" runs of ")[1].split(" s")[0])
        if per <= budget or c <= 16:
            break
        c //= 2
    cpu = prefill_cpu(wl, int(prefix[0]), c, 0.0, runs_min=args.steps, warmup=args.warmup)
    per = float(cpu["sample"].split(" runs of ")[1].split(" s")[0])
    res = {"metric": "paged chunked-prefill attention TFLOP/s", "value": cpu["value"], "unit": "TFLOP/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": wl_name}, "impl": "reference", "cpu_baseline": cpu,
           "e2e": {"value": cpu["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# ---------------------------------------------------------------------------
# K/V copies: chunk append, fused QK prep + append, dense gather
# ---------------------------------------------------------------------------
def rope_tables(positions: np.ndarray, d: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin ``[1, 1, T, D]`` of the half-split rotary embedding at the
    given positions (inverse frequencies theta^(-2i/D), the angle table
    repeated over both halves), rounded to bf16."""
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))
    ang = torch.from_numpy(positions.astype(np.float32)).to(device)[:, None] * inv[None, :]
    emb = torch.cat((ang, ang), dim=-1)
    return emb.cos().to(torch.bfloat16)[None, None], emb.sin().to(torch.bfloat16)[None, None]


class CopyWorkload:
    """One GPU's share of a K/V copy workload, device resident.

    append / qkprep: the chunk tokens of the chunked-prefill workload, packed
    on the token axis in the model's layout (``[1, T, H, D]`` memory viewed
    as ``[1, H, T, D]``), written into fresh pages after each request's
    prefix (one launch per step; repeated steps rewrite the same slots).
    gather: the decode workload's cached tokens read into a zero-padded
    ``[B, Hkv, Tmax, D]`` K/V pair (the reference's read + pad)."""

    def __init__(self, wl: dict, rank: int, world: int, device: torch.device):
        self.wl = wl
        self.op = wl["op"]
        self.device = device
        hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
        row = d * 2  # bytes of one bf16 row
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        if self.op == "gather":
            dw = DecodeWorkload(wl, rank, world, device)
            self.dw = dw
            self.batch, self.pool_blocks = dw.batch, dw.pool_blocks
            self.k_cache, self.v_cache, self.bt = dw.k_cache, dw.v_cache, dw.bt
            self.lens = list(dw.lens)
            self.seq = torch.tensor(self.lens, dtype=torch.int32, device=device)
            self.max_len = max(self.lens)
            shape = (self.batch, hkv, self.max_len, d)
            self.k_out = torch.empty(shape, dtype=torch.bfloat16, device=device)
            self.v_out = torch.empty_like(self.k_out)
            useful = sum(self.lens) * hkv * row
            pad = (self.batch * self.max_len - sum(self.lens)) * hkv * row
            # read + write of every cached K and V row, plus the zero rows of the padding
            self.bytes = 2 * (2 * useful) + 2 * pad
            self.tokens = sum(self.lens)
            self.kernel = "paged_gather_kernel"
        else:
            prefix_all, chunk_all = prefill_lengths(wl, 4321)
            mine = place_requests(prefix_all + chunk_all, world)[rank]
            self.prefix = [int(prefix_all[i]) for i in mine]
            self.chunk = [int(chunk_all[i]) for i in mine]
            b = len(mine)
            self.batch = b
            self.pool_blocks = wl["pool_blocks"]
            rs = np.random.RandomState(4321 + rank)
            free = list(rs.permutation(self.pool_blocks))
            totals = [p + c for p, c in zip(self.prefix, self.chunk)]
            tables = [[int(free.pop()) for _ in range(-(-n // bs))] for n in totals]
            bt = np.full((b, max(len(t) for t in tables)), -1, dtype=np.int32)
            for i, t in enumerate(tables):
                bt[i, : len(t)] = t
            self.bt = torch.from_numpy(bt).to(device)
            shape = (1, self.pool_blocks, hkv, bs, d)
            self.k_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
            self.v_cache = torch.empty(shape, dtype=torch.bfloat16, device=device)
            gen = torch.Generator(device=device)
            gen.manual_seed(4321 + rank)
            nc = sum(self.chunk)
            self.tokens = nc
            self.k_new = torch.randn((1, nc, hkv, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
            self.v_new = torch.randn((1, nc, hkv, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
            self.offs = torch.tensor(np.concatenate([[0], np.cumsum(self.chunk)]), dtype=torch.int32, device=device)
            self.starts = torch.tensor(self.prefix, dtype=torch.int32, device=device)
            self.max_chunk = max(self.chunk)
            if self.op == "append":
                # read + write of every new K and V row
                self.bytes = 2 * 2 * nc * hkv * row
                self.kernel = "paged_append_kernel"
            else:
                self.q = torch.randn((1, nc, hq, d), generator=gen, device=device).to(torch.bfloat16).transpose(1, 2)
                self.q_out = torch.empty((1, nc, hq, d), dtype=torch.bfloat16, device=device).transpose(1, 2)
                self.qw = (1 + 0.1 * torch.randn(d, generator=gen, device=device)).to(torch.bfloat16)
                self.kw = (1 + 0.1 * torch.randn(d, generator=gen, device=device)).to(torch.bfloat16)
                pos = np.concatenate([np.arange(p, p + c) for p, c in zip(self.prefix, self.chunk)])
                self.cos, self.sin = rope_tables(pos, d, 1e6, device)
                # read + write of every q, k and v row, plus one cos and one sin row per token
                self.bytes = 2 * nc * (hq + 2 * hkv) * row + 2 * nc * row
                self.kernel = "qk_prep_kernel"
        torch.cuda.synchronize(device)

    def step(self) -> None:
        from barellm_b200 import ops

        if self.op == "gather":
            ops.paged_gather(self.k_cache, self.v_cache, 0, self.bt, self.seq, self.max_len,
                             out=(self.k_out, self.v_out), err=self.err)
        elif self.op == "append":
            ops.paged_append(self.k_cache, self.v_cache, 0, self.bt, self.starts, self.k_new, self.v_new,
                             new_offsets=self.offs, max_new_tokens=self.max_chunk, err=self.err)
        else:
            ops.qk_norm_rope_append(self.q, self.k_new, self.v_new, self.qw, self.kw, self.cos, self.sin, 1e-6,
                                    self.k_cache, self.v_cache, 0, self.bt, self.starts, new_offsets=self.offs,
                                    max_new_tokens=self.max_chunk, q_out=self.q_out, err=self.err)


def copy_e2e(work: CopyWorkload, steps: int, warmup: int, device) -> dict:
    """The same copy through the public cache API with host buffers: append /
    qkprep through PackedBatchKVCache (inputs copied from pinned host memory
    every step, the error word or the prepared q read back); gather through
    BatchKVCache.read (the dense K/V copied back to pinned host memory)."""
    from barellm_b200 import BatchKVCache, BlockPool, KVCacheManager, PackedBatchKVCache, PagedKVCache, ops

    wl = work.wl
    hkv, d, bs = wl["hkv"], wl["d"], wl["bs"]
    if work.op == "gather":
        lens = work.lens
    else:
        lens = [p + c for p, c in zip(work.prefix, work.chunk)]
    need = sum(-(-n // bs) for n in lens)
    kv = PagedKVCache(1, need + 64, hkv, bs, d, dtype=torch.bfloat16, device=device, max_requests=work.batch)
    pool = BlockPool(need + 64)
    pool.free_ids = [int(x) for x in np.random.RandomState(11).permutation(need + 64)]
    mgr = KVCacheManager(bs, pool, kv)

    class Req:
        def __init__(self, i, n):
            self.id, self.seq_len = f"c{i}", n

    reqs = [Req(i, n) for i, n in enumerate(lens)]
    for r in reqs:
        assert mgr.allocate_request(r)
    views = [mgr.get_cache(r) for r in reqs]
    rows = np.array([kv.request_pages[v.request_id].row for v in views])
    if work.op == "gather":
        for i, vw in enumerate(views):
            n = lens[i]
            kd, vd = ops.paged_gather(work.k_cache, work.v_cache, 0, work.bt[i : i + 1],
                                      torch.tensor([n], dtype=torch.int32, device=device), n)
            vw.layer(0).append_only(kd, vd)
            del kd, vd
        shape = (work.batch, hkv, work.max_len, d)
        k_h = torch.empty(shape, dtype=torch.bfloat16).pin_memory()
        v_h = torch.empty(shape, dtype=torch.bfloat16).pin_memory()

        def one():
            k, v = BatchKVCache(views).layer(0).read()
            k_h.copy_(k, non_blocking=True)
            v_h.copy_(v, non_blocking=True)

        h2d, d2h = 0, 2 * k_h.numel() * 2
    else:
        prefix = np.array(work.prefix)
        nc = work.tokens
        k_h = work.k_new.transpose(1, 2).contiguous().cpu().pin_memory()
        v_h = work.v_new.transpose(1, 2).contiguous().cpu().pin_memory()
        k_d, v_d = torch.empty_like(k_h, device=device), torch.empty_like(v_h, device=device)
        err_h = torch.zeros(1, dtype=torch.int32).pin_memory()
        h2d, d2h = 2 * k_h.numel() * 2, 4
        if work.op == "qkprep":
            q_h = work.q.transpose(1, 2).contiguous().cpu().pin_memory()
            q_d = torch.empty_like(q_h, device=device)
            qo_h = torch.empty_like(q_h).pin_memory()
            h2d += q_h.numel() * 2
            d2h = qo_h.numel() * 2

        def one():
            kv.arena.lens[rows, 0] = prefix  # the same chunks are appended again every step
            k_d.copy_(k_h, non_blocking=True)
            v_d.copy_(v_h, non_blocking=True)
            layer = PackedBatchKVCache(views, work.chunk).layer(0)
            if work.op == "append":
                layer.append_only(k_d.transpose(1, 2), v_d.transpose(1, 2))
                err_h.copy_(kv.err, non_blocking=True)
            else:
                q_d.copy_(q_h, non_blocking=True)
                _, qo = layer.append_only_prepped(q_d.transpose(1, 2), k_d.transpose(1, 2), v_d.transpose(1, 2),
                                                  work.qw, work.kw, work.cos, work.sin, 1e-6)
                qo_h.copy_(qo.transpose(1, 2), non_blocking=True)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize(device)
    ms = time_steps(one, steps, device)
    kv.check_device_errors()
    return {"ms": ms, "h2d": h2d, "d2h": d2h}


def copy_cpu(wl: dict, work_like: dict, seconds: float, runs_min: int = 1, warmup: int = 1) -> dict:
    """The reference's CPU copy for a bounded sample (float32 numpy, one
    thread): append_only of one request's chunk, apply_rope(norm(.)) of its
    q / k rows plus the append, or read + pad of a few requests."""
    from oracle import paged_oracle as orc

    op = wl["op"]
    hq, hkv, d, bs = wl["hq"], wl["hkv"], wl["d"], wl["bs"]
    row = d * 2
    rs = np.random.RandomState(3)
    if op == "gather":
        lens = work_like["lens"]
        need = [-(-n // bs) for n in lens]
        perm = rs.permutation(sum(need))
        tables, at = [], 0
        for k in need:
            tables.append(perm[at : at + k])
            at += k
        kc = rs.standard_normal((1, sum(need), hkv, bs, d)).astype(np.float32)
        vc = rs.standard_normal((1, sum(need), hkv, bs, d)).astype(np.float32)
        tmax = max(lens)
        nbytes = 4 * sum(lens) * hkv * row + 2 * (len(lens) * tmax - sum(lens)) * hkv * row

        def run():
            orc.batch_read_pad(kc, vc, 0, tables, lens)

        sample = f"read + pad of {len(lens)} requests ({sum(lens)} cached tokens)"
    else:
        p, c = work_like["prefix"], work_like["chunk"]
        nb = -(-(p + c) // bs)
        kc = np.zeros((1, nb, hkv, bs, d), np.float32)
        vc = np.zeros_like(kc)
        table = rs.permutation(nb)
        k = rs.standard_normal((1, hkv, c, d)).astype(np.float32)
        v = rs.standard_normal((1, hkv, c, d)).astype(np.float32)
        if op == "append":
            nbytes = 4 * c * hkv * row

            def run():
                orc.append_only(kc, vc, 0, table, p, k, v)

            sample = f"append_only of one request's chunk ({c} tokens after a prefix of {p})"
        else:
            q = rs.standard_normal((1, hq, c, d)).astype(np.float32)
            w = (1 + 0.1 * rs.standard_normal(d)).astype(np.float32)
            pos = np.arange(p, p + c, dtype=np.float64)
            inv = 1.0 / (1e6 ** (np.arange(0, d, 2) / d))
            ang = np.concatenate([pos[:, None] * inv[None]] * 2, axis=-1)
            cos, sin = np.cos(ang).astype(np.float32)[None, None], np.sin(ang).astype(np.float32)[None, None]
            nbytes = 2 * c * (hq + 2 * hkv) * row + 2 * c * row

            def run():
                orc.qk_norm_rope(q, w, cos, sin, 1e-6)
                kr = orc.qk_norm_rope(k, w, cos, sin, 1e-6).astype(np.float32)
                orc.append_only(kc, vc, 0, table, p, kr, v)

            sample = f"q/k norm + rope and append_only of one request's chunk ({c} tokens after a prefix of {p})"
    for _ in range(warmup):
        run()
    t0 = time.perf_counter()
    runs = 0
    while runs < runs_min or time.perf_counter() - t0 < seconds:
        run()
        runs += 1
    el = (time.perf_counter() - t0) / runs
    return {"value": round(nbytes / el / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{sample}, {runs} runs of {el:.4f} s, float32 numpy restatement of the reference", "per": el}


COPY_METRIC = {"append": "paged K/V append GB/s", "qkprep": "fused QK-norm + RoPE + append GB/s",
               "gather": "paged K/V dense read GB/s"}


def copy_sample(wl: dict, work: CopyWorkload | None = None) -> dict:
    """The request(s) the CPU sample copies: the workload's first request (its
    first few for gather)."""
    if wl["op"] == "gather":
        lens = work.lens if work is not None else [int(x) for x in request_lengths(wl, 1234)]
        return {"lens": cpu_sample_lens(lens, 8, 20000)}
    if work is not None:
        return {"prefix": work.prefix[0], "chunk": work.chunk[0]}
    prefix, chunk = prefill_lengths(wl, 4321)
    return {"prefix": int(prefix[0]), "chunk": int(chunk[0])}


def run_copy(args, wl_name: str) -> None:
    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    wl = WORKLOADS[wl_name]
    work = CopyWorkload(wl, rank, world, device)
    steps, warmup = args.steps, args.warmup
    work.step()
    torch.cuda.synchronize(device)
    sampler = ClockSampler(local)
    barrier(world, device)
    with sampler:
        for _ in range(warmup):
            work.step()
        ms = time_steps(work.step, steps, device)
    barrier(world, device)
    if int(work.err.item()):
        raise RuntimeError(f"device error word {int(work.err.item())}")
    ms_max = allreduce(ms, "max", world, device)
    bytes_all = allreduce(float(work.bytes), "sum", world, device)
    value = bytes_all * steps / (ms_max / 1e3) / 1e9
    launch_ms = ms / steps  # one launch per step
    peak, peak_src = load_peaks()
    achieved = work.bytes / (launch_ms / 1e3) / 1e9
    traffic, traffic_note = traffic_from_profile(work.kernel, wl_name)
    e2e = copy_e2e(work, steps, warmup, device)
    e2e_ms = allreduce(e2e["ms"], "max", world, device)
    e2e_value = bytes_all * steps / (e2e_ms / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = copy_cpu(wl, copy_sample(wl, work), args.cpu_seconds)
        cpu.pop("per")
    if rank == 0:
        if work.op == "gather":
            cfg = {"lengths": f"uniform {wl['len_lo']}..{wl['len_hi']}", "requests_per_gpu": work.batch,
                   "output": "[B, Hkv, Tmax, D] K and V, zero padded", "step": "one paged_gather_kernel launch"}
        else:
            cfg = {"prefix": f"uniform {wl['prefix_lo']}..{wl['prefix_hi']}",
                   "chunk": f"uniform {wl['chunk_lo']}..{wl['chunk_hi']}", "requests_total": wl["batch"],
                   "tokens_per_gpu": work.tokens,
                   "step": f"one {work.kernel} launch over the packed chunks"}
        res = {
            "metric": COPY_METRIC[work.op],
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": warmup,
            "ms_per_step": ms_max / steps,
            "higher_is_better": True,
            "scaling": "strong" if wl["shard_batch"] else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": dict({"workload": wl_name, "model_shapes": f"{wl['hq']}q/{wl['hkv']}kv heads, head_dim "
                            f"{wl['d']}, block_size {wl['bs']}", "pool_blocks_per_gpu": work.pool_blocks,
                            "bytes_per_step_per_gpu": work.bytes, "parallelism": f"dp{world} by request",
                            "l2": "bytes per step > L2 (126 MB)"}, **cfg),
            "roofline": {"kernel": work.kernel, "bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "peak_source": f"{peak_src} hbm_gbs (copy)", "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_note": traffic_note,
                         "algorithmic_bytes_per_launch": work.bytes, "launch_ms": launch_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": e2e_ms / steps,
                    "path": ("BatchKVCache.read, pinned host outputs" if work.op == "gather" else
                             "PackedBatchKVCache.append_only" + ("_prepped" if work.op == "qkprep" else "") +
                             ", pinned host inputs")},
            "gpu_launches": steps,
            "clocks": sampler.summary(),
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_reference_copy(args, wl_name: str) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    wl = WORKLOADS[wl_name]
    sample = copy_sample(wl)
    cpu = copy_cpu(wl, sample, 0.0, runs_min=args.steps, warmup=args.warmup)
    per = cpu.pop("per")
    res = {"metric": COPY_METRIC[wl["op"]], "value": cpu["value"], "unit": "GB/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
           "scaling": "strong" if wl["shard_batch"] else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": {"workload": wl_name}, "impl": "reference", "cpu_baseline": cpu,
           "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


# ---------------------------------------------------------------------------
# end to end (model + engine)
# ---------------------------------------------------------------------------
def run_e2e(args, wl_name: str) -> None:
    from barellm_b200.engine import QWEN3_06B, PagedEngine, random_qwen3

    rank, world, local = dist_env()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=device)
    wl = WORKLOADS[wl_name]
    rs = np.random.RandomState(2024)
    lens = rs.randint(wl["prompt_lo"], wl["prompt_hi"] + 1, size=wl["batch"])
    prompts_all = [list(rs.randint(0, QWEN3_06B.vocab_size, size=int(n))) for n in lens]
    mine = place_requests(lens, world)[rank]
    prompts = [prompts_all[i] for i in mine]
    n_new = wl["new_tokens"]
    model = random_qwen3(QWEN3_06B, dtype=torch.bfloat16, device=device, seed=0)
    blocks = PagedEngine.blocks_needed([len(p) for p in prompts], n_new, 16) + 16
    engine = PagedEngine(model, num_blocks=blocks, max_requests=len(prompts))
    # warm-up: a short run over the first requests (kernels, allocator, cuBLAS)
    engine.generate(prompts[: min(4, len(prompts))], max_new_tokens=min(8, n_new))
    barrier(world, device)
    sampler = ClockSampler(local)
    tm: dict = {}
    with sampler:
        out = engine.generate(prompts, max_new_tokens=n_new, timings=tm)
    barrier(world, device)
    decode_tokens = allreduce(float(len(prompts) * tm["decode_steps"]), "sum", world, device)
    decode_ms = allreduce(tm["decode_ms"], "max", world, device)
    prefill_ms = allreduce(tm["prefill_ms"], "max", world, device)
    prompt_tokens = allreduce(float(sum(len(p) for p in prompts)), "sum", world, device)
    value = decode_tokens / (decode_ms / 1e3)
    s = QWEN3_06B
    mid = [len(p) + n_new // 2 for p in prompts]
    kv_mid = sum(mid) * s.num_layers * s.num_kv_heads * s.head_dim * 2 * 2
    if rank == 0:
        res = {
            "metric": "decode tok/s",
            "value": round(value, 1),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": tm["decode_steps"],
            "warmup": 1,
            "ms_per_step": decode_ms / tm["decode_steps"],
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random token ids, random-init weights)",
            "config": {"workload": wl_name, "model": "Qwen3-0.6B architecture (28 layers, 1024 hidden, 16q/8kv, "
                       "head_dim 128, vocab 151936, tied head)", "requests_total": wl["batch"],
                       "prompts": f"uniform {wl['prompt_lo']}..{wl['prompt_hi']}", "new_tokens": n_new,
                       "parallelism": f"dp{world} by request", "kv_bytes_per_decode_step_mid_run_gpu0": kv_mid},
            "prefill_tok_s": round(prompt_tokens / (prefill_ms / 1e3), 1),
            "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": 16 * len(prompts),
                    "d2h_bytes_per_step": 8 * len(prompts),
                    "path": "barellm_b200.engine.PagedEngine.generate (token ids in, token ids out)"},
            "gpu_launches": None,
            "clocks": sampler.summary(),
            "first_tokens_req0": out[0][:8] if out else [],
        }
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_refengine(args, wl_name: str) -> None:
    """Decode tok/s of the reference's own engine and model on one GPU, on its
    "sdpa" backend and with the paged CUDA path swapped in underneath."""
    rank, world, local = dist_env()
    if world != 1:
        raise SystemExit("refengine_qwen06b runs on one GPU")
    ref = reference_package()
    if ref is None:
        print(json.dumps({"unavailable": "the reference's installed copy (baseline/_ref) is not present",
                          "config": {"workload": wl_name}}))
        return
    import barellm.engine.engine as engine_mod
    from barellm.engine.events import DecodeBatchEnd, ModelForwardEnd, PrefillEnd, TimingConfig
    from barellm.engine.request import Request
    from barellm.engine.scheduler import Scheduler
    from barellm.models.qwen3 import Qwen3ForCausalLM

    import barellm_b200 as bb

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    wl = WORKLOADS[wl_name]
    L, H, HKV, D, VOCAB = 28, 16, 8, 128, 151936
    torch.manual_seed(0)
    with torch.device("cpu"):
        model = Qwen3ForCausalLM(VOCAB, 1024, 3072, D, L, H, HKV, use_qk_norm=True, attention_backend="sdpa")
        g = torch.Generator().manual_seed(7)
        with torch.no_grad():
            for name, prm in model.named_parameters():
                if "embed" in name:
                    prm.copy_(torch.randn(prm.shape, generator=g) * 0.02)
                elif prm.ndim == 2:
                    prm.copy_(torch.randn(prm.shape, generator=g) / prm.shape[1] ** 0.5)
    model = model.to(device=device, dtype=torch.bfloat16).eval()
    sdpa_backends = [blk.self_attn._backend for blk in model.layers]
    rs = np.random.RandomState(2024)
    lens = rs.randint(wl["prompt_lo"], wl["prompt_hi"] + 1, size=wl["batch"])
    prompts = [[int(x) for x in rs.randint(0, VOCAB, size=int(n))] for n in lens]
    n_new = wl["new_tokens"]
    blocks = sum(-(-(len(p) + n_new) // 16) for p in prompts) + 16

    def run(kind: str, prompt_list, new_tokens) -> dict:
        for blk, sd in zip(model.layers, sdpa_backends):
            blk.self_attn._backend = sd if kind == "sdpa" else bb.CudaPagedAttentionBackend()
        if kind == "sdpa":
            kv = ref.PagedKVCache(num_layers=L, max_blocks=blocks, num_kv_heads=HKV, block_size=16, head_dim=D,
                                  dtype=torch.bfloat16, device=device)
        else:
            kv = bb.PagedKVCache(L, blocks, HKV, 16, D, dtype=torch.bfloat16, device=device,
                                 max_requests=len(prompt_list))
        mgr = ref.KVCacheManager(16, ref.BlockPool(blocks), kv)
        eng = engine_mod.Engine(model=model, scheduler=Scheduler(max_batch=wl["max_batch"]), kv_cache_manager=mgr)
        reqs = [Request(id=f"r{i}", token_ids=torch.tensor([p], dtype=torch.long, device=device), temperature=0.0,
                        max_new_tokens=new_tokens) for i, p in enumerate(prompt_list)]
        for r in reqs:
            eng.scheduler.add_request(r)
        st = {"decode_s": 0.0, "decode_tokens": 0, "forward_s": 0.0, "prefill_s": 0.0}

        def on_event(ev):
            if isinstance(ev, DecodeBatchEnd):
                st["decode_s"] += ev.duration_seconds
                st["decode_tokens"] += len(ev.request_ids)
            elif isinstance(ev, ModelForwardEnd) and ev.phase == "decode":
                st["forward_s"] += ev.duration_seconds
            elif isinstance(ev, PrefillEnd):
                st["prefill_s"] += ev.duration_seconds

        eng.run(on_event=on_event, timing=TimingConfig(synchronize_device=True))
        st["tokens"] = [r.token_ids[0, len(p):].tolist() for r, p in zip(reqs, prompt_list)]
        return st

    # warm-up of both paths (kernels, allocator, cuBLAS)
    for kind in ("sdpa", "cuda"):
        run(kind, prompts[:2], 4)
    sampler = ClockSampler(local)
    with sampler:
        res = {kind: run(kind, prompts, n_new) for kind in ("sdpa", "cuda")}
    tok_s = {k: v["decode_tokens"] / v["decode_s"] for k, v in res.items()}
    same = sum(a == b for a, b in zip(res["sdpa"]["tokens"], res["cuda"]["tokens"]))
    first_div = [next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), len(a))
                 for a, b in zip(res["sdpa"]["tokens"], res["cuda"]["tokens"])]
    out = {
        "metric": "decode tok/s",
        "value": round(tok_s["cuda"], 1),
        "unit": "tok/s",
        "n_gpus": 1,
        "steps": n_new - 1,
        "warmup": 1,
        "ms_per_step": res["cuda"]["decode_s"] * 1e3 / max(n_new - 1, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random token ids, random-init weights)",
        "config": {"workload": wl_name, "model": "the reference's Qwen3ForCausalLM at Qwen3-0.6B architecture "
                   "(28 layers, 1024 hidden, 16q/8kv, head_dim 128, vocab 151936)",
                   "engine": f"the reference's Engine.run, Scheduler(max_batch={wl['max_batch']}), KVCacheManager, "
                             "BlockPool", "requests": wl["batch"],
                   "prompts": f"uniform {wl['prompt_lo']}..{wl['prompt_hi']}", "new_tokens": n_new,
                   "timing": "the engine's own DecodeBatchEnd events with TimingConfig(synchronize_device=True)"},
        "reference_sdpa_gpu": {"decode_tok_s": round(tok_s["sdpa"], 1),
                               "decode_model_forward_ms_per_step": res["sdpa"]["forward_s"] * 1e3 / max(n_new - 1, 1),
                               "path": "the reference's SDPAAttentionBackend and PagedKVCache (dense gather + pad + "
                                       "repeat_interleave + SDPA) on the same GPU"},
        "decode_model_forward_ms_per_step": res["cuda"]["forward_s"] * 1e3 / max(n_new - 1, 1),
        "speedup_over_reference_sdpa": round(tok_s["cuda"] / tok_s["sdpa"], 3),
        "greedy_streams": {"identical": f"{same} of {len(prompts)}",
                           "mean_tokens_before_first_difference": round(float(np.mean(first_div)), 1),
                           "note": "bf16 with random weights and a 151936-token vocabulary: a stream follows the "
                                   "other until the first step whose two best logits are within a few bf16 "
                                   "rounding steps (about 1 step in 20 here); the per-step agreement is checked "
                                   "teacher-forced in tests/test_gpu_e2e.py"},
        "e2e": {"value": round(tok_s["cuda"], 1), "unit": "tok/s", "h2d_bytes_per_step": 8 * wl["batch"],
                "d2h_bytes_per_step": 8 * wl["batch"],
                "path": "the reference's Engine.run with barellm_b200.PagedKVCache and the cuda backend"},
        "gpu_launches": None,
        "clocks": sampler.summary(),
    }
    print(json.dumps(out), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode_qwen8b_long")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pool-blocks", type=int, default=0,
                    help="override the KV pool size in blocks (smaller profiling captures)")
    ap.add_argument("--requests", type=int, default=0,
                    help="override the number of requests (smaller profiling captures)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.pool_blocks > 0 and ("pool_blocks" in wl or "pool_bytes" in wl):
        wl.pop("pool_bytes", None)
        wl["pool_blocks"] = args.pool_blocks
    if args.requests > 0 and "batch" in wl:
        wl["batch"] = args.requests
    if args.warmup < 3:
        args.warmup = 3
    kind = WORKLOADS[args.workload].get("kind")
    prefill = kind == "prefill"
    if kind == "e2e":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the end-to-end model workload has no CPU port "
                              "(the reference arm covers the decode and prefill kernels)"}))
            return
        run_e2e(args, args.workload)
        return
    if kind == "refengine":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "this workload's line already carries the "
                              "reference engine's own GPU run (reference_sdpa_gpu)"}))
            return
        run_refengine(args, args.workload)
        return
    if kind == "copy":
        (run_reference_copy if args.impl == "reference" else run_copy)(args, args.workload)
        return
    if kind == "heads":
        (run_reference if args.impl == "reference" else run_heads)(args, args.workload)
        return
    if args.impl == "reference":
        (run_reference_prefill if prefill else run_reference)(args, args.workload)
    else:
        (run_prefill if prefill else run_ours)(args, args.workload)


if __name__ == "__main__":
    main()
