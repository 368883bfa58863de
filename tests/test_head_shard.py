"""KV-head-sharded decode: the heads of one decode batch split across GPUs,
the per-head outputs all-gathered by the decode kernels' own stores into every
rank's buffer (bl_paged_decode_allgather).

CPU: the head partition (ranges cover every head once, query heads follow
their KV head) and, on two gloo ranks, that per-rank oracle decodes of the
shards reassemble the full decode through the collective gather.
GPU, one device: world 1 equals bl_paged_decode bit for bit; two ranks
emulated in sequence on one device (each call's wait is already satisfied
when it is launched) fill both gathered buffers; a barrier whose peer never
signals runs out and sets BL_DEVERR_TIMEOUT.  GPU, two devices: two
processes over NCCL, three calls in a row, bit-exact against the unsharded
decode and equal to the NCCL all-gather baseline."""

from __future__ import annotations

import ctypes
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import cases
from barellm_b200 import _native as nat
from barellm_b200 import head_shard as hs
from barellm_b200 import ops


# --------------------------------------------------------------------------
# partition (CPU)
# --------------------------------------------------------------------------
@pytest.mark.parametrize("hq,hkv", [(16, 8), (32, 8), (8, 8), (8, 2)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_ranges_cover_every_head_once(hq, hkv, world):
    if hkv % world:
        with pytest.raises(ValueError, match="divide evenly"):
            hs.kv_head_range(hkv, world, 0)
        return
    g = hq // hkv
    kv = [hs.kv_head_range(hkv, world, r) for r in range(world)]
    qh = [hs.q_head_range(hq, hkv, world, r) for r in range(world)]
    assert [h for lo, hi in kv for h in range(lo, hi)] == list(range(hkv))
    assert [h for lo, hi in qh for h in range(lo, hi)] == list(range(hq))
    for (k0, k1), (q0, q1) in zip(kv, qh):
        # query head h reads KV head h // G (repeat_interleave grouping)
        assert {h // g for h in range(q0, q1)} == set(range(k0, k1))


def test_head_ranges_reject_bad_worlds():
    with pytest.raises(ValueError):
        hs.kv_head_range(8, 0, 0)
    with pytest.raises(ValueError):
        hs.kv_head_range(8, 2, 2)
    with pytest.raises(ValueError):
        hs.kv_head_range(16, 16, 0)  # beyond BL_MAX_RANKS
    with pytest.raises(ValueError, match="num_heads must divide evenly"):
        hs.q_head_range(12, 8, 2, 0)


def test_head_sharded_decode_rejects_bad_arguments_before_touching_a_device():
    with pytest.raises(ValueError, match="two buffers"):
        hs.HeadShardedDecode(2, 16, 8, 128, torch.bfloat16, torch.device("cpu"), buffers=1)
    with pytest.raises(ValueError, match="unsupported dtype"):
        hs.HeadShardedDecode(2, 16, 8, 128, torch.int32, torch.device("cpu"))
    with pytest.raises(ValueError, match="num_heads must divide evenly"):
        hs.HeadShardedDecode(2, 12, 8, 128, torch.bfloat16, torch.device("cpu"))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dense_rows(case):
    k_rows = [np.concatenate([case.k_hist[b][0], case.k_new[b][:, :1]], axis=1) for b in range(case.batch)]
    v_rows = [np.concatenate([case.v_hist[b][0], case.v_new[b][:, :1]], axis=1) for b in range(case.batch)]
    return k_rows, v_rows


def _gloo_worker(rank: int, world: int, port: int, out) -> None:
    from oracle import paged_oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        case = cases.decode_case("decode_qwen06b_b4")
        k_rows, v_rows = _dense_rows(case)
        k0, k1 = hs.kv_head_range(case.num_kv_heads, world, rank)
        q0, q1 = hs.q_head_range(case.num_q_heads, case.num_kv_heads, world, rank)
        q = case.q[:, :, 0]
        local = orc.decode_attention_rows(q[:, q0:q1], [k[k0:k1] for k in k_rows], [v[k0:k1] for v in v_rows])
        gathered = hs.gather_heads_collective(torch.from_numpy(local))
        out.put((rank, gathered.numpy()))
    finally:
        dist.destroy_process_group()


def test_head_shards_reassemble_the_full_decode_on_two_gloo_ranks():
    from oracle import paged_oracle as orc

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    case = cases.decode_case("decode_qwen06b_b4")
    k_rows, v_rows = _dense_rows(case)
    full = orc.decode_attention_rows(case.q[:, :, 0], k_rows, v_rows)
    for r in range(world):
        np.testing.assert_allclose(results[r], full, rtol=0, atol=1e-12)


def test_allgather_argument_errors_before_any_launch(native_lib):
    a = nat.DecodeArgs()
    g = nat.HeadGather()
    assert native_lib.bl_paged_decode_allgather(ctypes.byref(a), ctypes.byref(g), None) == nat.BL_ERR_ARG
    assert "world" in nat.last_error()
    g.world, g.rank, g.epoch = 2, 0, 256
    assert native_lib.bl_paged_decode_allgather(ctypes.byref(a), ctypes.byref(g), None) == nat.BL_ERR_ARG
    assert "null gathered buffer" in nat.last_error()
    g.rank = 2
    assert native_lib.bl_paged_decode_allgather(ctypes.byref(a), ctypes.byref(g), None) == nat.BL_ERR_ARG
    assert "rank 2 outside" in nat.last_error()
    assert native_lib.bl_ipc_export(None, ctypes.byref(nat.IpcHandle())) == nat.BL_ERR_ARG
    assert native_lib.bl_ipc_close(ctypes.c_void_p(4096)) == nat.BL_ERR_ARG
    assert "not returned by bl_ipc_import" in nat.last_error()


# --------------------------------------------------------------------------
# one GPU
# --------------------------------------------------------------------------
def _state(name, dtype, device):
    import gpu_helpers as gh

    return gh.DecodeState(cases.decode_case(name), dtype, device)


def _shard(st, world, rank):
    c = st.case
    k0, k1 = hs.kv_head_range(c.num_kv_heads, world, rank)
    q0, q1 = hs.q_head_range(c.num_q_heads, c.num_kv_heads, world, rank)
    return (st.k_cache[:, :, k0:k1].contiguous(), st.v_cache[:, :, k0:k1].contiguous(), st.q[:, q0:q1], (q0, q1))


@pytest.mark.gpu
@pytest.mark.parametrize("name,dtype", [("decode_qwen8b_b3", torch.bfloat16), ("decode_qwen06b_b4", torch.float16),
                                        ("decode_tiny_gqa", torch.float32)])
def test_world1_equals_decode_bit_for_bit(cuda, native_lib, name, dtype):
    st = _state(name, dtype, cuda)
    c = st.case
    ref = st.decode()
    h = hs.HeadShardedDecode(c.batch, c.num_q_heads, c.num_kv_heads, c.head_dim, dtype, cuda)
    for _ in range(3):  # the buffers alternate; the epoch counts up
        out = h.decode(st.q, st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list), err=st.err)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    assert int(st.err.item()) == 0
    assert int(h.region[256:260].view(torch.int32).item()) == 3
    h.close()


@pytest.mark.gpu
def test_own_error_word_reports_a_bad_block_id(cuda, native_lib):
    """Without a caller error word the object's own word receives the
    kernels' error bits; check_device_errors (and close) raise on it."""
    st = _state("decode_qwen06b_b4", torch.bfloat16, cuda)
    c = st.case
    bt = st.bt.clone()
    bt[0, 0] = c.num_blocks + 5  # flagged by the kernel, the access skipped
    h = hs.HeadShardedDecode(c.batch, c.num_q_heads, c.num_kv_heads, c.head_dim, torch.bfloat16, cuda)
    h.decode(st.q, st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
    h.check_device_errors()  # a clean call leaves the word clear
    h.decode(st.q, st.k_cache, st.v_cache, 0, bt, st.seq_lens, max(st.seq_lens_list))
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        h.check_device_errors()
    with pytest.raises(RuntimeError, match="block id outside the pool"):
        h.close()
    assert h._closed


class _EmulatedRanks:
    """Two ranks' regions (signal pad, epoch, gathered buffer) on one device."""

    def __init__(self, st, device):
        c = st.case
        self.elems = c.batch * c.num_q_heads * c.head_dim
        esz = st.q.element_size()
        self.regions = [torch.zeros(512 + self.elems * esz, dtype=torch.uint8, device=device) for _ in range(2)]
        self.outs = [r[512:].view(st.q.dtype).view(c.batch, c.num_q_heads, c.head_dim) for r in self.regions]

    def pad(self, r):
        return self.regions[r][:32].view(torch.int32)

    def epoch(self, r):
        return int(self.regions[r][256:260].view(torch.int32).item())

    def gather(self, rank, head_offset, timeout_ns=0):
        g = nat.HeadGather()
        g.world, g.rank = 2, rank
        for r in range(2):
            g.peer_out[r] = self.regions[r].data_ptr() + 512
            g.peer_signal[r] = self.regions[r].data_ptr()
        g.epoch = self.regions[rank].data_ptr() + 256
        g.head_offset = head_offset
        g.timeout_ns = timeout_ns
        return g


def _call(native_lib, st, shard, g, gathered):
    # ``gathered`` gives the strides of the [B, Hq, D] buffers (the pointer
    # itself is not used: the outputs go to g.peer_out)
    k, v, q, (q0, q1) = shard
    a, _, _ = ops._decode_args(q, k, v, 0, st.bt, st.seq_lens, max(st.seq_lens_list), None, gathered[:, q0:q1],
                               None, None, False, st.err)
    rc = native_lib.bl_paged_decode_allgather(ctypes.byref(a), ctypes.byref(g), ops._stream(q.device))
    assert rc == nat.BL_OK, nat.last_error()


@pytest.mark.gpu
def test_two_ranks_emulated_in_sequence_fill_both_gathered_buffers(cuda, native_lib):
    st = _state("decode_qwen8b_b3", torch.bfloat16, cuda)
    ref = st.decode()
    em = _EmulatedRanks(st, cuda)
    shards = [_shard(st, 2, r) for r in range(2)]
    for step in (1, 2):
        # rank 0 runs first, so rank 1's announcement for this epoch is
        # written ahead of time; rank 1 then finds rank 0's already there
        em.pad(0)[1] = step
        _call(native_lib, st, shards[0], em.gather(0, shards[0][3][0]), em.outs[0])
        torch.cuda.synchronize()
        assert int(em.pad(1)[0].item()) == step and em.epoch(0) == step
        q0, q1 = shards[0][3]
        for r in range(2):  # rank 0's heads are in both buffers already
            assert torch.equal(em.outs[r][:, q0:q1], ref[:, q0:q1])
        _call(native_lib, st, shards[1], em.gather(1, shards[1][3][0]), em.outs[1])
        torch.cuda.synchronize()
        assert em.epoch(1) == step
        for r in range(2):
            assert torch.equal(em.outs[r], ref)
        em.outs[0].zero_()
        em.outs[1].zero_()
    assert int(st.err.item()) == 0


@pytest.mark.gpu
def test_barrier_whose_peer_never_signals_times_out(cuda, native_lib):
    st = _state("decode_qwen06b_b4", torch.bfloat16, cuda)
    ref = st.decode()
    em = _EmulatedRanks(st, cuda)
    shard = _shard(st, 2, 0)
    _call(native_lib, st, shard, em.gather(0, 0, timeout_ns=20_000_000), em.outs[0])  # nothing writes pad 0 slot 1
    torch.cuda.synchronize()
    assert int(st.err.item()) & nat.BL_DEVERR_TIMEOUT
    # the kernel returned; the context still works
    st.err.zero_()
    assert torch.equal(st.decode(), ref)
    assert int(st.err.item()) == 0


# --------------------------------------------------------------------------
# two GPUs
# --------------------------------------------------------------------------
def _two_gpu_worker(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    h = None
    try:
        st = _state("decode_qwen8b_b3", torch.bfloat16, dev)
        c = st.case
        k, v, _, (q0, q1) = _shard(st, world, rank)
        h = hs.HeadShardedDecode(c.batch, c.num_q_heads, c.num_kv_heads, c.head_dim, torch.bfloat16, dev)
        res = []
        for it in range(3):
            q = (st.q.float() * (1.0 + 0.5 * it)).to(torch.bfloat16)
            ref = ops.paged_decode(q, st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
            got = h.decode(q[:, q0:q1], k, v, 0, st.bt, st.seq_lens, max(st.seq_lens_list), err=st.err)
            torch.cuda.synchronize()
            got = got.clone()
            local = ops.paged_decode(q[:, q0:q1], k, v, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
            coll = hs.gather_heads_collective(local)
            torch.cuda.synchronize()
            res.append((bool(torch.equal(got, ref)), bool(torch.equal(coll, ref)),
                        float((got.float() - ref.float()).abs().max())))
        out.put((rank, res, int(st.err.item())))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out.put((rank, repr(e), -1))
    finally:
        if h is not None:
            h.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_fused_gather_equals_unsharded_decode():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (res, err)) for r, res, err in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        res, err = results[r]
        assert err == 0, res
        for fused_ok, coll_ok, diff in res:
            assert fused_ok and coll_ok, (r, res)


def _two_objects_worker(rank: int, world: int, port: int, out) -> None:
    """Two HeadShardedDecode objects alive at once in each process (their
    regions may share one allocation, so their peer mappings are shared);
    closing the first must leave the second's mappings intact."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    first = second = None
    try:
        st = _state("decode_qwen8b_b3", torch.bfloat16, dev)
        c = st.case
        k, v, _, (q0, q1) = _shard(st, world, rank)
        first = hs.HeadShardedDecode(c.batch, c.num_q_heads, c.num_kv_heads, c.head_dim, torch.bfloat16, dev)
        second = hs.HeadShardedDecode(c.batch, c.num_q_heads, c.num_kv_heads, c.head_dim, torch.bfloat16, dev)
        ref = ops.paged_decode(st.q, st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
        a = first.decode(st.q[:, q0:q1], k, v, 0, st.bt, st.seq_lens, max(st.seq_lens_list)).clone()
        first.close()
        res = [bool(torch.equal(a, ref))]
        for _ in range(3):
            b = second.decode(st.q[:, q0:q1], k, v, 0, st.bt, st.seq_lens, max(st.seq_lens_list))
            torch.cuda.synchronize()
            res.append(bool(torch.equal(b, ref)))
        second.check_device_errors()
        out.put((rank, res, 0))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out.put((rank, repr(e), -1))
    finally:
        for h in (first, second):
            if h is not None and not h._closed:
                h.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_gpus_two_objects_share_peer_mappings():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_objects_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (res, err)) for r, res, err in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        res, err = results[r]
        assert err == 0 and all(res), (r, res)
