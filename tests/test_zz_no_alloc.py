"""bl_paged_decode_noalloc: the decode entry point for callers that cannot
give the library device scratch (a host framework that owns all device memory
and passes only input/output pointers, or a decode loop that must stay clear
of cudaMalloc).  Its split-K scratch is a fixed 16 MiB array inside the
library, shared by every call.

The test calls it through the C ABI twice in a row, with different batches.
Both entry points run the same plan, attention and reduce kernels over the
same deterministic split, so each result must equal the regular entry point's
(bl_paged_decode with a caller workspace) bit for bit; it is also checked
against the float64 oracle within the bf16 parity tolerance used everywhere
else.  It lives in a file of its own, collected last, and needs no state from
the other tests."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cases
import gpu_helpers as gh
from barellm_b200 import ops

pytestmark = pytest.mark.gpu

BF16_MAX, BF16_MEAN = 2e-2, 2e-3


def _compare_oracle(out: torch.Tensor, st: gh.DecodeState) -> None:
    from oracle import paged_oracle as orc

    got = out.float().cpu().numpy()
    want = orc.decode_attention(st.q.float().cpu().numpy(), st.k_cache.float().cpu().numpy(),
                                st.v_cache.float().cpu().numpy(), 0, st.tables, st.seq_lens_list)[:, :, 0]
    err = np.abs(got - want)
    assert np.isfinite(got).all()
    assert err.max() <= BF16_MAX and err.mean() <= BF16_MEAN, (float(err.max()), float(err.mean()))


def test_noalloc_decode_matches_workspace_decode_two_calls(cuda, native_lib):
    # two different batches, both long enough to need split-K (several chunks)
    first = gh.DecodeState(cases.make_decode_case(101, 16, 32, 8, 128, 16, 4096, 600, 3000), torch.bfloat16, cuda)
    second = gh.DecodeState(cases.make_decode_case(102, 24, 16, 8, 128, 16, 4096, 50, 2500), torch.bfloat16, cuda)
    for st in (first, second):
        expected = st.decode()  # bl_paged_decode with a torch-owned workspace
        out = torch.empty_like(expected)
        ops.paged_decode_noalloc(st.q, st.k_cache, st.v_cache, 0, st.bt, st.seq_lens, max(st.seq_lens_list), out,
                                 err=st.err)
        torch.cuda.synchronize()
        assert int(st.err.item()) == 0
        assert torch.equal(out, expected)
        _compare_oracle(out, st)


def test_noalloc_decode_rejects_batches_beyond_its_scratch(cuda, native_lib):
    # 256 rows x 32k tokens x 32 heads needs far more than 16 MiB of split-K scratch
    kc = torch.zeros((1, 8, 8, 16, 128), dtype=torch.bfloat16, device=cuda)
    bt = torch.zeros((256, 2048), dtype=torch.int32, device=cuda)
    q = torch.zeros((256, 32, 128), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="built-in scratch"):
        ops.paged_decode_noalloc(q, kc, kc.clone(), 0, bt, torch.ones(256, dtype=torch.int32, device=cuda), 32768,
                                 torch.empty_like(q))
