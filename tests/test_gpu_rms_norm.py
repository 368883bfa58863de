"""The decoder's one-kernel residual add + RMSNorm (bl_rms_norm) against the
tensor-op chain it replaces (src/barellm/models/norm.py:14-21 and the block's
residual add).

Bars: float32 within 1e-5 (relative); bf16 / fp16 equal except rare elements
one step away (the mean square's summation order differs), never more."""

from __future__ import annotations

import pytest
import torch

from barellm_b200 import ops

pytestmark = pytest.mark.gpu


def reference_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * w).to(x.dtype)


def assert_norm_close(got: torch.Tensor, want: torch.Tensor) -> None:
    if got.dtype == torch.float32:
        torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
        return
    g, w = got.float(), want.float()
    step = torch.finfo(got.dtype).eps * w.abs().clamp_min(torch.finfo(got.dtype).tiny)
    diff = (g - w).abs()
    assert bool((diff <= step * 1.0001).all()), float((diff / step).max())
    assert (diff > 0).float().mean().item() < 0.01


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hidden", [1024, 4096, 1000])
def test_rms_norm_matches_tensor_ops(cuda, native_lib, dtype, hidden):
    g = torch.Generator(device=cuda)
    g.manual_seed(hidden)
    x = torch.randn((3, 37, hidden), generator=g, device=cuda).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=cuda)).to(dtype)
    assert_norm_close(ops.rms_norm(x, w, 1e-6), reference_norm(x, w, 1e-6))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_add_rms_norm_matches_tensor_ops(cuda, native_lib, dtype):
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    x = torch.randn((128, 1, 1024), generator=g, device=cuda).to(dtype)
    r = torch.randn((128, 1, 1024), generator=g, device=cuda).to(dtype)
    w = (1 + 0.1 * torch.randn(1024, generator=g, device=cuda)).to(dtype)
    s, h = ops.rms_norm(x, w, 1e-6, residual=r)
    assert torch.equal(s, x + r)  # the add is a rounded tensor add, bit for bit
    assert_norm_close(h, reference_norm(x + r, w, 1e-6))


def test_rms_norm_strided_rows(cuda, native_lib):
    """Rows taken from a wider tensor (every other row of a [2R, H] buffer)."""
    g = torch.Generator(device=cuda)
    g.manual_seed(2)
    big = torch.randn((64, 1024), generator=g, device=cuda).to(torch.bfloat16)
    x = big[::2]
    w = torch.ones(1024, dtype=torch.bfloat16, device=cuda)
    assert_norm_close(ops.rms_norm(x, w, 1e-6), reference_norm(x, w, 1e-6))


def test_rms_norm_rejects_bad_weight(cuda, native_lib):
    x = torch.zeros((4, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError):
        ops.rms_norm(x, torch.ones(32, dtype=torch.bfloat16, device=cuda), 1e-6)
