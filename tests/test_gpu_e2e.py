"""End to end on the GPU: a Qwen3 decoder driven through the paged engine
(CUDA append / prefill / decode kernels behind CudaPagedAttentionBackend)
against the same weights on the contiguous-cache SDPA oracle.

fp32: greedy tokens identical (the reference checks cached vs uncached and
batched vs independent decodes at 1e-5: tests/test_generate.py:230-288,
tests/test_batched_kv_cache.py:92-150).  bf16: identical up to the first
divergence, and a divergence may only happen where the oracle's top-2 logits
are a near-tie (bf16 logits round at ~1e-2 here)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from barellm_b200.engine import PagedEngine, Qwen3Shape, random_qwen3
from oracle.contiguous_engine import generate_contiguous

pytestmark = pytest.mark.gpu


def prompts_for(n: int, lo: int, hi: int, vocab: int, seed: int) -> list[list[int]]:
    rs = np.random.RandomState(seed)
    return [list(rs.randint(0, vocab, size=rs.randint(lo, hi + 1))) for _ in range(n)]


def test_fp32_paged_engine_matches_contiguous_oracle_exactly(cuda, native_lib):
    shape = Qwen3Shape(vocab_size=512, hidden_size=256, intermediate_size=512, head_dim=64, num_layers=3,
                       num_heads=4, num_kv_heads=2)
    model = random_qwen3(shape, dtype=torch.float32, device=cuda, seed=0)
    prompts = prompts_for(6, 5, 60, shape.vocab_size, seed=1)
    engine = PagedEngine(model, num_blocks=PagedEngine.blocks_needed([len(p) for p in prompts], 12, 16) + 4)
    got = engine.generate(prompts, max_new_tokens=12)
    want, _ = generate_contiguous(model, prompts, 12)
    assert got == want


def test_graph_decode_matches_eager_decode(cuda, native_lib):
    """The CUDA-graph decode loop replays exactly what the eager loop runs."""
    shape = Qwen3Shape(vocab_size=1024, num_layers=3)
    model = random_qwen3(shape, dtype=torch.bfloat16, device=cuda, seed=11)
    prompts = prompts_for(5, 10, 200, shape.vocab_size, seed=12)
    blocks = PagedEngine.blocks_needed([len(p) for p in prompts], 20, 16) + 4
    eager = PagedEngine(model, num_blocks=blocks).generate(prompts, 20, use_graph=False)
    graph = PagedEngine(model, num_blocks=blocks).generate(prompts, 20, use_graph=True)
    assert eager == graph


def test_fp32_uncached_recompute_matches_cached_decode(cuda, native_lib):
    """The reference's cached-vs-uncached greedy identity, with every forward
    (uncached: the full sequence each step) through the CUDA backend."""
    shape = Qwen3Shape(vocab_size=256, hidden_size=128, intermediate_size=256, head_dim=64, num_layers=2,
                       num_heads=4, num_kv_heads=1)
    model = random_qwen3(shape, dtype=torch.float32, device=cuda, seed=3)
    prompt = prompts_for(1, 9, 9, shape.vocab_size, seed=4)[0]
    engine = PagedEngine(model, num_blocks=8)
    cached = engine.generate([prompt], max_new_tokens=8)[0]
    toks = list(prompt)
    with torch.inference_mode():
        for _ in range(8):
            ids = torch.tensor([toks], device=cuda)
            pos = torch.arange(len(toks), device=cuda).unsqueeze(0)
            toks.append(int(torch.argmax(model(ids, pos, kv_cache=None)[0, -1]).item()))
    assert cached == toks[len(prompt):]


def test_bf16_qwen06b_attention_shapes_match_up_to_near_ties(cuda, native_lib):
    shape = Qwen3Shape(vocab_size=2048, num_layers=4)  # Qwen3-0.6B attention/MLP widths, fewer layers
    model = random_qwen3(shape, dtype=torch.bfloat16, device=cuda, seed=5)
    prompts = prompts_for(8, 20, 300, shape.vocab_size, seed=6)
    n_new = 24
    engine = PagedEngine(model, num_blocks=PagedEngine.blocks_needed([len(p) for p in prompts], n_new, 16) + 4)
    got = engine.generate(prompts, max_new_tokens=n_new)
    want, margins = generate_contiguous(model, prompts, n_new, record_margins=True)
    identical = 0
    for g, w, m in zip(got, want, margins):
        if g == w:
            identical += 1
            continue
        k = next(i for i, (a, b) in enumerate(zip(g, w)) if a != b)
        assert m[k] < 0.25, f"divergence at step {k} with oracle top-2 margin {m[k]:.3f}"
    assert identical >= len(prompts) // 2


def test_fp32_packed_chunked_prefill_matches_per_request_prefill(cuda, native_lib):
    """Batched prefill with a small token budget (prompts packed together and
    long prompts split into chunks over their cached earlier chunks) gives the
    same greedy tokens as one-request-per-forward prefill and as the
    contiguous-cache oracle."""
    shape = Qwen3Shape(vocab_size=512, hidden_size=256, intermediate_size=512, head_dim=64, num_layers=3,
                       num_heads=4, num_kv_heads=2)
    model = random_qwen3(shape, dtype=torch.float32, device=cuda, seed=21)
    prompts = prompts_for(7, 3, 90, shape.vocab_size, seed=22)
    blocks = PagedEngine.blocks_needed([len(p) for p in prompts], 10, 16) + 4
    packed = PagedEngine(model, num_blocks=blocks, prefill_tokens=48).generate(prompts, max_new_tokens=10)
    single = PagedEngine(model, num_blocks=blocks, prefill_tokens=0).generate(prompts, max_new_tokens=10)
    want, _ = generate_contiguous(model, prompts, 10)
    assert packed == single == want
