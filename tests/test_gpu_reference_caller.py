"""The drop-in under the reference's own caller chain, on the GPU.

The reference's Engine (src/barellm/engine/engine.py:187-546: one-request
prefill, then batched decode over a BatchKVCache of every running request)
drives its own Qwen3ForCausalLM (src/barellm/models/qwen3.py:84-158), whose
GroupedQueryAttention.forward (src/barellm/models/attention.py:140-183) calls
``backend.attend`` for every layer.  Here that whole chain is the reference's
installed code; only the pieces the integration swaps in come from this
package:

* ``minimal``: the reference's Engine, Scheduler, KVCacheManager, BlockPool
  and BatchKVCache; this package's PagedKVCache and, under the backend name
  "cuda", CudaPagedAttentionBackend (the one edit in
  src/barellm/attention/backend.py:64-79 that registers it).
* ``swapped``: the integration's import swaps as well -- this package's
  BlockPool, KVCacheManager and BatchKVCache (src/barellm/runtime.py:14-59,
  src/barellm/engine/engine.py:467-469).

Both are compared with the same weights run entirely by the reference
("sdpa" backend, its own PagedKVCache): fp32 greedy tokens must be identical,
as the reference's own cached-vs-uncached contract requires
(tests/test_generate.py:230-288).  The weights are drawn so that the greedy
streams do not collapse to one repeated token (token embeddings with std 0.02,
projections with std 1/sqrt(fan_in)); the test asserts that too.

Skipped when the reference's installed copy (baseline/_ref) is absent.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF / "barellm" / "engine" / "engine.py").exists():
        pytest.skip("the reference's installed copy (baseline/_ref) is not present")
    if str(REF) not in sys.path:
        sys.path.append(str(REF))
    import barellm.engine.engine as engine_mod
    import barellm.models.attention as attention_mod
    from barellm.engine.block_pool import BlockPool
    from barellm.engine.kv_cache_manager import KVCacheManager
    from barellm.engine.paged_kv_cache import PagedKVCache
    from barellm.engine.request import Request
    from barellm.engine.scheduler import Scheduler
    from barellm.models.qwen3 import Qwen3ForCausalLM

    return dict(engine_mod=engine_mod, attention_mod=attention_mod, BlockPool=BlockPool,
                KVCacheManager=KVCacheManager, PagedKVCache=PagedKVCache, Request=Request, Scheduler=Scheduler,
                Qwen3ForCausalLM=Qwen3ForCausalLM)


SHAPE = dict(vocab_size=512, hidden_size=256, intermediate_size=512, head_dim=64, num_layers=3, num_heads=4,
             num_kv_heads=2)


def register_cuda_backend(monkeypatch, ref) -> None:
    """The integration's edit of create_attention_backend: the name "cuda"
    gives this package's backend, every other name the reference's."""
    from barellm_b200 import CudaPagedAttentionBackend

    original = ref["attention_mod"].create_attention_backend

    def create(name, *, sdpa=None):
        if name == "cuda":
            return CudaPagedAttentionBackend()
        return original(name, sdpa=sdpa)

    monkeypatch.setattr(ref["attention_mod"], "create_attention_backend", create)


def build_model(ref, backend: str, device):
    torch.manual_seed(0)
    m = ref["Qwen3ForCausalLM"](SHAPE["vocab_size"], SHAPE["hidden_size"], SHAPE["intermediate_size"],
                                SHAPE["head_dim"], SHAPE["num_layers"], SHAPE["num_heads"], SHAPE["num_kv_heads"],
                                use_qk_norm=True, attention_backend=backend)
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():
        for name, p in m.named_parameters():
            if "embed" in name:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            elif p.ndim == 2:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[1] ** 0.5)
    return m.to(device).eval()


def prompts(n: int, seed: int = 1) -> list[list[int]]:
    rs = np.random.RandomState(seed)
    return [[int(x) for x in rs.randint(0, SHAPE["vocab_size"], size=int(rs.randint(5, 70)))] for _ in range(n)]


def run_engine(ref, model, paged_kv_cache, block_pool, manager_cls, prompt_list, new_tokens, max_batch, device):
    manager = manager_cls(16, block_pool, paged_kv_cache)
    engine = ref["engine_mod"].Engine(model=model, scheduler=ref["Scheduler"](max_batch=max_batch),
                                      kv_cache_manager=manager)
    reqs = [ref["Request"](id=f"r{i}", token_ids=torch.tensor([p], dtype=torch.long, device=device),
                           temperature=0.0, max_new_tokens=new_tokens) for i, p in enumerate(prompt_list)]
    for r in reqs:
        engine.scheduler.add_request(r)
    engine.run()
    assert not engine.scheduler.has_work()
    return [r.token_ids[0, len(p):].tolist() for r, p in zip(reqs, prompt_list)]


def reference_tokens(ref, prompt_list, new_tokens, max_batch, device, blocks):
    model = build_model(ref, "sdpa", device)
    kv = ref["PagedKVCache"](SHAPE["num_layers"], blocks, SHAPE["num_kv_heads"], 16, SHAPE["head_dim"],
                             dtype=torch.float32, device=device)
    return run_engine(ref, model, kv, ref["BlockPool"](blocks), ref["KVCacheManager"], prompt_list, new_tokens,
                      max_batch, device)


@pytest.mark.parametrize("mode", ["minimal", "swapped"])
def test_reference_engine_and_model_on_the_cuda_backend(mode, ref, monkeypatch, cuda, native_lib):
    import barellm_b200 as bb

    device = cuda
    prompt_list = prompts(6)
    new_tokens = 16
    blocks = 64
    want = reference_tokens(ref, prompt_list, new_tokens, 4, device, blocks)
    assert all(len(set(t)) >= 4 for t in want), want  # the greedy streams are not degenerate

    register_cuda_backend(monkeypatch, ref)
    model = build_model(ref, "cuda", device)
    assert all(isinstance(layer.self_attn._backend, bb.CudaPagedAttentionBackend) for layer in model.layers)
    kv = bb.PagedKVCache(SHAPE["num_layers"], blocks, SHAPE["num_kv_heads"], 16, SHAPE["head_dim"],
                         dtype=torch.float32, device=device)
    if mode == "minimal":
        pool, manager_cls = ref["BlockPool"](blocks), ref["KVCacheManager"]
    else:
        monkeypatch.setattr(ref["engine_mod"], "BatchKVCache", bb.BatchKVCache)
        pool, manager_cls = bb.BlockPool(blocks), bb.KVCacheManager
    # max_batch 4 < 6 requests: the last two are admitted as the first finish
    got = run_engine(ref, model, kv, pool, manager_cls, prompt_list, new_tokens, 4, device)
    kv.check_device_errors()
    assert got == want
    # every request was freed back to the pool by the engine's cleanup
    assert len(pool.free_ids) == blocks and not kv.request_pages
