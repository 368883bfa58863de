"""Contiguous-cache SDPA engine: the end-to-end oracle.  TEST INFRASTRUCTURE ONLY.

Restates, in torch, the reference's contiguous-cache decode path that the
greedy-token comparison is made against:
  * ContiguousLayerKV / ContiguousKVCache (src/barellm/engine/contiguous_kv_cache.py:6-65):
    ``torch.cat`` along the token axis;
  * BatchLayerKV over contiguous members (src/barellm/engine/batched_kv_cache.py:40-102):
    per-row append, zero-padded read, boolean valid-key mask;
  * SDPAAttentionBackend.attend (src/barellm/attention/backend.py:34-61):
    repeat_interleave(G) + scaled_dot_product_attention, ``is_causal`` only
    when there is no mask and more than one query.
It drives the same ``barellm_b200.engine.Qwen3`` module (same weights), so two
runs differ only in the attention backend and cache.  Only tests may use it.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


class ContiguousLayerKV:
    def __init__(self) -> None:
        self.key: torch.Tensor | None = None
        self.value: torch.Tensor | None = None

    @property
    def seq_len(self) -> int:
        return 0 if self.key is None else self.key.shape[2]

    def append_only(self, key: torch.Tensor, value: torch.Tensor) -> None:
        if self.key is None:
            self.key, self.value = key, value
        else:
            self.key = torch.cat([self.key, key], dim=2)
            self.value = torch.cat([self.value, value], dim=2)

    def read(self):
        return self.key, self.value


class ContiguousKVCache:
    def __init__(self, num_layers: int) -> None:
        self.layers = [ContiguousLayerKV() for _ in range(num_layers)]

    def layer(self, i: int) -> ContiguousLayerKV:
        return self.layers[i]


class BatchContiguousLayer:
    def __init__(self, members: list[ContiguousLayerKV]) -> None:
        self.members = members


class BatchContiguous:
    def __init__(self, caches: list[ContiguousKVCache]) -> None:
        self.caches = caches

    def layer(self, i: int) -> BatchContiguousLayer:
        return BatchContiguousLayer([c.layer(i) for c in self.caches])


class SDPAContiguousBackend:
    def attend(self, q, new_k, new_v, layer_cache, group_size):
        if isinstance(layer_cache, BatchContiguousLayer):
            for row, m in enumerate(layer_cache.members):
                m.append_only(new_k[row : row + 1], new_v[row : row + 1])
            lens = [m.seq_len for m in layer_cache.members]
            tmax = max(lens)
            b, h, _, d = new_k.shape
            key = torch.zeros((b, h, tmax, d), dtype=new_k.dtype, device=new_k.device)
            value = torch.zeros_like(key)
            for row, m in enumerate(layer_cache.members):
                key[row, :, : lens[row]] = m.key[0]
                value[row, :, : lens[row]] = m.value[0]
            lt = torch.tensor(lens, device=new_k.device)
            mask = (torch.arange(tmax, device=new_k.device)[None, :] < lt[:, None])[:, None, None, :]
            mask = mask.expand(-1, 1, q.shape[2], -1)
        else:
            if layer_cache is None:
                key, value = new_k, new_v
            else:
                layer_cache.append_only(new_k, new_v)
                key, value = layer_cache.read()
            mask = None
        key = key.repeat_interleave(group_size, dim=1)
        value = value.repeat_interleave(group_size, dim=1)
        return F.scaled_dot_product_attention(q, key, value, attn_mask=mask, is_causal=mask is None and q.shape[2] > 1)


def _spacing(x: float, dtype: torch.dtype) -> float:
    """The gap between adjacent representable values of ``dtype`` at |x|
    (the logits' rounding step); 0 for float32, where margins stay absolute."""
    mant = {torch.bfloat16: 7, torch.float16: 10}.get(dtype)
    if mant is None:
        return 0.0
    return 2.0 ** (math.floor(math.log2(max(abs(x), 2.0 ** -14))) - mant)


@torch.inference_mode()
def generate_contiguous(model, prompts: list[list[int]], max_new_tokens: int, record_margins: bool = False):
    """Per-request prefill, then batched greedy decode, over contiguous caches.
    Returns (new tokens per request, top-2 logit margins per step per request);
    with 16-bit logits a margin is counted in rounding steps of the top logit
    (2 means the two best logits are two representable values apart)."""
    dev = next(model.parameters()).device
    saved = model.backend
    model.set_backend(SDPAContiguousBackend())
    try:
        caches = [ContiguousKVCache(len(model.layers)) for _ in prompts]
        toks = [list(p) for p in prompts]
        margins: list[list[float]] = [[] for _ in prompts]

        def pick(logits_row):
            if record_margins:
                # top-2 margin in units of the logits' rounding step at the top
                # value (16-bit logits), or absolute (float32 logits)
                top = torch.topk(logits_row.float(), 2).values
                gap = float(top[0] - top[1])
                step = _spacing(float(top[0]), logits_row.dtype)
                return int(torch.argmax(logits_row).item()), (gap / step if step > 0 else gap)
            return int(torch.argmax(logits_row).item()), 0.0

        for i, c in enumerate(caches):
            ids = torch.tensor([toks[i]], dtype=torch.long, device=dev)
            pos = torch.arange(len(toks[i]), device=dev).unsqueeze(0)
            logits = model(ids, pos, kv_cache=c)
            t, m = pick(logits[0, -1])
            toks[i].append(t)
            margins[i].append(m)
        for _ in range(max_new_tokens - 1):
            ids = torch.tensor([[t[-1]] for t in toks], dtype=torch.long, device=dev)
            pos = torch.tensor([[len(t) - 1] for t in toks], dtype=torch.long, device=dev)
            logits = model(ids, pos, kv_cache=BatchContiguous(caches))
            for i in range(len(toks)):
                t, m = pick(logits[i, -1])
                toks[i].append(t)
                margins[i].append(m)
        return [t[len(p):] for t, p in zip(toks, prompts)], margins
    finally:
        model.set_backend(saved)
