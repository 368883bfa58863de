"""The callers of the paged-KV path: a Qwen3 decoder and a batched engine loop.

This is the harness that drives the path end to end (prefill every request,
then batched greedy decode), the way the reference's Engine does
(src/barellm/engine/engine.py:187-546) over its Qwen3 model
(src/barellm/models/qwen3.py, block.py, attention.py, rope.py, norm.py,
mlp.py, embedding.py).  The model math follows the reference exactly --
pre-norm blocks, QK-RMSNorm before half-split RoPE, GQA attention through an
``AttentionBackend``, SwiGLU, tied LM head -- so that two runs of the same
weights differ only in the attention backend and cache.  Weights are random
(no checkpoint is needed to measure the path).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F
from torch import nn

from . import ops
from .backend import CudaPagedAttentionBackend
from .batched_kv_cache import BatchKVCache, PackedBatchKVCache
from .block_pool import BlockPool
from .kv_cache_manager import KVCacheManager
from .paged_kv_cache import PagedKVCache


@dataclass(frozen=True)
class Qwen3Shape:
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    head_dim: int = 128
    num_layers: int = 28
    num_heads: int = 16
    num_kv_heads: int = 8
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6


QWEN3_06B = Qwen3Shape()


def _fused_norm_ok(x: torch.Tensor) -> bool:
    """bf16 / fp16 activations on a CUDA device take the one-kernel norm; fp32
    keeps the tensor-op chain (the exact-match reference runs are fp32)."""
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and x.stride(-1) == 1


class RMSNorm(nn.Module):
    """fp32 mean-square normalisation, weight applied in fp32, cast back (norm.py)."""

    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _fused_norm_ok(x):
            return ops.rms_norm(x, self.weight, self.eps)
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (xf * self.weight).to(x.dtype)

    def add_forward(self, x: torch.Tensor, residual: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """``(x + residual, norm(x + residual))``: one kernel for 16-bit CUDA
        activations."""
        if _fused_norm_ok(x) and residual.stride(-1) == 1:
            return ops.rms_norm(x, self.weight, self.eps, residual=residual)
        y = x + residual
        return y, self(y)


def rope_cos_sin(head_dim: int, theta: float, position_ids: torch.Tensor, dtype: torch.dtype):
    """Half-split RoPE tables [B, 1, T, D] in the activation dtype (rope.py:25-50)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=position_ids.device) / head_dim))
    angles = position_ids.to(torch.float32)[..., None] * inv_freq
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().unsqueeze(1).to(dtype), angles.sin().unsqueeze(1).to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


class Attention(nn.Module):
    def __init__(self, s: Qwen3Shape, backend) -> None:
        super().__init__()
        self.s = s
        self.q_proj = nn.Linear(s.hidden_size, s.num_heads * s.head_dim, bias=False)
        self.k_proj = nn.Linear(s.hidden_size, s.num_kv_heads * s.head_dim, bias=False)
        self.v_proj = nn.Linear(s.hidden_size, s.num_kv_heads * s.head_dim, bias=False)
        self.o_proj = nn.Linear(s.num_heads * s.head_dim, s.hidden_size, bias=False)
        self.q_norm = RMSNorm(s.head_dim, s.rms_norm_eps)
        self.k_norm = RMSNorm(s.head_dim, s.rms_norm_eps)
        self.backend = backend
        self.fused_prep = True  # QK-norm + RoPE + append in one kernel when the cache is paged
        self._qkv: torch.Tensor | None = None  # [q; k; v] weights, the three projections are views into it

    def fuse_projections(self) -> None:
        """One [q; k; v] weight matrix (one GEMM per forward instead of three);
        q_proj / k_proj / v_proj keep their parameters as views into it."""
        w = torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight]).detach()
        nq, nk = self.q_proj.weight.shape[0], self.k_proj.weight.shape[0]
        self.q_proj.weight = nn.Parameter(w[:nq], requires_grad=False)
        self.k_proj.weight = nn.Parameter(w[nq : nq + nk], requires_grad=False)
        self.v_proj.weight = nn.Parameter(w[nq + nk :], requires_grad=False)
        self._qkv = w

    def _projections(self, x: torch.Tensor):
        b, t, _ = x.shape
        s = self.s
        nq, nk = s.num_heads * s.head_dim, s.num_kv_heads * s.head_dim
        w = self._qkv
        if w is not None and w.data_ptr() == self.q_proj.weight.data_ptr() and w.dtype == x.dtype:
            qkv = F.linear(x, w)
            q = qkv[..., :nq].view(b, t, s.num_heads, s.head_dim)
            k = qkv[..., nq : nq + nk].view(b, t, s.num_kv_heads, s.head_dim)
            v = qkv[..., nq + nk :].view(b, t, s.num_kv_heads, s.head_dim)
        else:
            q = self.q_proj(x).view(b, t, s.num_heads, s.head_dim)
            k = self.k_proj(x).view(b, t, s.num_kv_heads, s.head_dim)
            v = self.v_proj(x).view(b, t, s.num_kv_heads, s.head_dim)
        return q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)

    def forward(self, x, cos, sin, layer_cache) -> torch.Tensor:
        b, t, _ = x.shape
        s = self.s
        q, k, v = self._projections(x)
        group = s.num_heads // s.num_kv_heads
        prepped = getattr(self.backend, "attend_prepped", None)
        if self.fused_prep and prepped is not None and layer_cache is not None:
            # QK-norm + RoPE fused with the paged append (one kernel)
            ctx = prepped(q, k, v, self.q_norm.weight, self.k_norm.weight, self.q_norm.eps, cos, sin, layer_cache,
                          group)
        else:
            q = apply_rope(self.q_norm(q), cos, sin)
            k = apply_rope(self.k_norm(k), cos, sin)
            ctx = self.backend.attend(q, k, v, layer_cache, group)
        return self.o_proj(ctx.transpose(1, 2).reshape(b, t, -1))


class Block(nn.Module):
    def __init__(self, s: Qwen3Shape, backend) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(s.hidden_size, s.rms_norm_eps)
        self.self_attn = Attention(s, backend)
        self.post_attention_layernorm = RMSNorm(s.hidden_size, s.rms_norm_eps)
        self.gate_proj = nn.Linear(s.hidden_size, s.intermediate_size, bias=False)
        self.up_proj = nn.Linear(s.hidden_size, s.intermediate_size, bias=False)
        self.down_proj = nn.Linear(s.intermediate_size, s.hidden_size, bias=False)
        self._gate_up: torch.Tensor | None = None  # [gate; up] weights, the two projections are views into it

    def fuse_projections(self) -> None:
        """One [gate; up] weight matrix (one GEMM instead of two) and the
        attention's fused [q; k; v]."""
        w = torch.cat([self.gate_proj.weight, self.up_proj.weight]).detach()
        n = self.gate_proj.weight.shape[0]
        self.gate_proj.weight = nn.Parameter(w[:n], requires_grad=False)
        self.up_proj.weight = nn.Parameter(w[n:], requires_grad=False)
        self._gate_up = w
        self.self_attn.fuse_projections()

    def _mlp(self, h: torch.Tensor) -> torch.Tensor:
        w = self._gate_up
        if w is not None and w.data_ptr() == self.gate_proj.weight.data_ptr() and w.dtype == h.dtype:
            gu = F.linear(h, w)
            n = self.gate_proj.weight.shape[0]
            return self.down_proj(F.silu(gu[..., :n]) * gu[..., n:])
        return self.down_proj(F.silu(self.gate_proj(h)) * self.up_proj(h))

    def forward(self, x, cos, sin, layer_cache) -> torch.Tensor:
        a = self.self_attn(self.input_layernorm(x), cos, sin, layer_cache)
        x, h = self.post_attention_layernorm.add_forward(x, a)
        return x + self._mlp(h)


class Qwen3(nn.Module):
    """Qwen3 decoder with tied embeddings; attention goes through ``backend``."""

    def __init__(self, s: Qwen3Shape = QWEN3_06B, backend=None) -> None:
        super().__init__()
        self.s = s
        self.backend = backend if backend is not None else CudaPagedAttentionBackend()
        self.embed = nn.Parameter(torch.empty(s.vocab_size, s.hidden_size))
        nn.init.normal_(self.embed, mean=0.0, std=0.02)
        self.layers = nn.ModuleList([Block(s, self.backend) for _ in range(s.num_layers)])
        self.norm = RMSNorm(s.hidden_size, s.rms_norm_eps)

    def fuse_projections(self) -> None:
        """Fused [q; k; v] and [gate; up] weights in every block (same values,
        fewer GEMM launches); idempotent."""
        for blk in self.layers:
            if blk._gate_up is None:
                blk.fuse_projections()

    def set_backend(self, backend) -> None:
        self.backend = backend
        for blk in self.layers:
            blk.self_attn.backend = backend

    def forward(self, token_ids: torch.Tensor, position_ids: torch.Tensor, kv_cache=None,
                logits_index: torch.Tensor | None = None) -> torch.Tensor:
        """``logits_index``: token positions (on the T axis) whose logits are
        wanted; the LM head then runs on those rows only."""
        h = self.embed[token_ids]
        cos, sin = rope_cos_sin(self.s.head_dim, self.s.rope_theta, position_ids, h.dtype)
        for i, blk in enumerate(self.layers):
            h = blk(h, cos, sin, None if kv_cache is None else kv_cache.layer(i))
        if logits_index is not None:
            h = h[:, logits_index]
        return torch.matmul(self.norm(h), self.embed.T)


def random_qwen3(shape: Qwen3Shape = QWEN3_06B, dtype=torch.bfloat16, device="cuda", seed: int = 0,
                 init: str = "spread") -> Qwen3:
    """A randomly initialised decoder.  ``init="spread"`` (default): token
    embeddings ~ N(0, 0.02^2) and every projection ~ N(0, 1/fan_in), so the
    attention and MLP outputs outweigh the token's own embedding in the
    residual stream and a greedy stream does not collapse onto one repeated
    token (with nn.Linear's smaller default init the tied head mostly returns
    the input token).  ``init="default"``: nn.Linear's own init."""
    torch.manual_seed(seed)
    with torch.device("cpu"):
        model = Qwen3(shape)
        if init == "spread":
            with torch.no_grad():
                for m in model.modules():
                    if isinstance(m, nn.Linear):
                        m.weight.normal_(0.0, m.weight.shape[1] ** -0.5)
        elif init != "default":
            raise ValueError(f"unknown init {init!r}")
    return model.to(device=device, dtype=dtype).eval()


class _Request:
    def __init__(self, rid: str, tokens: list[int]) -> None:
        self.id = rid
        self.tokens = list(tokens)

    @property
    def seq_len(self) -> int:
        return len(self.tokens)


def plan_prefill_chunks(prompt_lens: list[int], budget: int) -> list[list[tuple[int, int, int]]]:
    """Groups of (request, first token, token count) runs, each group at most
    ``budget`` tokens, taking prompts in order and splitting a prompt where a
    group's budget ends (its remainder opens the next group)."""
    check_positive = budget > 0 and all(n > 0 for n in prompt_lens)
    if not check_positive:
        raise ValueError("prefill budget and prompt lengths must be positive")
    groups: list[list[tuple[int, int, int]]] = []
    group: list[tuple[int, int, int]] = []
    left = budget
    for r, n in enumerate(prompt_lens):
        s = 0
        while s < n:
            take = min(n - s, left)
            group.append((r, s, take))
            s += take
            left -= take
            if left == 0:
                groups.append(group)
                group, left = [], budget
    if group:
        groups.append(group)
    return groups


class PagedEngine:
    """Prefill-then-batched-greedy-decode over a paged cache on one GPU.

    Prefill packs the prompts of many requests into one forward of at most
    ``prefill_tokens`` tokens, splitting a long prompt into chunks that each
    continue over the request's cached earlier chunks (PackedBatchKVCache; the
    reference prefills one request per forward, engine.py:226-257, and has no
    chunked prefill, docs/ROADMAP.md:131).  ``prefill_tokens=0`` prefills each
    request on its own through the single-request PagedLayerKV path, as the
    reference does.  Every decode step then runs all requests as one
    BatchKVCache batch (engine.py:458-488)."""

    def __init__(self, model: Qwen3, num_blocks: int, block_size: int = 16, max_requests: int = 256,
                 prefill_tokens: int = 8192) -> None:
        s = model.s
        dev = next(model.parameters()).device
        dtype = next(model.parameters()).dtype
        self.model = model
        model.fuse_projections()
        self.block_size = block_size
        self.cache = PagedKVCache(s.num_layers, num_blocks, s.num_kv_heads, block_size, s.head_dim, dtype=dtype,
                                  device=dev, max_requests=max_requests)
        self.pool = BlockPool(num_blocks)
        self.manager = KVCacheManager(block_size, self.pool, self.cache)
        self.device = dev
        self.prefill_tokens = int(prefill_tokens)

    @staticmethod
    def blocks_needed(prompt_lens: list[int], max_new: int, block_size: int) -> int:
        return sum(math.ceil((n + max_new) / block_size) for n in prompt_lens)

    @torch.inference_mode()
    def generate(self, prompts: list[list[int]], max_new_tokens: int, timings: dict | None = None,
                 use_graph: bool = True) -> list[list[int]]:
        """Greedy generation.  ``use_graph``: after one eager decode step, the
        decode step (all layers, append + attention kernels, argmax) is captured
        once as a CUDA graph and replayed; each replay only needs the next
        tokens, positions and lengths copied in."""
        reqs = [_Request(f"req-{i}", p) for i, p in enumerate(prompts)]
        dev = self.device
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t2 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for r in reqs:
            if not self.manager.allocate_request(r):
                raise RuntimeError("KV pool exhausted during prefill")
        if self.prefill_tokens > 0:
            self._prefill_packed(reqs)
        else:
            for r in reqs:
                ids = torch.tensor([r.tokens], dtype=torch.long, device=dev)
                pos = torch.arange(r.seq_len, device=dev).unsqueeze(0)
                last = torch.tensor([r.seq_len - 1], device=dev)
                logits = self.model(ids, pos, kv_cache=self.manager.get_cache(r), logits_index=last)
                r.tokens.append(int(torch.argmax(logits[0, -1]).item()))
        t1.record()
        if use_graph and max_new_tokens > 2:
            self._decode_graph(reqs, max_new_tokens - 1)
        else:
            for _ in range(max_new_tokens - 1):
                for r in reqs:
                    if not self.manager.allocate_request(r):
                        raise RuntimeError("KV pool exhausted during decode")
                ids = torch.tensor([[r.tokens[-1]] for r in reqs], dtype=torch.long, device=dev)
                pos = torch.tensor([[r.seq_len - 1] for r in reqs], dtype=torch.long, device=dev)
                logits = self.model(ids, pos, kv_cache=BatchKVCache([self.manager.get_cache(r) for r in reqs]))
                nxt = torch.argmax(logits[:, -1], dim=-1).tolist()
                for r, tok in zip(reqs, nxt):
                    r.tokens.append(int(tok))
        t2.record()
        torch.cuda.synchronize(dev)
        self.cache.check_device_errors()
        if timings is not None:
            timings["prefill_ms"] = t0.elapsed_time(t1)
            timings["decode_ms"] = t1.elapsed_time(t2)
            timings["decode_steps"] = max_new_tokens - 1
        out = [r.tokens[len(p):] for r, p in zip(reqs, prompts)]
        for r in reqs:
            self.manager.free_request(r.id)
        return out

    def _prefill_packed(self, reqs: list[_Request]) -> None:
        """One forward per group of ``plan_prefill_chunks``; a request's first
        token comes from the forward holding its prompt's last token."""
        dev = self.device
        plens = [r.seq_len for r in reqs]
        for group in plan_prefill_chunks(plens, self.prefill_tokens):
            ids = np.concatenate([reqs[m].tokens[s:s + n] for m, s, n in group])
            pos = np.concatenate([np.arange(s, s + n) for _, s, n in group])
            ends = np.cumsum([n for _, _, n in group]) - 1
            finishing = [k for k, (m, s, n) in enumerate(group) if s + n == plens[m]]
            cache = PackedBatchKVCache([self.manager.get_cache(reqs[m]) for m, _, _ in group], [n for _, _, n in group])
            ids_d = torch.from_numpy(ids.astype(np.int64)).to(dev, non_blocking=True).unsqueeze(0)
            pos_d = torch.from_numpy(pos.astype(np.int64)).to(dev, non_blocking=True).unsqueeze(0)
            idx_d = torch.from_numpy(ends[finishing].astype(np.int64)).to(dev, non_blocking=True)
            logits = self.model(ids_d, pos_d, kv_cache=cache, logits_index=idx_d)
            if finishing:
                for k, tok in zip(finishing, torch.argmax(logits[0], dim=-1).tolist()):
                    reqs[group[k][0]].tokens.append(int(tok))

    def _decode_graph(self, reqs: list[_Request], steps: int) -> None:
        dev = self.device
        b = len(reqs)
        # every block the decode will need, up front: the captured kernels hold
        # the block-table pointer, so the arena must not grow afterwards
        final = [_Request(r.id, r.tokens + [0] * (steps - 1)) for r in reqs]
        for r in final:
            if not self.manager.allocate_request(r):
                raise RuntimeError("KV pool exhausted during decode")
        bound = max(len(r.tokens) for r in final)
        batch = BatchKVCache([self.manager.get_cache(r) for r in reqs], static_max_seq_len=bound)
        rows = batch.rows
        lens = self.cache.arena.lens
        ids_h = torch.empty((b, 1), dtype=torch.long).pin_memory()
        pos_h = torch.empty((b, 1), dtype=torch.long).pin_memory()
        ids_d = torch.empty((b, 1), dtype=torch.long, device=dev)
        pos_d = torch.empty((b, 1), dtype=torch.long, device=dev)
        nxt_d = torch.empty((b,), dtype=torch.long, device=dev)

        def stage_inputs():
            ids_h[:, 0] = torch.tensor([r.tokens[-1] for r in reqs])
            pos_h[:, 0] = torch.from_numpy(lens[rows, 0].copy())
            ids_d.copy_(ids_h, non_blocking=True)
            pos_d.copy_(pos_h, non_blocking=True)

        def body():
            logits = self.model(ids_d, pos_d, kv_cache=batch)
            nxt_d.copy_(torch.argmax(logits[:, -1], dim=-1))

        def take():
            for r, tok in zip(reqs, nxt_d.tolist()):
                r.tokens.append(int(tok))

        # step 1 eager: sizes the workspace, warms cuBLAS and the allocator
        stage_inputs()
        body()
        take()
        if steps == 1:
            return
        # step 2 captured (capturing runs the host side, advancing lengths),
        # then replayed to execute it
        stage_inputs()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            body()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph.replay()
        take()
        meta = batch._static
        for _ in range(steps - 2):
            meta.stage(lens[rows, 0].copy(), 1)
            stage_inputs()
            graph.replay()
            lens[rows, :] += 1
            take()
        del graph
