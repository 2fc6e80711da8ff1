"""A random-initialised Llama-3 decode step whose linears run through ZipGEMM.

The benchmarked decode step (a full decode step of a random-init
Llama-3-8B architecture with its linears on ZipGEMM, per-step latency at
TP = 1/2/4/8 against cuBLAS BF16): 32 layers, hidden 4096, 32 query and 8
KV heads of dim 128, SwiGLU intermediate 14336, vocabulary 128256 with an
untied, compressed lm_head, RMSNorm weights 1.0, every linear N(0, 0.02)
BF16, and a KV cache of `context` random entries per sequence. One step
takes one token per sequence through the whole model and picks the next
token greedily.

Tensor parallelism is Megatron's: the fused qkv projection is split by
heads (each rank keeps its query heads and its KV heads), gate_up by
intermediate rows (each rank keeps the same rows of gate and of up), both
with no collective; o and down are split on K (the rank's heads / its
intermediate slice) and their outputs all-reduced; the lm_head is split by
vocabulary rows (padded to a multiple of 64 per rank) and the greedy token
is the best of the ranks' local maxima. Every rank draws the full weights
from the same seeds and keeps its shard, so the model is the same at every
TP degree.

The same object runs in two modes over the same weights: "zipgemm" (every
linear packed on the GPU and multiplied by the fused kernel) and "dense"
(the BF16 weights and F.linear, i.e. cuBLAS). Attention is PyTorch's
scaled_dot_product_attention over the cache; norms, RoPE and SwiGLU are
plain tensor ops. `capture` records a whole step in a CUDA graph.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import Tensor

from . import runtime


@dataclass(frozen=True)
class LlamaShape:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    context: int = 2048
    rope_theta: float = 500000.0
    eps: float = 1e-5


LLAMA3_8B = LlamaShape()


def _draw(shape, seed: int, device) -> Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16)


class DecodeStep:
    """One rank's shard of the model, its KV cache (for up to `max_batch`
    sequences) and the step function."""

    def __init__(self, shape: LlamaShape, max_batch: int, device, *, mode: str = "zipgemm",
                 world: int = 1, rank: int = 0, group=None, seed: int = 0, linear=None,
                 pack=None):
        if mode not in ("zipgemm", "dense"):
            raise ValueError("mode must be zipgemm or dense")
        s = shape
        if s.heads % world or s.kv_heads % world or s.ffn % world:
            raise ValueError("heads, KV heads and the intermediate size must split over ranks")
        self.shape, self.mode, self.world, self.rank, self.group = s, mode, world, rank, group
        self.device = torch.device(device)
        self.hq, self.hkv = s.heads // world, s.kv_heads // world
        self.fl = s.ffn // world
        per_rank = -(-s.vocab // (64 * world)) * 64
        self.vocab_rank = per_rank
        self.vocab_begin = rank * per_rank
        self._linear = linear or runtime.linear
        self._pack = pack or runtime.compress_device
        hd = s.head_dim
        self.layers = []
        for li in range(s.layers):
            base = 1000 * (seed + 1) + 10 * li
            w_qkv = _draw(((s.heads + 2 * s.kv_heads) * hd, s.hidden), base + 0, self.device)
            q0, k0 = s.heads * hd, (s.heads + s.kv_heads) * hd
            qkv = torch.cat((w_qkv[rank * self.hq * hd:(rank + 1) * self.hq * hd],
                             w_qkv[q0 + rank * self.hkv * hd:q0 + (rank + 1) * self.hkv * hd],
                             w_qkv[k0 + rank * self.hkv * hd:k0 + (rank + 1) * self.hkv * hd]))
            o = _draw((s.hidden, s.heads * hd), base + 1, self.device)
            o = o[:, rank * self.hq * hd:(rank + 1) * self.hq * hd]
            gu = _draw((2 * s.ffn, s.hidden), base + 2, self.device)
            gu = torch.cat((gu[rank * self.fl:(rank + 1) * self.fl],
                            gu[s.ffn + rank * self.fl:s.ffn + (rank + 1) * self.fl]))
            down = _draw((s.hidden, s.ffn), base + 3, self.device)
            down = down[:, rank * self.fl:(rank + 1) * self.fl]
            self.layers.append({name: self._weight(w) for name, w in
                                (("qkv", qkv), ("o", o), ("gate_up", gu), ("down", down))})
            del w_qkv, gu, down
        head = _draw((per_rank * world, s.hidden), 1000 * (seed + 1) - 1, self.device)
        head[s.vocab:] = 0  # padding rows (their logits are masked)
        self.lm_head = self._weight(head[rank * per_rank:(rank + 1) * per_rank])
        del head
        self.embed = _draw((s.vocab, s.hidden), 1000 * (seed + 1) - 2, self.device)
        # Random KV cache: `context` past positions; the step writes position
        # `context`. Drawn per (layer, global KV head) so every TP degree
        # sees the same cache.
        cache_shape = (s.layers, max_batch, self.hkv, s.context + 1, hd)
        self.k_cache = torch.empty(cache_shape, device=self.device, dtype=torch.bfloat16)
        self.v_cache = torch.empty(cache_shape, device=self.device, dtype=torch.bfloat16)
        for li in range(s.layers):
            for i in range(self.hkv):
                g = torch.Generator(device=self.device).manual_seed(
                    7 + seed + 1000 * li + (rank * self.hkv + i))
                for cache in (self.k_cache, self.v_cache):
                    cache[li, :, i] = torch.randn((max_batch, s.context + 1, hd), generator=g,
                                                  device=self.device, dtype=torch.bfloat16)
        inv = 1.0 / (s.rope_theta ** (torch.arange(0, hd, 2, device=self.device).float() / hd))
        ang = float(s.context) * inv
        self.cos = torch.cat((ang.cos(), ang.cos())).to(torch.bfloat16)
        self.sin = torch.cat((ang.sin(), ang.sin())).to(torch.bfloat16)
        self.scale = 1.0 / math.sqrt(hd)
        self.exchange = None

    @classmethod
    def packed_from(cls, dense: "DecodeStep", pack=None, linear=None,
                    exchange=None) -> "DecodeStep":
        """The "zipgemm" twin of a dense model: the same weights packed on the
        GPU, sharing the embedding and the KV cache. With a tp.PeerExchange,
        the row-parallel o and down projections sum their outputs across
        ranks inside the fused kernel instead of with an all-reduce."""
        if dense.mode != "dense":
            raise ValueError("packed_from needs a dense model")
        twin = cls.__new__(cls)
        twin.__dict__.update(dense.__dict__)
        twin.mode = "zipgemm"
        twin._pack = pack or runtime.compress_device
        twin._linear = linear or runtime.linear
        twin.layers = [{name: twin._pack(w) for name, w in layer.items()} for layer in dense.layers]
        twin.lm_head = twin._pack(dense.lm_head)
        twin.exchange = exchange
        return twin

    def _weight(self, w: Tensor):
        w = w.contiguous()
        return self._pack(w) if self.mode == "zipgemm" else w

    def weight_bytes(self) -> int:
        def size(w):
            return w.storage_bytes if isinstance(w, runtime.PackedWeight) else w.numel() * 2
        return sum(size(w) for layer in self.layers for w in layer.values()) + size(self.lm_head)

    def _lin(self, x: Tensor, w) -> Tensor:
        if isinstance(w, runtime.PackedWeight):
            return self._linear(x, w)
        return F.linear(x, w)

    def _norm(self, x: Tensor) -> Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.shape.eps)).to(x.dtype)

    def _rope(self, x: Tensor) -> Tensor:
        half = x.shape[-1] // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * self.cos + rot * self.sin

    def _reduce(self, y: Tensor) -> Tensor:
        if self.world > 1:
            dist.all_reduce(y, group=self.group)
        return y

    def _row(self, x: Tensor, w) -> Tensor:
        """Row-parallel linear summed over ranks (inside the kernel when an
        exchange is set, else an all-reduce after it)."""
        if self.exchange is not None and isinstance(w, runtime.PackedWeight):
            return self.exchange.linear(x, w)
        return self._reduce(self._lin(x, w))

    def logits(self, tokens: Tensor) -> Tensor:
        """[B] token ids -> this rank's [B, vocab_rank] logits (FP32, padding -inf)."""
        s, hd = self.shape, self.shape.head_dim
        b = tokens.shape[0]
        h = self.embed[tokens]
        for li, L in enumerate(self.layers):
            x = self._norm(h)
            qkv = self._lin(x, L["qkv"])
            q = qkv[:, :self.hq * hd].view(b, self.hq, 1, hd)
            k = qkv[:, self.hq * hd:(self.hq + self.hkv) * hd].view(b, self.hkv, hd)
            v = qkv[:, (self.hq + self.hkv) * hd:].view(b, self.hkv, hd)
            q = self._rope(q)
            kc, vc = self.k_cache[li, :b], self.v_cache[li, :b]
            kc[:, :, s.context] = self._rope(k)
            vc[:, :, s.context] = v
            attn = F.scaled_dot_product_attention(q, kc, vc, scale=self.scale, enable_gqa=True)
            h = h + self._row(attn.reshape(b, self.hq * hd), L["o"])
            x = self._norm(h)
            gu = self._lin(x, L["gate_up"])
            a = F.silu(gu[:, :self.fl]) * gu[:, self.fl:]
            h = h + self._row(a, L["down"])
        logits = self._lin(self._norm(h), self.lm_head).float()
        cols = torch.arange(self.vocab_rank, device=logits.device) + self.vocab_begin
        return logits.masked_fill(cols >= s.vocab, float("-inf"))

    def step(self, tokens: Tensor) -> Tensor:
        """Greedy next tokens for a batch of sequences ([B] int64)."""
        logits = self.logits(tokens)
        best, idx = logits.max(dim=-1)
        idx = idx + self.vocab_begin
        if self.world == 1:
            return idx
        vals = [torch.empty_like(best) for _ in range(self.world)]
        ids = [torch.empty_like(idx) for _ in range(self.world)]
        dist.all_gather(vals, best, group=self.group)
        dist.all_gather(ids, idx, group=self.group)
        pick = torch.stack(vals).argmax(dim=0)
        return torch.stack(ids).gather(0, pick.unsqueeze(0)).squeeze(0)

    def capture(self, tokens: Tensor, stream=None):
        """A CUDA graph of one step on `tokens` (a static buffer); returns
        (graph, output buffer)."""
        stream = stream or torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            self.step(tokens)  # warm-up on the capture stream
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                out = self.step(tokens)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        return graph, out
