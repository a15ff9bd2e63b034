"""Llama-shaped decoder stacks whose linears are packed Block-RVQ layers.

The benchmark configurations describe random-init Llama-3-style decoders (1B,
8B, 70B shapes) in which every q/k/v/o/gate/up/down projection is a Block-RVQ
linear (d = 8, R = 2 stages of 256 entries, cfg0 distributions) and the
lm_head stays dense bf16, as in the reference's model surgery (reference
``src/runtime.py:41-49`` lists exactly those seven projection suffixes).  This
module builds such stacks without materialising dense weights and runs
autoregressive decode steps with a bf16 KV cache.

Projections sharing an input are fused into one launch: q/k/v form one packed
linear with three row groups (each with its own codebooks, exactly like three
separate layers) and gate/up one with two.

Tensor parallelism (``tp_size > 1``, one process per GPU, NCCL): q/k/v and
gate/up are split by output rows (heads / MLP columns: column-parallel), o and
down by input blocks (row-parallel) and their fp32 partial outputs are summed
with one all-reduce each; the lm_head is split by vocabulary rows and its
logits all-gathered.  Block boundaries (d = 8) divide every split.

A ``DenseLlama`` twin with bf16 ``F.linear`` projections (cuBLAS) runs the same
glue code, so the two decode rates differ only in the linears.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .runtime import PackedGroupedBlockRVQLinear


@dataclass(frozen=True)
class LlamaShape:
    layers: int
    hidden: int
    mlp: int
    heads: int
    kv_heads: int
    vocab: int
    rope_theta: float = 500000.0
    eps: float = 1e-5
    tied_embeddings: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


LLAMA_1B = LlamaShape(16, 2048, 8192, 32, 8, 128256, tied_embeddings=True)
LLAMA_8B = LlamaShape(32, 4096, 14336, 32, 8, 128256)
LLAMA_70B = LlamaShape(80, 8192, 28672, 64, 8, 128256)
SHAPES = {"1b": LLAMA_1B, "8b": LLAMA_8B, "70b": LLAMA_70B}


class TPContext:
    """Tensor-parallel rank info; all-reduce/all-gather through torch.distributed."""

    def __init__(self, rank: int = 0, size: int = 1, group=None):
        self.rank, self.size, self.group = int(rank), int(size), group

    def all_reduce_(self, t: Tensor) -> Tensor:
        if self.size > 1:
            torch.distributed.all_reduce(t, group=self.group)
        return t

    def all_gather_last(self, t: Tensor) -> Tensor:
        if self.size == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(self.size)]
        torch.distributed.all_gather(parts, t.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)


def _split(n: int, size: int, what: str) -> int:
    if n % size:
        raise ValueError(f"{what} ({n}) is not divisible by the tensor-parallel size {size}")
    return n // size


class DecoderLayer(nn.Module):
    """One decoder block: RMSNorm -> qkv -> RoPE/KV cache/attention -> o -> RMSNorm -> gate_up -> SiLU*mul -> down."""

    def __init__(self, shape: LlamaShape, make_linear: Callable[[list[int], int], nn.Module], tp: TPContext,
                 device, gen: Optional[torch.Generator]):
        super().__init__()
        self.shape, self.tp = shape, tp
        hd = shape.head_dim
        self.hq = _split(shape.heads, tp.size, "heads")
        self.hkv = _split(shape.kv_heads, tp.size, "kv heads")
        self.mlp = _split(shape.mlp, tp.size, "mlp")
        self.qkv = make_linear([self.hq * hd, self.hkv * hd, self.hkv * hd], shape.hidden)
        self.o = make_linear([shape.hidden], self.hq * hd)
        self.gate_up = make_linear([self.mlp, self.mlp], shape.hidden)
        self.down = make_linear([shape.hidden], self.mlp)
        self.register_buffer("in_norm", 1.0 + 0.1 * torch.randn(shape.hidden, device=device, generator=gen).to(torch.bfloat16))
        self.register_buffer("post_norm", 1.0 + 0.1 * torch.randn(shape.hidden, device=device, generator=gen).to(torch.bfloat16))

    def _row_parallel(self, lin: nn.Module, x: Tensor) -> Tensor:
        if self.tp.size == 1:
            return lin(x)
        if isinstance(lin, PackedGroupedBlockRVQLinear):  # fp32 partial straight from the GEMV
            y = torch.empty((x.shape[0], lin.out_features), device=x.device, dtype=torch.float32)
            lin.gemv_into(x, y)
        else:
            y = lin(x).float()
        return self.tp.all_reduce_(y).to(torch.bfloat16)

    def forward(self, h: Tensor, cos: Tensor, sin: Tensor, k_cache: Tensor, v_cache: Tensor, pos: int) -> Tensor:
        shape = self.shape
        hd = shape.head_dim
        B = h.shape[0]
        x = F.rms_norm(h, (shape.hidden,), self.in_norm, shape.eps)
        qkv = self.qkv(x)
        q, k, v = qkv.split([self.hq * hd, self.hkv * hd, self.hkv * hd], dim=-1)
        q = _rope(q.view(B, self.hq, hd), cos, sin)
        k = _rope(k.view(B, self.hkv, hd), cos, sin)
        k_cache[:, :, pos] = k
        v_cache[:, :, pos] = v.view(B, self.hkv, hd)
        attn = F.scaled_dot_product_attention(q.unsqueeze(2), k_cache[:, :, : pos + 1], v_cache[:, :, : pos + 1],
                                              enable_gqa=True)
        h = h + self._row_parallel(self.o, attn.reshape(B, self.hq * hd))
        x = F.rms_norm(h, (shape.hidden,), self.post_norm, shape.eps)
        g, u = self.gate_up(x).split([self.mlp, self.mlp], dim=-1)
        return h + self._row_parallel(self.down, F.silu(g) * u)


def _rope(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotary embedding (rotate-half convention) for one position; x [B, H, hd]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    rot = torch.cat((-x2, x1), dim=-1)
    return (x.float() * cos + rot.float() * sin).to(x.dtype)


class LlamaStack(nn.Module):
    """Decoder stack with a bf16 KV cache; ``decode_step`` advances every sequence by one token."""

    def __init__(self, shape: LlamaShape, make_linear: Callable[[list[int], int], nn.Module], *, device="cuda",
                 seed: int = 0, tp: Optional[TPContext] = None):
        super().__init__()
        self.shape = shape
        self.tp = tp or TPContext()
        device = torch.device(device)
        gen = torch.Generator(device=device).manual_seed(int(seed))
        self.layers = nn.ModuleList(DecoderLayer(shape, make_linear, self.tp, device, gen) for _ in range(shape.layers))
        self.register_buffer("embed", (torch.randn(shape.vocab, shape.hidden, device=device, generator=gen) * 0.02).to(torch.bfloat16))
        self.register_buffer("final_norm", torch.ones(shape.hidden, device=device, dtype=torch.bfloat16))
        vshard = _split(shape.vocab, self.tp.size, "vocab")
        if shape.tied_embeddings and self.tp.size == 1:
            self.lm_head = self.embed
        else:
            self.register_buffer("lm_head", (torch.randn(vshard, shape.hidden, device=device, generator=gen) * 0.02).to(torch.bfloat16))
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, shape.head_dim, 2, device=device, dtype=torch.float32) / shape.head_dim))
        self.register_buffer("inv_freq", inv)
        self.k_cache: list[Tensor] = []
        self.v_cache: list[Tensor] = []

    def allocate_cache(self, batch: int, max_len: int, *, fill_random: bool = True, seed: int = 1) -> None:
        hkv = self.layers[0].hkv
        hd = self.shape.head_dim
        dev = self.embed.device
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.k_cache, self.v_cache = [], []
        for _ in self.layers:
            k = torch.empty(batch, hkv, max_len, hd, device=dev, dtype=torch.bfloat16)
            v = torch.empty_like(k)
            if fill_random:
                k.normal_(generator=gen)
                v.normal_(generator=gen)
            self.k_cache.append(k)
            self.v_cache.append(v)

    def rope_tables(self, pos: int) -> tuple[Tensor, Tensor]:
        ang = float(pos) * self.inv_freq
        emb = torch.cat((ang, ang))
        return emb.cos(), emb.sin()

    @torch.no_grad()
    def decode_step(self, tokens: Tensor, pos: int, cos: Tensor, sin: Tensor) -> Tensor:
        """tokens [B] int64 at position ``pos`` (cache holds positions < pos) -> logits [B, vocab] bf16."""
        h = self.embed[tokens]
        for layer, kc, vc in zip(self.layers, self.k_cache, self.v_cache):
            h = layer(h, cos, sin, kc, vc, pos)
        h = F.rms_norm(h, (self.shape.hidden,), self.final_norm, self.shape.eps)
        logits = F.linear(h, self.lm_head)
        return self.tp.all_gather_last(logits)

    def linear_bytes(self) -> int:
        """Bytes of the projection weights a decode step streams (packed or dense)."""
        total = 0
        for m in self.modules():
            if isinstance(m, PackedGroupedBlockRVQLinear):
                total += m.compressed_bytes()
            elif isinstance(m, DenseLinear):
                total += m.weight.numel() * 2
        return total


class DenseLinear(nn.Module):
    """bf16 linear without bias (cuBLAS through F.linear); weight [out, in]."""

    def __init__(self, out_features: int, in_features: int, device, gen):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_buffer("weight", (torch.randn(out_features, in_features, device=device, generator=gen) * 0.02).to(torch.bfloat16))

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight)


def rvq_llama(shape: LlamaShape, *, device="cuda", seed: int = 0, tp: Optional[TPContext] = None) -> LlamaStack:
    """Random-init Llama-shaped stack with Block-RVQ projections (d=8, R=2, 256 entries)."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(int(seed) + 1000)

    def make(rows: list[int], k: int) -> nn.Module:
        return PackedGroupedBlockRVQLinear.random(rows, k, block_size=8, num_stages=2, entries=256,
                                                  generator=gen, device=device)

    return LlamaStack(shape, make, device=device, seed=seed, tp=tp)


def dense_llama(shape: LlamaShape, *, device="cuda", seed: int = 0, tp: Optional[TPContext] = None) -> LlamaStack:
    """The same stack with dense bf16 projections (comparison baseline)."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(int(seed) + 2000)

    def make(rows: list[int], k: int) -> nn.Module:
        return DenseLinear(int(sum(rows)), k, device, gen)

    return LlamaStack(shape, make, device=device, seed=seed, tp=tp)


@torch.no_grad()
def time_decode(stack: LlamaStack, batch: int, context: int, *, steps: int = 20, warmup: int = 3,
                graph: bool = True) -> dict:
    """Time one decode step at a fixed context length (cache pre-filled), optionally as a CUDA graph."""
    stack.allocate_cache(batch, context + 1)
    dev = stack.embed.device
    tokens = torch.randint(0, stack.shape.vocab, (batch,), device=dev)
    cos, sin = stack.rope_tables(context)
    for _ in range(warmup):
        stack.decode_step(tokens, context, cos, sin)
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            stack.decode_step(tokens, context, cos, sin)
        for _ in range(warmup):
            g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        if g is not None:
            g.replay()
        else:
            stack.decode_step(tokens, context, cos, sin)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del g
    return {"ms_per_step": ms, "tok_s": batch * 1e3 / ms, "batch": batch, "context": context}
