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

from .decode_ops import decode_attention, decode_attention_workspace, residual_rmsnorm, rope_kv_append, silu_mul
from .runtime import PackedGroupedBlockRVQLinear
from .tp import COLUMN, ROW, shard_bounds, shard_packed


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
    """Tensor-parallel rank info; collectives through torch.distributed (NCCL on GPUs)."""

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


# A linear factory gets the FULL layer's group row counts, its full in_features
# and the split mode, and returns this rank's shard.
LinearFactory = Callable[[list[int], int, str], nn.Module]


class DecoderLayer(nn.Module):
    """One decoder block: RMSNorm -> qkv -> RoPE/KV cache/attention -> o -> RMSNorm -> gate_up -> SiLU*mul -> down."""

    def __init__(self, shape: LlamaShape, make_linear: LinearFactory, tp: TPContext, device,
                 gen: Optional[torch.Generator]):
        super().__init__()
        self.shape, self.tp = shape, tp
        hd = shape.head_dim
        self.hq = _split(shape.heads, tp.size, "heads")
        self.hkv = _split(shape.kv_heads, tp.size, "kv heads")
        self.mlp = _split(shape.mlp, tp.size, "mlp")
        self.qkv = make_linear([shape.heads * hd, shape.kv_heads * hd, shape.kv_heads * hd], shape.hidden, COLUMN)
        self.o = make_linear([shape.hidden], shape.heads * hd, ROW)
        self.gate_up = make_linear([shape.mlp, shape.mlp], shape.hidden, COLUMN)
        self.down = make_linear([shape.hidden], shape.mlp, ROW)
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
        """Operator-by-operator decode step (PyTorch glue); the fused step must match it."""
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


class _DecodeBuffers:
    """Preallocated activations of the fused decode step for one batch size."""

    def __init__(self, stack: "LlamaStack", batch: int):
        s, dev, bf = stack.shape, stack.embed.device, torch.bfloat16
        l0 = stack.layers[0]
        hd = s.head_dim
        self.h = torch.empty(batch, s.hidden, device=dev, dtype=bf)
        self.x = torch.empty(batch, s.hidden, device=dev, dtype=bf)
        self.qkv = torch.empty(batch, (l0.hq + 2 * l0.hkv) * hd, device=dev, dtype=bf)
        self.q = torch.empty(batch, l0.hq * hd, device=dev, dtype=bf)
        self.attn = torch.empty(batch, l0.hq * hd, device=dev, dtype=bf)
        self.gu = torch.empty(batch, 2 * l0.mlp, device=dev, dtype=bf)
        self.act = torch.empty(batch, l0.mlp, device=dev, dtype=bf)
        self.y32 = torch.empty(batch, s.hidden, device=dev, dtype=torch.float32)
        self.ybf = torch.empty(batch, s.hidden, device=dev, dtype=bf)  # a dense linear's output before a push
        cache_len = stack.k_cache[0].shape[2] if stack.k_cache else 1
        self.attn_ws = decode_attention_workspace(batch, l0.hq, l0.hkv, hd, cache_len, dev)
        self.cache_len = cache_len


class LlamaStack(nn.Module):
    """Decoder stack with a bf16 KV cache; ``decode_step`` advances every sequence by one token.

    ``decode_step_fused`` is the production step: the linears plus four glue
    kernels per block (RoPE/KV append, split-K decode attention, SiLU*mul,
    residual + RMSNorm after each row-parallel linear) and, with
    ``exchange="push"`` under tensor parallelism, the peer-memory exchange
    instead of an NCCL all-reduce.
    ``decode_step`` is the same computation with PyTorch operators.
    """

    def __init__(self, shape: LlamaShape, make_linear: LinearFactory, *, device="cuda", seed: int = 0,
                 tp: Optional[TPContext] = None):
        super().__init__()
        self.shape = shape
        self.tp = tp or TPContext()
        device = torch.device(device)
        gen = torch.Generator(device=device).manual_seed(int(seed))
        self.layers = nn.ModuleList(DecoderLayer(shape, make_linear, self.tp, device, gen) for _ in range(shape.layers))
        self.register_buffer("embed", (torch.randn(shape.vocab, shape.hidden, device=device, generator=gen) * 0.02).to(torch.bfloat16))
        self.register_buffer("final_norm", torch.ones(shape.hidden, device=device, dtype=torch.bfloat16))
        v0, v1 = shard_bounds(shape.vocab, self.tp.rank, self.tp.size, 1, "vocab")
        if shape.tied_embeddings:
            head = self.embed
        else:
            head = (torch.randn(shape.vocab, shape.hidden, device=device, generator=gen) * 0.02).to(torch.bfloat16)
        self.register_buffer("lm_head", head[v0:v1].contiguous() if self.tp.size > 1 else head)
        inv = 1.0 / (shape.rope_theta ** (torch.arange(0, shape.head_dim, 2, device=device, dtype=torch.float32) / shape.head_dim))
        self.register_buffer("inv_freq", inv)
        self.k_cache: list[Tensor] = []
        self.v_cache: list[Tensor] = []
        self.exchange = None  # PeerExchange for exchange="push"
        self._bufs: dict[int, _DecodeBuffers] = {}

    def allocate_cache(self, batch: int, max_len: int, *, fill_random: bool = True, seed: int = 1,
                       consistent: bool = False) -> None:
        """bf16 caches [batch, local kv heads, max_len, head_dim] per layer.

        ``consistent``: draw the full (all-rank) cache and keep this rank's
        heads, so shards of one model hold slices of the same cache.
        """
        hkv = self.layers[0].hkv
        hd = self.shape.head_dim
        dev = self.embed.device
        gen = torch.Generator(device=dev).manual_seed(seed)
        self.k_cache, self.v_cache = [], []
        h0 = self.tp.rank * hkv
        for _ in self.layers:
            if fill_random and consistent:
                k = torch.randn(batch, self.shape.kv_heads, max_len, hd, device=dev, generator=gen).to(torch.bfloat16)
                v = torch.randn(batch, self.shape.kv_heads, max_len, hd, device=dev, generator=gen).to(torch.bfloat16)
                k, v = k[:, h0:h0 + hkv].contiguous(), v[:, h0:h0 + hkv].contiguous()
            else:
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

    def enable_push_exchange(self, max_batch: int) -> None:
        """Create the peer-memory exchange used by ``decode_step_fused(exchange="push")``."""
        from .tp import PeerExchange

        if self.exchange is not None and self.exchange.max_rows < max_batch:
            self.exchange.close()  # every rank re-creates it together (same call order)
            self.exchange = None
        if self.exchange is None:
            self.exchange = PeerExchange(self.tp.rank, self.tp.size, max_batch, self.shape.hidden,
                                         self.embed.device, group=self.tp.group)

    def close(self) -> None:
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    def _row_parallel_fused(self, lin: nn.Module, a: Tensor, slot: int, norm_w: Tensor, bufs: _DecodeBuffers,
                            exchange: str) -> None:
        """h += (sum over ranks of) lin(a); x = RMSNorm(h) * norm_w."""
        eps = self.shape.eps
        if exchange == "push" and self.tp.size > 1:
            slot %= self.exchange.SLOTS
            if isinstance(lin, PackedGroupedBlockRVQLinear):
                self.exchange.push_gemv(lin, a, slot)  # the GEMV's epilogue stores the tagged words
            else:
                torch.matmul(a, lin.weight.t(), out=bufs.ybf)
                self.exchange.push_rows(bufs.ybf, slot)
            self.exchange.reduce_residual_norm(slot, bufs.h, norm_w, eps, bufs.x)
            return
        if isinstance(lin, PackedGroupedBlockRVQLinear):
            lin.gemv_into(a, bufs.y32)
        else:
            bufs.y32.copy_(F.linear(a, lin.weight))
        if self.tp.size > 1:
            self.tp.all_reduce_(bufs.y32)
        residual_rmsnorm(bufs.h, norm_w, eps, bufs.x, partial=bufs.y32)

    @torch.no_grad()
    def decode_step_fused(self, tokens: Tensor, pos: int, cos: Tensor, sin: Tensor, *,
                          exchange: str = "nccl") -> Tensor:
        """The decode step on this package's kernels; same inputs and result as ``decode_step``."""
        if exchange not in ("nccl", "push"):
            raise ValueError("exchange must be 'nccl' or 'push'")
        if exchange == "push" and self.tp.size > 1 and self.exchange is None:
            raise ValueError("call enable_push_exchange() before decode_step_fused(exchange='push')")
        B = tokens.shape[0]
        bufs = self._bufs.get(B)
        if bufs is None or bufs.cache_len < self.k_cache[0].shape[2]:
            bufs = self._bufs[B] = _DecodeBuffers(self, B)
        s = self.shape
        hd = s.head_dim
        torch.index_select(self.embed, 0, tokens, out=bufs.h)
        residual_rmsnorm(bufs.h, self.layers[0].in_norm, s.eps, bufs.x)
        n = len(self.layers)
        for i, (layer, kc, vc) in enumerate(zip(self.layers, self.k_cache, self.v_cache)):
            _linear_into(layer.qkv, bufs.x, bufs.qkv)
            rope_kv_append(bufs.qkv, layer.hq, layer.hkv, hd, cos, sin, pos, bufs.q, kc, vc)
            decode_attention(bufs.q, kc, vc, pos + 1, bufs.attn, bufs.attn_ws)
            self._row_parallel_fused(layer.o, bufs.attn, 2 * i, layer.post_norm, bufs, exchange)
            _linear_into(layer.gate_up, bufs.x, bufs.gu)
            silu_mul(bufs.gu, bufs.act)
            nxt = self.layers[i + 1].in_norm if i + 1 < n else self.final_norm
            self._row_parallel_fused(layer.down, bufs.act, 2 * i + 1, nxt, bufs, exchange)
        logits = F.linear(bufs.x, self.lm_head)
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


def _linear_into(lin: nn.Module, x: Tensor, y: Tensor) -> None:
    if isinstance(lin, PackedGroupedBlockRVQLinear):
        lin.gemv_into(x, y)
    else:
        torch.matmul(x, lin.weight.t(), out=y)


class DenseLinear(nn.Module):
    """bf16 linear without bias (cuBLAS through F.linear); weight [out, in]."""

    def __init__(self, weight: Tensor):
        super().__init__()
        self.out_features, self.in_features = (int(v) for v in weight.shape)
        self.register_buffer("weight", weight.contiguous())

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight)


def _shard_rows_cols(w: Tensor, rows: list[int], mode: str, tp: TPContext) -> Tensor:
    if tp.size == 1:
        return w
    if mode == COLUMN:
        parts, r = [], 0
        for n in rows:
            a, b = shard_bounds(n, tp.rank, tp.size, 16, "group rows")
            parts.append(w[r + a:r + b])
            r += n
        return torch.cat(parts)
    a, b = shard_bounds(w.shape[1], tp.rank, tp.size, 128, "in_features")
    return w[:, a:b]


def rvq_llama(shape: LlamaShape, *, device="cuda", seed: int = 0, tp: Optional[TPContext] = None) -> LlamaStack:
    """Random-init Llama-shaped stack with Block-RVQ projections (d=8, R=2, 256 entries).

    Every rank draws the full layers from the same seed and keeps its shard,
    so the shards of a tensor-parallel stack are slices of one model.
    """
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(int(seed) + 1000)
    ctx = tp or TPContext()

    def make(rows: list[int], k: int, mode: str) -> nn.Module:
        full = PackedGroupedBlockRVQLinear.random(rows, k, block_size=8, num_stages=2, entries=256,
                                                  generator=gen, device=device)
        return full if ctx.size == 1 else shard_packed(full, ctx.rank, ctx.size, mode)

    return LlamaStack(shape, make, device=device, seed=seed, tp=ctx)


def dense_llama(shape: LlamaShape, *, device="cuda", seed: int = 0, tp: Optional[TPContext] = None) -> LlamaStack:
    """The same stack with dense bf16 projections (comparison baseline)."""
    device = torch.device(device)
    gen = torch.Generator(device=device).manual_seed(int(seed) + 2000)
    ctx = tp or TPContext()

    def make(rows: list[int], k: int, mode: str) -> nn.Module:
        w = (torch.randn(int(sum(rows)), k, device=device, generator=gen) * 0.02).to(torch.bfloat16)
        return DenseLinear(_shard_rows_cols(w, rows, mode, ctx))

    return LlamaStack(shape, make, device=device, seed=seed, tp=ctx)


@torch.no_grad()
def time_decode(stack: LlamaStack, batch: int, context: int, *, steps: int = 20, warmup: int = 3,
                graph: bool = True, fused: bool = True, exchange: str = "nccl") -> dict:
    """Time one decode step at a fixed context length (cache pre-filled), optionally as a CUDA graph.

    Under tensor parallelism every rank runs this together: the timed region
    is bracketed by barriers and the reported time is the max over ranks.
    """
    import torch.distributed as dist

    tp = stack.tp
    stack.allocate_cache(batch, context + 1)
    dev = stack.embed.device
    gen = torch.Generator(device=dev).manual_seed(7)
    tokens = torch.randint(0, stack.shape.vocab, (batch,), device=dev, generator=gen)
    cos, sin = stack.rope_tables(context)
    if fused and exchange == "push" and tp.size > 1:
        stack.enable_push_exchange(batch)

    def step():
        if fused:
            return stack.decode_step_fused(tokens, context, cos, sin, exchange=exchange)
        return stack.decode_step(tokens, context, cos, sin)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(warmup):
            g.replay()
    torch.cuda.synchronize()
    if tp.size > 1:
        dist.barrier(group=tp.group)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        if g is not None:
            g.replay()
        else:
            step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if tp.size > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=tp.group)
        ms = float(t.item())
    if stack.exchange is not None:
        stack.exchange.check_status()
    del g
    return {"ms_per_step": ms, "tok_s": batch * 1e3 / ms, "batch": batch, "context": context,
            "fused": fused, "exchange": exchange if tp.size > 1 else "none", "tp": tp.size}
