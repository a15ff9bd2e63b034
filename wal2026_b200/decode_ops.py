"""Decode-step glue kernels of the Llama-shaped stacks (C ABI wrappers).

``residual_rmsnorm``, ``rope_kv_append`` and ``silu_mul`` run the glue
between the Block-RVQ linears of a decoder block as three sm_100a kernels
(see ``csrc/wal_decode_glue.cu``) instead of a dozen PyTorch operators.  Each
call launches on the current stream; none has a CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _abi


def _cuda(*ts: Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("decode ops run on CUDA tensors only")


def residual_rmsnorm(h: Tensor, norm_w: Tensor, eps: float, x_out: Tensor, partial: Optional[Tensor] = None) -> None:
    """h <- bf16(h + bf16(partial)) (when given), x_out <- bf16(RMSNorm(h) * norm_w).

    h, x_out: bf16 [M, N]; partial: fp32 [M, N] (one local partial output).
    """
    _cuda(h, norm_w, x_out)
    M, N = h.shape
    lib = _abi.load()
    if partial is not None:
        _cuda(partial)
        if partial.dtype != torch.float32 or tuple(partial.shape) != (M, N):
            raise ValueError("partial must be fp32 [M, N]")
    st = lib.wal_residual_rmsnorm(None if partial is None else partial.data_ptr(),
                                  N if partial is None else partial.stride(0), h.data_ptr(), h.stride(0),
                                  norm_w.data_ptr(), float(eps), x_out.data_ptr(), x_out.stride(0), M, N,
                                  _abi.stream_handle(h.device))
    _abi.check(st, "wal_residual_rmsnorm")


def rope_kv_append(qkv: Tensor, hq: int, hkv: int, hd: int, cos: Tensor, sin: Tensor, pos: int, q_out: Tensor,
                   k_cache: Tensor, v_cache: Tensor) -> None:
    """RoPE of q/k at `pos` (q -> q_out [M, hq*hd]) and append k, v to the caches [M, hkv, L, hd]."""
    _cuda(qkv, cos, sin, q_out, k_cache, v_cache)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous() and q_out.is_contiguous()):
        raise ValueError("caches and q_out must be contiguous")
    if cos.dtype != torch.float32 or sin.dtype != torch.float32:
        raise ValueError("cos/sin tables must be fp32 [head_dim]")
    lib = _abi.load()
    st = lib.wal_rope_kv_append(qkv.data_ptr(), qkv.stride(0), qkv.shape[0], hq, hkv, hd, cos.data_ptr(),
                                sin.data_ptr(), int(pos), q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                k_cache.shape[2], _abi.stream_handle(qkv.device))
    _abi.check(st, "wal_rope_kv_append")


def silu_mul(gu: Tensor, out: Tensor) -> None:
    """out[:, :I] = bf16(bf16(silu(gu[:, :I])) * gu[:, I:2I])."""
    _cuda(gu, out)
    M, I = out.shape
    lib = _abi.load()
    st = lib.wal_silu_mul(gu.data_ptr(), gu.stride(0), M, I, out.data_ptr(), out.stride(0),
                          _abi.stream_handle(gu.device))
    _abi.check(st, "wal_silu_mul")


def decode_attention_workspace(B: int, hq: int, hkv: int, hd: int, max_len: int, device) -> Tensor:
    """Zero-filled scratch for ``decode_attention`` calls with up to ``max_len`` positions."""
    nbytes = int(_abi.load().wal_decode_attention_workspace(B, hq, hkv, hd, max_len))
    if nbytes == 0:
        raise ValueError("invalid attention shape")
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def decode_attention(q: Tensor, k_cache: Tensor, v_cache: Tensor, n: int, out: Tensor, workspace: Tensor,
                     scale: Optional[float] = None) -> None:
    """out[b] = softmax(q[b] k^T * scale) v over cache positions [0, n) (grouped-query heads).

    q, out: bf16 [B, hq * hd]; caches: bf16 [B, hkv, cache_len, hd] contiguous;
    ``workspace`` from ``decode_attention_workspace`` (not shared by overlapping calls).
    """
    _cuda(q, k_cache, v_cache, out, workspace)
    B, hkv, L, hd = (int(v) for v in k_cache.shape)
    hq = int(q.shape[1]) // hd
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    scale = float(hd) ** -0.5 if scale is None else float(scale)
    lib = _abi.load()
    st = lib.wal_decode_attention(q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), B, hq, hkv, hd,
                                  L, int(n), scale, out.data_ptr(), out.stride(0), workspace.data_ptr(),
                                  workspace.numel(), _abi.stream_handle(q.device))
    _abi.check(st, "wal_decode_attention")

