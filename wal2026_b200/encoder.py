"""Block-RVQ encoder on the GPU (reference ``src/block_vq.py:199-531``).

Residual vector quantisation of a weight matrix: rows are scaled by their
absolute maximum (fp16 row scale), split into blocks of ``block_size`` columns
(optionally normalised per block, optionally split into product sub-blocks),
and every stage fits a k-means codebook on a seeded sample of the residual
blocks, assigns all blocks to their nearest entry and subtracts it.

The assignments, the inner loop of both the fit and the full pass, run in
``wal_rvq_assign`` (CUDA); the k-means bookkeeping (initial entries,
centroid means, reseeding of empty entries) follows the reference's
``_fit_kmeans`` with the same seeded CPU generator draws, so the same inputs
give the same initial codebook.  Centroid sums are accumulated in float64
(order-independent to fp32 precision) and rounded to fp32, where the
reference sums in fp32 in index order; a block whose two best entries are
within a few fp32 units can therefore be assigned differently, after which
the two fits may drift apart slightly.  The result is a ``BlockRVQEncoding``
that this package's kernels (and the reference) decode.

Supported: plain stages, product splits (``stages_per_split``) and block
normalisation (``normalize_blocks``); transforms, sign residuals and
stage-scale calibration raise ``ValueError``.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _abi
from .block_vq import BlockRVQEncoding


def assign_to_codebook(blocks: Tensor, codebook: Tensor) -> tuple[Tensor, Tensor]:
    """Nearest entry of every block (reference ``_assign_to_codebook``): (int64 ids, fp32 minimum distances)."""
    if not blocks.is_cuda:
        raise ValueError("assign_to_codebook runs on CUDA only")
    if blocks.ndim != 2 or codebook.ndim != 2 or blocks.shape[1] != codebook.shape[1]:
        raise ValueError("blocks [n, d] and codebook [entries, d] must share d")
    if blocks.shape[0] == 0:
        raise ValueError("blocks must be non-empty")
    x = blocks.to(torch.float32).contiguous()
    cb = codebook.to(device=x.device, dtype=torch.float32).contiguous()
    ids = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    dist = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        st = _abi.load().wal_rvq_assign(x.data_ptr(), x.shape[0], x.shape[1], cb.data_ptr(), cb.shape[0],
                                        ids.data_ptr(), dist.data_ptr(), _abi.stream_handle(x.device))
    _abi.check(st, "wal_rvq_assign")
    return ids.to(torch.int64), dist


def fit_kmeans(blocks: Tensor, codebook_size: int, iters: int) -> Tensor:
    """k-means codebook of ``blocks`` (reference ``_fit_kmeans``, ``src/block_vq.py:199-227``).

    Initial entries: the blocks at the first ``codebook_size`` positions of a
    permutation drawn from a CPU generator seeded with 0; each iteration
    assigns, replaces every used entry by the mean of its blocks and reseeds
    empty entries with blocks drawn from the same generator.
    """
    if blocks.ndim != 2:
        raise ValueError("expected 2D blocks")
    n = int(blocks.shape[0])
    if n < codebook_size:
        raise ValueError("sample set must be at least as large as codebook_size")
    x = blocks.to(torch.float32)
    gen = torch.Generator(device="cpu").manual_seed(0)
    perm = torch.randperm(n, generator=gen)
    codebook = x[perm[:codebook_size].to(x.device)].clone()
    for _ in range(iters):
        ids, _ = assign_to_codebook(x, codebook)
        counts = torch.bincount(ids, minlength=codebook_size)
        sums = torch.zeros(codebook_size, x.shape[1], dtype=torch.float64, device=x.device)
        sums.index_add_(0, ids, x.to(torch.float64))
        used = counts > 0
        updated = codebook.clone()
        updated[used] = sums[used].to(torch.float32) / counts[used].to(torch.float32).unsqueeze(1)
        empty = (~used).nonzero(as_tuple=True)[0]
        if empty.numel() > 0:
            reseed = torch.randint(0, n, (int(empty.numel()),), generator=gen)
            updated[empty] = x[reseed.to(x.device)]
        codebook = updated
    return codebook


@torch.no_grad()
def encode_block_rvq(weight: Tensor, *, block_size: int = 32, codebook_size: int = 256, num_stages: int = 2,
                     product_splits: int = 1, stages_per_split: Optional[tuple[int, ...]] = None,
                     normalize_blocks: str = "none", transform_kind: str = "none",
                     calibrate_stage_scales: bool = False, residual_correction: str = "none",
                     sample_limit: int = 131_072, kmeans_iters: int = 8) -> BlockRVQEncoding:
    """Encode a 2-D weight on its CUDA device (reference ``encode_block_residual_vq`` arguments)."""
    if weight.ndim != 2:
        raise ValueError("expected 2D weight")
    if not weight.is_cuda:
        raise ValueError("encode_block_rvq runs on CUDA only")
    if transform_kind != "none" or residual_correction != "none" or calibrate_stage_scales:
        raise ValueError("the GPU encoder covers plain stages, product splits and block normalisation")
    if num_stages < 1:
        raise ValueError("num_stages must be >= 1")
    if product_splits < 1 or block_size % product_splits != 0:
        raise ValueError("product_splits must divide block_size and be >= 1")
    counts = tuple(int(num_stages) for _ in range(product_splits)) if stages_per_split is None \
        else tuple(int(c) for c in stages_per_split)
    if len(counts) != product_splits or any(c < 1 for c in counts):
        raise ValueError("stages_per_split must have product_splits entries, each >= 1")
    dev = weight.device
    rows, cols = (int(v) for v in weight.shape)
    row_scale = weight.abs().amax(dim=-1, keepdim=True).clamp_min(1e-8).to(torch.float16)
    w_norm = weight.to(torch.float32) / row_scale.to(torch.float32)
    padded = -(-cols // block_size) * block_size
    if padded != cols:
        w_norm = torch.nn.functional.pad(w_norm, (0, padded - cols), value=0.0)
    nb = padded // block_size
    blocks = w_norm.reshape(rows * nb, block_size)
    block_scale = None
    if normalize_blocks == "amax":
        block_scale = blocks.abs().amax(dim=1, keepdim=True).clamp_min(1e-8)
        blocks = blocks / block_scale
    elif normalize_blocks == "l2":
        block_scale = blocks.square().mean(dim=1, keepdim=True).sqrt().clamp_min(1e-8)
        blocks = blocks / block_scale
    elif normalize_blocks != "none":
        raise ValueError("normalize_blocks must be one of: none, amax, l2")
    residual = blocks.clone()
    sample_limit = max(int(sample_limit), int(codebook_size))
    gen = torch.Generator(device="cpu").manual_seed(0)
    pick = torch.randperm(residual.shape[0], generator=gen)[:min(sample_limit, residual.shape[0])].to(dev)
    sample = residual[pick].clone()
    id_dtype = torch.uint8 if codebook_size <= 256 else (torch.int16 if codebook_size <= 32767 else torch.int32)
    stage_ids, codebooks, value_dims = [], [], []
    sub = block_size // product_splits
    for split, count in enumerate(counts):
        lo, hi = split * sub, (split + 1) * sub
        for _ in range(count):
            cb = fit_kmeans(sample[:, lo:hi], codebook_size, kmeans_iters)
            ids, _ = assign_to_codebook(residual[:, lo:hi].contiguous(), cb)
            residual[:, lo:hi] -= cb[ids]
            sids, _ = assign_to_codebook(sample[:, lo:hi].contiguous(), cb)
            sample[:, lo:hi] -= cb[sids]
            full = torch.zeros(codebook_size, block_size, dtype=torch.float32, device=dev)
            full[:, lo:hi] = cb
            stage_ids.append(ids.view(rows, nb).to(id_dtype))
            codebooks.append(full.to(torch.float16))
            value_dims.append(sub if product_splits > 1 else block_size)
    # the reported error uses the stored (fp16) codebooks, as the decoder sees them
    recon = torch.zeros_like(blocks)
    for ids, cb in zip(stage_ids, codebooks):
        recon += cb.to(torch.float32)[ids.reshape(-1).to(torch.int64)]
    sample_rel = float(((blocks[pick] - recon[pick]).square().mean() / blocks[pick].square().mean().clamp_min(1e-12)))
    return BlockRVQEncoding(
        stage_ids=tuple(stage_ids), codebooks=tuple(codebooks), stage_value_dims=tuple(value_dims),
        stages_per_split=counts, stage_scales=None, residual_correction="none", residual_signs=None,
        residual_scale=None, row_scale=row_scale,
        block_scale=None if block_scale is None else block_scale.view(rows, nb).to(torch.float16),
        transform_kind="none", transform_matrix=None, transform_bias=None, product_splits=product_splits,
        original_shape=(rows, cols), padded_cols=padded, block_size=block_size, sample_rel_mse=sample_rel,
    )


__all__ = ["assign_to_codebook", "fit_kmeans", "encode_block_rvq"]
