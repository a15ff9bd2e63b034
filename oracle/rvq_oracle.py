"""CPU oracle for the Block-RVQ runtime linear: TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the reference's dequantise-then-matmul path
(``matmul_strategy="per_group"``) so that tests can check the CUDA kernels
against it.  Nothing in the product imports it: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may.

Algorithm followed, with the reference lines it restates:

* ``PackedBlockRVQGroup.reconstruct_weight`` (reference
  ``src/runtime.py:379-414``): an fp32 accumulator starts at +0.0; for each
  stage in order, ``recon += float32(codebook[ids])`` (``:383-388``); the
  plain encodings used here skip the optional corrections (``:389-412``); the
  result is sliced to ``in_features`` columns, rounded to bf16 and multiplied
  by the bf16-rounded fp16 row scale, the product being rounded to bf16 again
  (``:413-414``).
* ``PackedGroupedBlockRVQLinear.forward`` default branch (reference
  ``src/runtime.py:1501-1507``): per row group ``F.linear(x, weight, bias)``
  with bf16 operands and the groups concatenated along the output dimension.
  The oracle accumulates that product exactly (float64 over exact bf16*bf16
  products), which is the fp32-accumulate result up to accumulation order.

Rounding helpers follow PyTorch's float -> bfloat16 conversion
(round-to-nearest-even on the fp32 bit pattern, NaN -> 0x7FC0), which the
reference uses through ``Tensor.to(torch.bfloat16)``.

Parity of this restatement is pinned by ``tests/golden/`` fixtures produced by
running the reference itself (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 (RNE), returned as uint16 bit patterns."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> np.uint64(16)) & np.uint64(1)
    r = ((u + np.uint64(0x7FFF) + lsb) >> np.uint64(16)).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = np.uint16(0x7FC0)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def stage_sum_f32(stage_ids: list[np.ndarray], codebooks: list[np.ndarray],
                  stage_scales: np.ndarray | None = None) -> np.ndarray:
    """fp32 sum of the gathered stage entries, ``[rows, blocks, d]`` (``src/runtime.py:381-388``).

    With per-stage scales each stage is multiplied in fp32 before it is added
    (``src/block_vq.py:264-268``).
    """
    rows, blocks = stage_ids[0].shape
    d = codebooks[0].shape[1]
    acc = np.zeros((rows, blocks, d), dtype=np.float32)
    for s, (ids, book) in enumerate(zip(stage_ids, codebooks)):
        entries = np.asarray(book, dtype=np.float16).astype(np.float32)
        stage = entries[np.asarray(ids).astype(np.int64)]
        if stage_scales is not None:
            stage = stage * np.asarray(stage_scales, dtype=np.float32).reshape(-1)[s]
        acc += stage
    return acc


def reconstruct_group_bits(
    stage_ids: list[np.ndarray],
    codebooks: list[np.ndarray],
    row_scale: np.ndarray,
    in_features: int,
    stage_scales: np.ndarray | None = None,
) -> np.ndarray:
    """bf16 weight bits ``[rows, in_features]`` of one plain group (``src/runtime.py:379-414``)."""
    acc = stage_sum_f32(stage_ids, codebooks, stage_scales)
    rows = acc.shape[0]
    w = acc.reshape(rows, -1)[:, :in_features]
    w_bf = bf16_bits_to_f32(f32_to_bf16_bits(w))
    rho = np.asarray(row_scale, dtype=np.float16).astype(np.float32).reshape(rows, 1)
    rho_bf = bf16_bits_to_f32(f32_to_bf16_bits(rho))
    return f32_to_bf16_bits(w_bf * rho_bf)


def _round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the weight type, returned as float32 values of that type."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(a))
    if dtype == "f16":
        return a.astype(np.float16).astype(np.float32)
    return a


def reconstruct_group_typed(stage_ids: list[np.ndarray], codebooks: list[np.ndarray], row_scale: np.ndarray,
                            in_features: int, dtype: str = "bf16", mode: str = "exact",
                            stage_scales: np.ndarray | None = None) -> np.ndarray:
    """Weight values (float32 array holding ``dtype`` values) of one group.

    ``mode="exact"`` restates ``reconstruct_weight(out_dtype)`` (reference
    ``src/runtime.py:379-414``): fp32 stage sum from +0.0 (stage scales applied
    in fp32), rounded to ``dtype``, times the ``dtype``-rounded row scale with
    one more rounding (fp32 keeps the fp32 product).
    ``mode="fast"`` restates ``reconstruct_weight_fast`` (``src/runtime.py:431-448``,
    ``:568-598``): every stage table converted to ``dtype`` (times the
    ``dtype``-rounded stage scale, rounded), the gathered stages added in
    ``dtype`` in order starting from the first stage's value, then the row
    scale multiply rounded to ``dtype``.  Sums and products of two bf16 or fp16
    values are formed in float32 and rounded once, which equals the rounded
    exact result for these types.
    """
    rho = _round_to(np.asarray(row_scale, dtype=np.float16).astype(np.float32).reshape(-1, 1), dtype)
    if mode == "exact":
        acc = stage_sum_f32(stage_ids, codebooks, stage_scales)
        w = acc.reshape(acc.shape[0], -1)[:, :in_features]
        return _round_to(_round_to(w, dtype) * rho, dtype)
    if mode != "fast":
        raise ValueError(f"unknown mode {mode!r}")
    acc = None
    for s, (ids, book) in enumerate(zip(stage_ids, codebooks)):
        table = _round_to(np.asarray(book, dtype=np.float16).astype(np.float32), dtype)
        if stage_scales is not None:
            sc = _round_to(np.float32(np.asarray(stage_scales, dtype=np.float32).reshape(-1)[s]), dtype)
            table = _round_to(table * sc, dtype)
        v = table[np.asarray(ids).astype(np.int64)]
        acc = v if acc is None else _round_to(acc + v, dtype)
    w = acc.reshape(acc.shape[0], -1)[:, :in_features]
    return _round_to(w * rho, dtype)


def _hadamard_t(n: int):
    """Normalised Sylvester Hadamard matrix as the reference builds it (torch, ``src/block_vq.py:10-22``)."""
    import math

    import torch

    mat = torch.tensor([[1.0]], dtype=torch.float32)
    while mat.shape[0] < n:
        mat = torch.cat((torch.cat((mat, mat), dim=1), torch.cat((mat, -mat), dim=1)), dim=0)
    return mat / math.sqrt(float(n))


def _rand_hadamard(n: int) -> np.ndarray:
    """The randomised Hadamard / sign-correction matrix (reference ``src/block_vq.py:25-35``, ``:106-107``):
    rows permuted and signed by draws from a CPU generator seeded with 0, in the reference's order."""
    import torch

    base = _hadamard_t(n)
    gen = torch.Generator(device="cpu").manual_seed(0)
    perm = torch.randperm(n, generator=gen)
    flip = torch.randint(0, 2, (n,), generator=gen, dtype=torch.int64) > 0
    signs = torch.where(flip, torch.ones(n), -torch.ones(n))
    return (base[perm] * signs.unsqueeze(1)).numpy()


def _fixed_transform(kind: str, n: int) -> np.ndarray | None:
    """DCT / Hadamard / randomised Hadamard matrices (reference ``src/block_vq.py:10-61``)."""
    if kind == "hadamard":
        return _hadamard_t(n).numpy()
    if kind == "rand_hadamard":
        return _rand_hadamard(n)
    if kind == "dct":
        import math

        import torch

        idx = torch.arange(n, dtype=torch.float32)
        mat = torch.cos(math.pi / float(n) * (idx + 0.5)[None, :] * idx[:, None])
        mat[0] *= math.sqrt(1.0 / float(n))
        if n > 1:
            mat[1:] *= math.sqrt(2.0 / float(n))
        return mat.numpy()
    return None


def _matmul_rows(v: np.ndarray, m: np.ndarray) -> np.ndarray:
    """Rows of v times m: each output the exact dot product rounded once to float32."""
    return (v.astype(np.float64) @ m.astype(np.float64)).astype(np.float32)


def apply_corrections(acc: np.ndarray, g: dict) -> np.ndarray:
    """Per-block corrections of reference ``src/runtime.py:389-412`` on fp32 block vectors ``[rows, blocks, d]``.

    Sign residual ``(sigma * residual_scale) @ H``, block scale, inverse polar
    transform or ``@ M`` (DCT, Hadamard, randomised Hadamard or the stored PCA
    matrix), transform bias - in that order, in float32 (matrix products as
    exact dot products rounded once; the reference's CPU matrix product may
    differ from that in the last bit).
    """
    rows, blocks, d = acc.shape
    v = acc.reshape(rows * blocks, d).astype(np.float32)
    if g.get("residual_signs") is not None and g.get("residual_scale") is not None \
            and g.get("residual_correction", "sign") != "none":
        words = np.asarray(g["residual_signs"]).astype(np.int64).reshape(rows * blocks, -1)
        bits = np.stack([(words[:, c // 32] >> (c % 32)) & 1 for c in range(d)], axis=1)
        sigma = np.where(bits == 1, np.float32(1.0), np.float32(-1.0)).astype(np.float32)
        rs = np.asarray(g["residual_scale"], dtype=np.float16).astype(np.float32).reshape(-1, 1)
        v = (v + _matmul_rows(sigma * rs, _rand_hadamard(d))).astype(np.float32)
    if g.get("block_scale") is not None:
        v = (v * np.asarray(g["block_scale"], dtype=np.float16).astype(np.float32).reshape(-1, 1)).astype(np.float32)
    kind = g.get("transform_kind", "none")
    if kind == "polar":
        cur = v[:, :1]
        offset, width = 1, 1
        while width < d:
            ang = (np.float32(np.pi) * v[:, offset:offset + width]).astype(np.float32)
            cur = np.stack((cur * np.cos(ang), cur * np.sin(ang)), axis=-1).reshape(v.shape[0], 2 * width)
            cur = cur.astype(np.float32)
            offset += width
            width *= 2
        v = cur
    else:
        m = g.get("transform_matrix")
        m = _fixed_transform(kind, d) if m is None else np.asarray(m, dtype=np.float16).astype(np.float32)
        if m is not None:
            v = _matmul_rows(v, m)
    if g.get("transform_bias") is not None:
        v = (v + np.asarray(g["transform_bias"], dtype=np.float16).astype(np.float32).reshape(1, d)).astype(np.float32)
    return v.reshape(rows, blocks, d)


def reconstruct_group_corrected(g: dict, in_features: int, dtype: str = "bf16") -> np.ndarray:
    """Weight values of one group with per-block corrections (exact reconstruction, ``dtype`` values in float32)."""
    acc = apply_corrections(stage_sum_f32(g["stage_ids"], g["codebooks"], g.get("stage_scales")), g)
    rho = _round_to(np.asarray(g["row_scale"], dtype=np.float16).astype(np.float32).reshape(-1, 1), dtype)
    w = acc.reshape(acc.shape[0], -1)[:, :in_features]
    return _round_to(_round_to(w, dtype) * rho, dtype)


def reconstruct_typed(groups: list[dict], in_features: int, dtype: str = "bf16", mode: str = "exact") -> np.ndarray:
    """Concatenated group weights in ``dtype`` for either reconstruction mode (float32 values)."""
    parts = []
    for g in groups:
        if g.get("corrected"):
            parts.append(reconstruct_group_corrected(g, in_features, dtype))
        else:
            parts.append(reconstruct_group_typed(g["stage_ids"], g["codebooks"], g["row_scale"], in_features, dtype,
                                                 mode, g.get("stage_scales")))
    return np.concatenate(parts, axis=0)


def reconstruct_bits(groups: list[dict], in_features: int) -> np.ndarray:
    """Concatenate per-group weights (``PackedGroupedBlockRVQLinear.reconstruct_weight``, ``src/runtime.py:1234-1236``).

    Each group is a dict with ``stage_ids`` (list of ``[rows, blocks]`` int arrays),
    ``codebooks`` (list of ``[entries, d]`` fp16 arrays) and ``row_scale``.
    """
    parts = [reconstruct_group_bits(g["stage_ids"], g["codebooks"], g["row_scale"], in_features,
                                    g.get("stage_scales")) for g in groups]
    return np.concatenate(parts, axis=0)


def linear_exact(x_bits: np.ndarray, w_bits: np.ndarray, bias_bits: np.ndarray | None = None) -> np.ndarray:
    """``y = x @ w.T (+ bias)`` over bf16 operands, accumulated in float64 (``src/runtime.py:1505``)."""
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    y = x @ w.T
    if bias_bits is not None:
        y = y + bf16_bits_to_f32(bias_bits).astype(np.float64)[None, :]
    return y


def forward_f32(x_bits: np.ndarray, groups: list[dict], in_features: int,
                bias_bits: np.ndarray | None = None) -> np.ndarray:
    """fp32 (pre-output-rounding) result of the per_group forward."""
    w = reconstruct_bits(groups, in_features)
    return linear_exact(x_bits, w, bias_bits).astype(np.float32)


def unpack_route_code(ids: np.ndarray, entries_per_route: int = 256) -> tuple[np.ndarray, np.ndarray]:
    """Split single-stage routed ids ``route * entries + code`` back into (route, code)."""
    ids = np.asarray(ids).astype(np.int64)
    return (ids // entries_per_route).astype(np.uint8), (ids % entries_per_route).astype(np.uint8)


def groups_from_encoding(enc) -> list[dict]:
    """Convert a (grouped) encoding object with torch tensors into oracle group dicts."""
    groups = enc.groups if hasattr(enc, "groups") else (enc,)
    out = []
    for g in groups:
        out.append(
            {
                "stage_ids": [t.cpu().numpy() for t in g.stage_ids],
                "codebooks": [t.cpu().numpy().astype(np.float16) for t in g.codebooks],
                "row_scale": g.row_scale.cpu().numpy(),
                "stage_scales": None if getattr(g, "stage_scales", None) is None
                else g.stage_scales.cpu().float().numpy(),
            }
        )
        if hasattr(g, "is_plain") and not g.is_plain():
            out[-1].update({
                "corrected": True,
                "residual_correction": g.residual_correction,
                "residual_signs": None if g.residual_signs is None else g.residual_signs.cpu().numpy(),
                "residual_scale": None if g.residual_scale is None else g.residual_scale.cpu().numpy(),
                "block_scale": None if g.block_scale is None else g.block_scale.cpu().numpy(),
                "transform_kind": g.transform_kind,
                "transform_matrix": None if g.transform_matrix is None else g.transform_matrix.cpu().numpy(),
                "transform_bias": None if g.transform_bias is None else g.transform_bias.cpu().numpy(),
            })
    return out


# ---------------------------------------------------------------------------
# ID-route linear (reference src/runtime.py:52-97, PackedIDRouteLinear)
# ---------------------------------------------------------------------------
def idroute_weight_f16_bits(ids: np.ndarray, codebook_sum_bits: np.ndarray, row_scale_bits: np.ndarray) -> np.ndarray:
    """fp16 weight bits of ``reconstruct_weight`` (src/runtime.py:89-93): gather, times row scale, fp16 rounding.

    The product of two fp16 values is exact in float32, so one float32 multiply
    followed by the round-to-nearest-even cast to float16 is the fp16 multiply.
    """
    cs = np.asarray(codebook_sum_bits, dtype=np.uint16).view(np.float16).astype(np.float32)
    rho = np.asarray(row_scale_bits, dtype=np.uint16).view(np.float16).astype(np.float32).reshape(-1, 1)
    w = (cs[np.asarray(ids).astype(np.int64)] * rho).astype(np.float16)
    return w.view(np.uint16)


def idroute_weight_bits(ids: np.ndarray, codebook_sum_bits: np.ndarray, row_scale_bits: np.ndarray) -> np.ndarray:
    """bf16 weight bits of the forward (src/runtime.py:95-97: ``w.to(x.dtype)``)."""
    w16 = idroute_weight_f16_bits(ids, codebook_sum_bits, row_scale_bits).view(np.float16)
    return f32_to_bf16_bits(w16.astype(np.float32))



# ---------------------------------------------------------------------------
# Encoder (reference src/block_vq.py:180-196, _assign_to_codebook)
# ---------------------------------------------------------------------------
def assign_to_codebook(blocks: np.ndarray, codebook: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Nearest entry per block: argmin of ||x||^2 + ||c||^2 - 2 x.c in float32 (first minimum on ties)."""
    x = np.asarray(blocks, dtype=np.float32)
    c = np.asarray(codebook, dtype=np.float32)
    xsq = (x * x).sum(axis=1, dtype=np.float32)[:, None]
    csq = (c * c).sum(axis=1, dtype=np.float32)[None, :]
    dot = (x @ c.T).astype(np.float32)
    dist = ((xsq + csq).astype(np.float32) - np.float32(2.0) * dot).astype(np.float32)
    ids = dist.argmin(axis=1)
    return ids, dist[np.arange(x.shape[0]), ids]
