"""Generate golden fixtures by running the reference implementation itself.

Run in a container that has the reference source tree (it is not needed, and
not present, where the tests run):

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

For every case the script builds the synthetic encoding with
``wal2026_b200.synthetic`` (seeded, fixed draw order), converts it into the
reference's own ``BlockRVQEncoding``/``GroupedBlockRVQEncoding`` dataclasses,
wraps it in the reference's ``PackedGroupedBlockRVQLinear`` with
``matmul_strategy="per_group"`` (the dequantise-then-matmul path) and records:

* ``w_bits``/``w_sha256`` - the bf16 weight from ``reconstruct_weight(torch.bfloat16)``;
* ``y_ref_bf16``          - the reference forward output (bf16 bits);
* ``y_ref32``             - ``x.float() @ W.float().T (+ bias)`` accumulated in float64;
* SHA-256 digests of every input array, so the tests can prove that the
  synthetic generator still produces the same bytes.

ID-route cases (``idroute_*``) run the reference's ``PackedIDRouteLinear``
and record its route table, fp16 ``reconstruct_weight()`` and forward output.

Small cases store all arrays; the two full-size configurations store input
digests, the weight digest and a bounded slice of the outputs.
"""
from __future__ import annotations

import argparse
import dataclasses
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from wal2026_b200 import synthetic  # noqa: E402
from wal2026_b200.block_vq import BlockRVQEncoding, GroupedBlockRVQEncoding, single_group  # noqa: E402


def sha(t: torch.Tensor | np.ndarray) -> str:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            t = t.view(torch.int16)
        t = t.numpy()
    return hashlib.sha256(np.ascontiguousarray(t).tobytes()).hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def to_reference(enc: GroupedBlockRVQEncoding, ref_block_vq):
    groups = []
    for g in enc.groups:
        kwargs = {f.name: getattr(g, f.name) for f in dataclasses.fields(ref_block_vq.BlockRVQEncoding)}
        groups.append(ref_block_vq.BlockRVQEncoding(**kwargs))
    return ref_block_vq.GroupedBlockRVQEncoding(groups=tuple(groups), row_slices=enc.row_slices,
                                                original_shape=enc.original_shape)


def run_case(name, enc, Ms, x_seed, bias, ref_runtime, ref_block_vq, *, full: bool, y_rows: int | None = None,
             extra: dict | None = None):
    ref_enc = to_reference(enc, ref_block_vq)
    mod = ref_runtime.PackedGroupedBlockRVQLinear(ref_enc, bias, matmul_strategy="per_group")
    with torch.no_grad():
        w = mod.reconstruct_weight(torch.bfloat16)
    out = {"name": np.array(name), "w_sha256": np.array(sha(w)),
           "N": np.array(enc.original_shape[0]), "K": np.array(enc.original_shape[1])}
    if full:
        out["w_bits"] = bits(w)
    for gi, g in enumerate(enc.groups):
        for s, (ids, book) in enumerate(zip(g.stage_ids, g.codebooks)):
            out[f"g{gi}_ids{s}_sha256"] = np.array(sha(ids))
            out[f"g{gi}_book{s}_sha256"] = np.array(sha(book))
            if full:
                out[f"g{gi}_ids{s}"] = ids.numpy()
                out[f"g{gi}_book{s}"] = book.numpy()
        out[f"g{gi}_rho_sha256"] = np.array(sha(g.row_scale))
        if full:
            out[f"g{gi}_rho"] = g.row_scale.numpy()
            if g.stage_scales is not None:
                out[f"g{gi}_scales"] = g.stage_scales.numpy()
    if bias is not None:
        out["bias_bits"] = bits(bias)
    for key, value in (extra or {}).items():
        out[key] = np.array(value)
    for M in Ms:
        x = synthetic.activations(M, enc.original_shape[1], seed=x_seed)
        with torch.no_grad():
            y = mod(x)
        y32 = x.double() @ w.double().T
        if bias is not None:
            y32 = y32 + bias.double()[None, :]
        rows = slice(None) if y_rows is None else slice(0, y_rows)
        out[f"x{M}_sha256"] = np.array(sha(x))
        if full:
            out[f"x{M}_bits"] = bits(x)
        out[f"y{M}_ref32"] = y32[:, rows].float().numpy()
        out[f"y{M}_ref_bf16"] = bits(y[:, rows])
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz  w_sha256={out['w_sha256']}")


def run_idroute_case(name, inp, Ms, x_seed, bias, ref_runtime):
    """Reference PackedIDRouteLinear (src/runtime.py:52-97) on seeded inputs."""
    mod = ref_runtime.PackedIDRouteLinear(inp.ids, inp.codebook_w, inp.row_scale, bias)
    with torch.no_grad():
        w16 = mod.reconstruct_weight()
    wb = w16.to(torch.bfloat16)
    out = {"name": np.array(name), "N": np.array(inp.ids.shape[0]), "K": np.array(inp.ids.shape[1]),
           "ids": inp.ids.to(torch.int16).numpy(), "codebook_w_bits": bits(inp.codebook_w),
           "codebook_sum_bits": bits(mod.codebook_sum), "rho_bits": bits(inp.row_scale.reshape(-1)),
           "w16_bits": bits(w16), "w16_sha256": np.array(sha(w16))}
    if bias is not None:
        out["bias_f16_bits"] = bits(bias)
    for M in Ms:
        x = synthetic.activations(M, inp.ids.shape[1], seed=x_seed)
        with torch.no_grad():
            y = mod(x)
        y32 = x.double() @ wb.double().T
        if bias is not None:
            y32 = y32 + bias.to(torch.bfloat16).double()[None, :]
        out[f"x{M}_bits"] = bits(x)
        out[f"y{M}_ref32"] = y32.float().numpy()
        out[f"y{M}_ref_bf16"] = bits(y)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz  w16_sha256={out['w16_sha256']}")


def run_stage_drop_case(name, enc, k, Ms, x_seed, ref_runtime, ref_block_vq):
    """Reference variable-stage decoding (src/runtime.py:352-377, :568-598): effective_stages_per_split = k
    under the full_weight_fast strategy, which sums only the active stages (in bf16)."""
    ref_enc = to_reference(enc, ref_block_vq)
    mod = ref_runtime.PackedGroupedBlockRVQLinear(ref_enc, None, matmul_strategy="full_weight_fast")
    n = ref_runtime.set_global_effective_stages(mod, k)
    active = [list(g._compute_active_stage_indices()) for g in mod.groups]
    with torch.no_grad():
        w_full = mod.reconstruct_weight(torch.bfloat16)
        w_fast = mod.reconstruct_weight_fast(torch.bfloat16)
    out = {"name": np.array(name), "k": np.array(k), "groups_updated": np.array(n),
           "N": np.array(enc.original_shape[0]), "K": np.array(enc.original_shape[1]),
           "w_bits": bits(w_full), "w_fast_bits": bits(w_fast), "stages_per_split": np.array(
               [list(g.stages_per_split) for g in enc.groups])}
    for gi, (g, act) in enumerate(zip(enc.groups, active)):
        out[f"g{gi}_active"] = np.array(act)
        for s, (ids, book) in enumerate(zip(g.stage_ids, g.codebooks)):
            out[f"g{gi}_ids{s}"] = ids.numpy()
            out[f"g{gi}_book{s}"] = book.numpy()
        out[f"g{gi}_rho"] = g.row_scale.numpy()
    for M in Ms:
        x = synthetic.activations(M, enc.original_shape[1], seed=x_seed)
        with torch.no_grad():
            y = mod(x)
        out[f"x{M}_bits"] = bits(x)
        out[f"y{M}_fast32"] = (x.double() @ w_fast.double().T).float().numpy()
        out[f"y{M}_fast_bf16"] = bits(y)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz  active={active}")


def f16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def run_dtype_case(name, enc, Ms, x_seed, bias, ref_runtime, ref_block_vq):
    """The reference forward in float16 and float32 (src/runtime.py:1501-1507 builds the weight with
    reconstruct_weight(x.dtype), :379-414) and its fast reconstruction (:568-598) in every dtype."""
    ref_enc = to_reference(enc, ref_block_vq)
    exact = ref_runtime.PackedGroupedBlockRVQLinear(ref_enc, bias, matmul_strategy="per_group")
    fast = ref_runtime.PackedGroupedBlockRVQLinear(ref_enc, bias, matmul_strategy="full_weight_fast")
    with torch.no_grad():
        w16 = exact.reconstruct_weight(torch.float16)
        w32 = exact.reconstruct_weight(torch.float32)
        wf16 = fast.reconstruct_weight_fast(torch.float16)
        wfb = fast.reconstruct_weight_fast(torch.bfloat16)
        wf32 = fast.reconstruct_weight_fast(torch.float32)
    out = {"name": np.array(name), "N": np.array(enc.original_shape[0]), "K": np.array(enc.original_shape[1]),
           "w16_bits": f16_bits(w16), "w32": w32.numpy(), "wfast16_bits": f16_bits(wf16),
           "wfast_bf16_bits": bits(wfb), "wfast32": wf32.numpy()}
    for gi, g in enumerate(enc.groups):
        for s, (ids, book) in enumerate(zip(g.stage_ids, g.codebooks)):
            out[f"g{gi}_ids{s}"] = ids.numpy()
            out[f"g{gi}_book{s}"] = book.numpy()
        out[f"g{gi}_rho"] = g.row_scale.numpy()
        if g.stage_scales is not None:
            out[f"g{gi}_scales"] = g.stage_scales.numpy()
    if bias is not None:
        out["bias_bits"] = bits(bias)
    bdouble = None if bias is None else bias.double()[None, :]
    for M in Ms:
        xb = synthetic.activations(M, enc.original_shape[1], seed=x_seed)
        x16, x32 = xb.to(torch.float16), xb.to(torch.float32)
        with torch.no_grad():
            y16 = exact(x16)
            y32 = exact(x32)
            yfb = fast(xb)
        out[f"x{M}_bits"] = bits(xb)  # x16 and x32 are exact conversions of these bf16 values
        out[f"y{M}_f16_bits"] = f16_bits(y16)
        out[f"y{M}_f32"] = y32.numpy()
        r16 = x16.double() @ w16.double().T
        r32 = x32.double() @ w32.double().T
        rfb = xb.double() @ wfb.double().T
        if bdouble is not None:
            r16, r32, rfb = r16 + bdouble, r32 + bdouble, rfb + bdouble
        out[f"y{M}_f16_ref32"] = r16.float().numpy()
        out[f"y{M}_f32_ref64"] = r32.numpy()
        out[f"y{M}_fast_bf16_bits"] = bits(yfb)
        out[f"y{M}_fast_ref32"] = rfb.float().numpy()
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz")


def dtype_cases(ref_runtime, ref_block_vq) -> None:
    def scaled(enc, scales_per_group):
        groups = tuple(dataclasses.replace(g, stage_scales=torch.tensor(sc, dtype=torch.float16))
                       for g, sc in zip(enc.groups, scales_per_group))
        return dataclasses.replace(enc, groups=groups)

    run_dtype_case("dtype_r2_d8", single_group(synthetic.rvq_encoding(48, 192, d=8, R=2, seed=41)), [1, 6], 41,
                   synthetic.bias_vector(48, seed=41), ref_runtime, ref_block_vq)
    run_dtype_case("dtype_scaled_grouped",
                   scaled(synthetic.grouped_encoding([32, 16], 128, d=16, R=3, seed=42),
                          [[1.0, 0.5, 0.333251953125], [0.9, 1.1, 0.7]]), [3], 42, None, ref_runtime, ref_block_vq)
    run_dtype_case("dtype_route", single_group(synthetic.route_inputs(40, 96, d=16, G=4, seed=43).encoding()), [2],
                   43, synthetic.bias_vector(40, seed=43), ref_runtime, ref_block_vq)
    run_dtype_case("dtype_scaled_r1", scaled(single_group(synthetic.rvq_encoding(32, 64, d=8, R=1, seed=44)),
                                             [[1.2001953125]]), [2], 44, None, ref_runtime, ref_block_vq)


def run_correction_case(name, ref_enc, Ms, x_seed, bias, ref_runtime, ref_io):
    """A reference-encoded grouped encoding with per-block corrections (src/runtime.py:389-412): the encoding
    itself (written by the reference's own map saver), its weights in every dtype and the forward."""
    ref_io.save_grouped_encoding_map(HERE / f"{name}.pt", {"layer": ref_enc})
    mod = ref_runtime.PackedGroupedBlockRVQLinear(ref_enc, bias, matmul_strategy="per_group")
    with torch.no_grad():
        wb = mod.reconstruct_weight(torch.bfloat16)
        w16 = mod.reconstruct_weight(torch.float16)
        w32 = mod.reconstruct_weight(torch.float32)
    out = {"name": np.array(name), "N": np.array(ref_enc.original_shape[0]), "K": np.array(ref_enc.original_shape[1]),
           "w_bits": bits(wb), "w16_bits": f16_bits(w16), "w32": w32.numpy(),
           "kinds": np.array([g.transform_kind for g in ref_enc.groups]),
           "signs": np.array([g.residual_signs is not None for g in ref_enc.groups]),
           "block_scale": np.array([g.block_scale is not None for g in ref_enc.groups])}
    if bias is not None:
        out["bias_bits"] = bits(bias)
    for M in Ms:
        x = synthetic.activations(M, ref_enc.original_shape[1], seed=x_seed)
        with torch.no_grad():
            y = mod(x)
        y32 = x.double() @ wb.double().T
        if bias is not None:
            y32 = y32 + bias.double()[None, :]
        out[f"x{M}_bits"] = bits(x)
        out[f"y{M}_ref32"] = y32.float().numpy()
        out[f"y{M}_ref_bf16"] = bits(y)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"wrote {name}.npz/.pt  kinds={out['kinds']} signs={out['signs']} block_scale={out['block_scale']}")


def correction_cases(ref_runtime, ref_block_vq) -> None:
    from src import encoding_io as ref_io  # type: ignore

    def enc(seed, rows, cols, **kw):
        torch.manual_seed(seed)
        weight = torch.randn(rows, cols) * 0.02
        return ref_block_vq.encode_block_residual_vq(weight, codebook_size=256, kmeans_iters=3, **kw)

    def grouped(*encs):
        rows, slices = 0, []
        for e in encs:
            slices.append((rows, rows + e.original_shape[0]))
            rows += e.original_shape[0]
        return ref_block_vq.GroupedBlockRVQEncoding(groups=tuple(encs), row_slices=tuple(slices),
                                                    original_shape=(rows, encs[0].original_shape[1]))

    run_correction_case("corr_sign_amax", grouped(enc(61, 48, 128, block_size=8, num_stages=2, normalize_blocks="amax",
                                                      residual_correction="sign")), [1, 5], 61,
                        synthetic.bias_vector(48, seed=61), ref_runtime, ref_io)
    run_correction_case("corr_dct_l2", grouped(enc(62, 32, 128, block_size=8, num_stages=2, normalize_blocks="l2",
                                                   transform_kind="dct", residual_correction="sign")), [3], 62, None,
                        ref_runtime, ref_io)
    run_correction_case("corr_hadamard_d16", grouped(enc(63, 32, 160, block_size=16, num_stages=1,
                                                         transform_kind="hadamard", residual_correction="sign")), [2],
                        63, None, ref_runtime, ref_io)
    run_correction_case("corr_grouped_pca_rand",
                        grouped(enc(64, 32, 128, block_size=8, num_stages=2, transform_kind="pca"),
                                enc(65, 16, 128, block_size=8, num_stages=2, transform_kind="rand_hadamard",
                                    normalize_blocks="amax")), [4], 64, None, ref_runtime, ref_io)
    run_correction_case("corr_polar", grouped(enc(66, 32, 128, block_size=8, num_stages=2, transform_kind="polar")),
                        [3], 66, None, ref_runtime, ref_io)


def encoder_cases(ref_block_vq) -> None:
    """The reference's own k-means assignment, fit and encoder (src/block_vq.py:180-531) on seeded inputs."""
    g = torch.Generator().manual_seed(71)
    blocks = torch.randn(4096, 8, generator=g) * 0.3
    sample = blocks[:2048].clone()
    codebook = ref_block_vq._fit_kmeans(sample, codebook_size=64, iters=4)
    ids, dist = ref_block_vq._assign_to_codebook(blocks, codebook)
    out = {"blocks": blocks.numpy(), "sample_rows": np.array(2048), "fit_entries": np.array(64),
           "fit_iters": np.array(4), "fit_codebook": codebook.numpy(), "ids": ids.numpy(), "min_dist": dist.numpy()}
    weight = torch.randn(96, 256, generator=g) * 0.02
    e1 = ref_block_vq.encode_block_residual_vq(weight, block_size=8, codebook_size=64, num_stages=2, kmeans_iters=3)
    e2 = ref_block_vq.encode_block_residual_vq(weight, block_size=8, codebook_size=64, num_stages=2, product_splits=2,
                                               stages_per_split=(2, 1), normalize_blocks="amax", kmeans_iters=3)
    out["weight"] = weight.numpy()
    for tag, e in (("plain", e1), ("split", e2)):
        for si, (ids_s, cb_s) in enumerate(zip(e.stage_ids, e.codebooks)):
            out[f"{tag}_ids{si}"] = ids_s.numpy()
            out[f"{tag}_book{si}"] = cb_s.numpy()
        out[f"{tag}_rho"] = e.row_scale.numpy()
        out[f"{tag}_rel_mse"] = np.array(e.sample_rel_mse)
        if e.block_scale is not None:
            out[f"{tag}_block_scale"] = e.block_scale.numpy()
    np.savez_compressed(HERE / "encoder.npz", **out)
    print("wrote encoder.npz")


def stage_drop_cases(ref_runtime, ref_block_vq) -> None:
    run_stage_drop_case("stage_drop_r3", single_group(synthetic.rvq_encoding(64, 192, d=8, R=3, seed=31)), 2,
                        [1, 5], 31, ref_runtime, ref_block_vq)
    run_stage_drop_case("stage_drop_r3_k1", synthetic.grouped_encoding([32, 48], 128, d=16, R=3, seed=32), 1,
                        [3], 32, ref_runtime, ref_block_vq)
    # product splits (2 splits x 2 stages, split-major), encoded by the reference's own encoder;
    # keeping one stage per split leaves stages 0 and 2
    torch.manual_seed(33)
    weight = torch.randn(48, 128) * 0.02
    ref_enc = ref_block_vq.encode_block_residual_vq(weight, block_size=8, codebook_size=256, num_stages=2,
                                                    product_splits=2, stages_per_split=(2, 2), kmeans_iters=4)
    ours = BlockRVQEncoding(**{f.name: getattr(ref_enc, f.name) for f in dataclasses.fields(BlockRVQEncoding)})
    run_stage_drop_case("stage_drop_splits", single_group(ours), 1, [2], 33, ref_runtime, ref_block_vq)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--skip-full", action="store_true")
    ap.add_argument("--only", default="", help="comma-separated groups to (re)generate: stage_drop, dtype, corrections, encoder")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from src import block_vq as ref_block_vq  # type: ignore
    from src import runtime as ref_runtime  # type: ignore

    torch.set_num_threads(max(1, torch.get_num_threads()))
    only = {v for v in args.only.split(",") if v}
    if only:
        if "stage_drop" in only:
            stage_drop_cases(ref_runtime, ref_block_vq)
        if "dtype" in only:
            dtype_cases(ref_runtime, ref_block_vq)
        if "corrections" in only:
            correction_cases(ref_runtime, ref_block_vq)
        if "encoder" in only:
            encoder_cases(ref_block_vq)
        return
    small = [
        ("small_r2_d8", single_group(synthetic.rvq_encoding(37, 64, d=8, R=2, seed=11)), [1, 3], 11, True),
        ("small_r1_ragged", single_group(synthetic.rvq_encoding(48, 100, d=8, R=1, C=200, seed=12)), [5], 12, False),
        ("small_r3_d16", single_group(synthetic.rvq_encoding(64, 96, d=16, R=3, seed=13)), [2, 16], 13, False),
        ("small_grouped", synthetic.grouped_encoding([16, 24, 9], 128, d=8, R=2, seed=14), [4], 14, True),
        ("small_route", single_group(synthetic.route_inputs(40, 64, d=16, G=4, seed=15).encoding()), [3], 15, False),
        ("small_d32", single_group(synthetic.rvq_encoding(33, 128, d=32, R=2, seed=16)), [16], 16, True),
        ("small_r4_wide", single_group(synthetic.rvq_encoding(20, 272, d=8, R=4, seed=17)), [9], 17, False),
    ]
    for name, enc, Ms, seed, with_bias in small:
        bias = synthetic.bias_vector(enc.original_shape[0], seed=seed) if with_bias else None
        run_case(name, enc, Ms, seed, bias, ref_runtime, ref_block_vq, full=True)
    # per-stage scales (fp16, as the reference's encoder stores them, src/block_vq.py:522)
    def scaled(enc, scales_per_group):
        groups = tuple(dataclasses.replace(g, stage_scales=torch.tensor(sc, dtype=torch.float16))
                       for g, sc in zip(enc.groups, scales_per_group))
        return dataclasses.replace(enc, groups=groups)

    run_case("small_scaled_r2", scaled(single_group(synthetic.rvq_encoding(48, 136, d=8, R=2, seed=18)),
                                       [[0.8125, 1.3125]]), [1, 7], 18, None, ref_runtime, ref_block_vq, full=True)
    run_case("small_scaled_r1", scaled(single_group(synthetic.rvq_encoding(32, 64, d=8, R=1, seed=19)),
                                       [[1.2001953125]]), [2], 19, None, ref_runtime, ref_block_vq, full=True)
    run_case("small_scaled_grouped",
             scaled(synthetic.grouped_encoding([32, 16], 96, d=16, R=3, seed=20),
                    [[1.0, 0.5, 0.333251953125], [0.9, 1.1, 0.7]]), [3], 20, None, ref_runtime, ref_block_vq,
             full=True)
    # product splits, encoded by the reference's own encoder (src/block_vq.py:340-531): split 0
    # (columns 0..3 of every 8-column block) has two stages, split 1 one; each stage's codebook is
    # stored full width with zeros outside its split, so the fused path sums three stages
    torch.manual_seed(23)
    weight = torch.randn(48, 128) * 0.02
    ref_enc = ref_block_vq.encode_block_residual_vq(weight, block_size=8, codebook_size=256, num_stages=2,
                                                    product_splits=2, stages_per_split=(2, 1), kmeans_iters=4)
    ours = BlockRVQEncoding(**{f.name: getattr(ref_enc, f.name) for f in dataclasses.fields(BlockRVQEncoding)})
    run_case("small_product_splits", single_group(ours), [1, 6], 23, synthetic.bias_vector(48, seed=23),
             ref_runtime, ref_block_vq, full=True, extra={"product_splits": 2, "stages_per_split": [2, 1],
                                                          "stage_value_dims": list(ref_enc.stage_value_dims)})
    # an encoding map written by the reference's own saver (src/encoding_io.py:77-85)
    from src import encoding_io as ref_io  # type: ignore

    enc_a = to_reference(scaled(single_group(synthetic.rvq_encoding(48, 136, d=8, R=2, seed=18)),
                                [[0.8125, 1.3125]]), ref_block_vq)
    enc_b = to_reference(synthetic.grouped_encoding([16, 24, 9], 128, d=8, R=2, seed=14), ref_block_vq)
    ref_io.save_grouped_encoding_map(HERE / "encoding_map_small.pt",
                                     {"model.layers.0.mlp.up_proj": enc_a, "model.layers.0.self_attn.q_proj": enc_b})
    print("wrote encoding_map_small.pt")
    # ID-route linear (reference PackedIDRouteLinear): fp16 bias as the reference stores it
    run_idroute_case("idroute_small", synthetic.idroute_inputs(40, 136, routes=300, seed=21), [1, 5], 21,
                     synthetic.bias_vector(40, seed=21).to(torch.float16), ref_runtime)
    run_idroute_case("idroute_medium", synthetic.idroute_inputs(256, 1024, routes=1536, seed=22), [3, 16], 22,
                     None, ref_runtime)
    stage_drop_cases(ref_runtime, ref_block_vq)
    dtype_cases(ref_runtime, ref_block_vq)
    correction_cases(ref_runtime, ref_block_vq)
    encoder_cases(ref_block_vq)
    if args.skip_full:
        return
    run_case("cfg0", synthetic.cfg0_encoding(0), [1, 4, 16], 0, None, ref_runtime, ref_block_vq, full=False)
    run_case("cfg1", single_group(synthetic.cfg1_inputs(1).encoding()), [1, 8], 1, None, ref_runtime,
             ref_block_vq, full=False, y_rows=2048)


if __name__ == "__main__":
    main()
