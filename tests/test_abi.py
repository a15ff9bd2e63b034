"""C ABI checks that need no GPU: exported symbols, host packing, argument validation."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from tests import goldens
from wal2026_b200 import _abi, synthetic
from wal2026_b200.block_vq import single_group
from wal2026_b200.packing import pack_grouped, pack_routes
from wal2026_b200.runtime import PackedGroupedBlockRVQLinear, RouteCodebookLinear

HEADER = Path(__file__).resolve().parents[1] / "include" / "wal_rvq.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"WAL_API\s+[\w\s\*]+?\b(wal_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    names = declared_functions()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
        assert name in _abi.SIGNATURES, f"{name} has no ctypes signature"
    assert lib.wal_version() >= 100
    assert lib.wal_status_string(4).decode().startswith("id")


def unpack_numpy(packed: np.ndarray, table: np.ndarray, R: int, idw: int, N: int, blocks: int) -> np.ndarray:
    """Independent reader of the packed layout documented in include/wal_rvq.h."""
    chunks = -(-blocks // 16)
    V = R * idw
    out = np.zeros((R, N, blocks), dtype=np.uint16 if idw == 2 else np.uint8)
    view = packed.reshape(-1, chunks, V, 16, 16)  # tile, chunk, vector, row, byte
    for t, (g, row0, nrows, _) in enumerate(table):
        for s in range(R):
            for c in range(chunks):
                nb = min(16, blocks - 16 * c)
                if idw == 1:
                    ids = view[t, c, s, :nrows, :nb]
                else:
                    raw = np.concatenate([view[t, c, 2 * s, :nrows], view[t, c, 2 * s + 1, :nrows]], axis=1)
                    ids = raw.view(np.uint16)[:, :nb]
                out[s, row0:row0 + nrows, 16 * c:16 * c + nb] = ids
    return out


@pytest.mark.parametrize("name", goldens.SMALL_CASES)
def test_host_pack_round_trips(name):
    fx = goldens.load(name)
    enc = goldens.encoding_from_fixture(fx)
    p = pack_grouped(enc)
    g = p.geometry
    blocks = -(-g.in_features // g.block_size)
    idw = 1 if g.num_entries <= 256 else 2
    got = unpack_numpy(p.packed_ids.numpy(), p.tile_table.numpy(), g.num_stages, idw, g.out_features, blocks)
    want = np.stack([np.concatenate([gr.stage_ids[s].numpy().view(got.dtype) for gr in enc.groups])
                     for s in range(g.num_stages)])
    assert np.array_equal(got, want)
    assert p.packed_ids.numel() % 256 == 0
    assert p.codebooks.shape == (len(enc.groups), g.num_stages, g.num_entries, g.block_size)


def test_route_pack_equals_single_stage_pack():
    inp = synthetic.route_inputs(40, 64, d=16, G=4, seed=15)
    a = pack_routes(inp.route, inp.code, inp.codebooks, inp.row_scale, 64)
    b = pack_grouped(single_group(inp.encoding()))
    assert torch.equal(a.packed_ids, b.packed_ids)
    assert torch.equal(a.tile_table, b.tile_table)
    assert torch.equal(a.codebooks, b.codebooks)


def _geom(**kw):
    base = dict(out_features=32, in_features=64, block_size=8, num_stages=2, num_entries=256, num_groups=1)
    base.update(kw)
    return _abi.Geometry(**base)


def _size(geom, rows):
    lib = _abi.load()
    arr = (ctypes.c_int64 * len(rows))(*rows)
    nb, nt = ctypes.c_size_t(0), ctypes.c_int64(0)
    return lib.wal_rvq_packed_size(ctypes.byref(geom), arr, ctypes.byref(nb), ctypes.byref(nt)), nb.value, nt.value


def test_packed_size_and_validation_codes():
    st, nb, nt = _size(_geom(), [32])
    assert st == _abi.WAL_OK and nt == 2 and nb == 2 * 1 * 2 * 256  # 2 tiles x 1 chunk x 2 vectors x 256 B
    assert _size(_geom(block_size=12), [32])[0] == _abi.WAL_ERR_UNSUPPORTED
    assert _size(_geom(num_stages=5), [32])[0] == _abi.WAL_ERR_UNSUPPORTED
    assert _size(_geom(num_entries=300), [32])[0] == _abi.WAL_ERR_UNSUPPORTED
    assert _size(_geom(in_features=66), [32])[0] == _abi.WAL_ERR_UNSUPPORTED
    assert _size(_geom(), [31])[0] == _abi.WAL_ERR_SHAPE
    assert _size(_geom(num_groups=2), [16, 16])[0] == _abi.WAL_OK
    assert _size(_geom(out_features=0), [0])[0] == _abi.WAL_ERR_SHAPE


def test_pack_rejects_out_of_range_ids_and_small_buffers():
    lib = _abi.load()
    geom = _geom(num_entries=200, num_stages=1)
    ids = np.full((32, 8), 199, dtype=np.uint8)
    ids[3, 5] = 200
    rows = (ctypes.c_int64 * 1)(32)
    ptrs = (ctypes.c_void_p * 1)(ids.ctypes.data)
    buf = np.zeros(4096, dtype=np.uint8)
    table = np.zeros((2, 4), dtype=np.int32)
    tp = table.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    assert lib.wal_rvq_pack(ctypes.byref(geom), rows, ptrs, buf.ctypes.data, buf.nbytes, tp) == _abi.WAL_ERR_ID_RANGE
    ids[3, 5] = 0
    assert lib.wal_rvq_pack(ctypes.byref(geom), rows, ptrs, buf.ctypes.data, 16, tp) == _abi.WAL_ERR_BUFFER_TOO_SMALL
    assert lib.wal_rvq_pack(ctypes.byref(geom), rows, ptrs, buf.ctypes.data, buf.nbytes, tp) == _abi.WAL_OK
    assert lib.wal_rvq_pack(None, rows, ptrs, buf.ctypes.data, buf.nbytes, tp) == _abi.WAL_ERR_INVALID_ARGUMENT


def test_route_pack_rejects_bad_route():
    inp = synthetic.route_inputs(16, 32, d=16, G=4, seed=3)
    route = inp.route.clone()
    route[2, 1] = 4
    with pytest.raises(ValueError, match="out of range"):
        pack_routes(route, inp.code, inp.codebooks, inp.row_scale, 32)


def test_device_entry_points_validate_before_touching_the_gpu():
    lib = _abi.load()
    layer = _abi.Layer(geom=_geom(), num_tiles=2, packed_ids=None, tile_table=None, codebooks=None, row_scale=None,
                       bias=None)
    assert lib.wal_rvq_gemv(ctypes.byref(layer), None, 1, 64, None, 32, 0, None) == _abi.WAL_ERR_INVALID_ARGUMENT
    assert lib.wal_rvq_dequant(None, None, 64, None) == _abi.WAL_ERR_INVALID_ARGUMENT
    layer.geom.block_size = 7
    assert lib.wal_rvq_unpack_ids(ctypes.byref(layer), None, None) == _abi.WAL_ERR_UNSUPPORTED


def test_module_builds_on_cpu_and_refuses_cpu_forward():
    enc = synthetic.cfg0_encoding(0)
    mod = PackedGroupedBlockRVQLinear(enc, None)
    assert mod.in_features == 2048 and mod.out_features == 2048 and len(mod.groups) == 1
    assert mod.compressed_bytes() == 2048 * 256 * 2 + 2 * 256 * 8 * 2 + 2048 * 2
    with pytest.raises(ValueError, match="CUDA"):
        mod(torch.zeros(1, 2048, dtype=torch.bfloat16))


def test_strategy_validation_matches_reference():
    enc = single_group(synthetic.rvq_encoding(16, 32, seed=1))
    with pytest.raises(ValueError, match="unsupported matmul_strategy"):
        PackedGroupedBlockRVQLinear(enc, matmul_strategy="nope")
    with pytest.raises(ValueError, match="chunked_weight requires"):
        PackedGroupedBlockRVQLinear(enc, matmul_strategy="chunked_weight")
    with pytest.raises(ValueError, match="requires a positive hot_topk"):
        PackedGroupedBlockRVQLinear(enc, matmul_strategy="full_weight_hot")
    for s in ("per_group", "full_weight_fast", "triton_block_rvq", "stagewise_einsum"):
        assert PackedGroupedBlockRVQLinear(enc, matmul_strategy=s).matmul_strategy == s


def test_unsupported_encodings_raise_value_error():
    enc = synthetic.rvq_encoding(16, 32, seed=1)
    import dataclasses

    dct = dataclasses.replace(enc, transform_kind="dct")
    with pytest.raises(ValueError, match="per-block corrections"):
        pack_grouped(single_group(dct))  # the id packer alone covers the stage sum only
    mod = PackedGroupedBlockRVQLinear(single_group(dct))  # the module packs the corrections beside it
    assert mod.has_corrections and mod.corr_flags.tolist() == [_abi.WAL_CORR_MATRIX]
    with pytest.raises(ValueError, match="transform_kind must be one of"):
        PackedGroupedBlockRVQLinear(single_group(dataclasses.replace(enc, transform_kind="wavelet")))
    scaled = dataclasses.replace(enc, stage_scales=torch.tensor([1.5, 0.5], dtype=torch.float16))
    mod = PackedGroupedBlockRVQLinear(single_group(scaled))  # per-stage scales are supported
    assert torch.equal(mod.stage_scales, torch.tensor([[1.5, 0.5]]))
    odd = synthetic.rvq_encoding(16, 30, d=8, seed=1)
    with pytest.raises(ValueError, match="multiple of 4"):
        PackedGroupedBlockRVQLinear(single_group(odd))


def test_route_module_shape():
    inp = synthetic.route_inputs(40, 64, d=16, G=4, seed=15)
    mod = RouteCodebookLinear.from_routes(inp.route, inp.code, inp.codebooks, inp.row_scale, in_features=64)
    assert mod.num_entries == 1024 and mod.num_stages == 1 and mod.out_features == 40


def test_profile_cases_cli_lists_its_cases():
    from wal2026_b200 import profile_cases

    assert set(profile_cases.CASES) == {"cfg1_gemv", "gemv_window", "idroute_mlp", "attention", "prefill_gate_up",
                                        "tp_breakdown"}
    assert profile_cases.main(["no_such_case"]) == 2


def test_product_split_encoding_is_accepted():
    """Reference-encoded product splits: full-width codebooks summed like any other stages."""
    fx = goldens.load("small_product_splits")
    mod = PackedGroupedBlockRVQLinear(goldens.encoding_from_fixture(fx))
    g = mod.groups[0]  # split metadata lives on the row group, as in the reference's PackedBlockRVQGroup
    assert g.product_splits == 2 and g.stages_per_split == (2, 1) and mod.num_stages == 3


def test_attention_workspace_covers_every_shorter_call():
    # the size for max_n must cover each n <= max_n (the split count itself is
    # not monotone in n), so the reported size never decreases as n grows
    lib = _abi.load()
    for B, hkv, hq in ((1, 8, 32), (2, 8, 64), (3, 2, 8), (16, 8, 32)):
        sizes = [int(lib.wal_decode_attention_workspace(B, hq, hkv, 128, n)) for n in range(1, 5000)]
        assert all(a <= b for a, b in zip(sizes, sizes[1:])), (B, hkv)
        assert sizes[0] > 0


def _documented_struct(name: str) -> list[tuple[str, str]]:
    """(field, ctypes type text) pairs of a ctypes struct in INTEGRATION.md's binding snippet."""
    text = (HEADER.parents[1] / "INTEGRATION.md").read_text()
    m = re.search(rf"class {name}\(ctypes\.Structure\):\s*_fields_ = \[(.*?)\][^\n]*\n", text, re.S)
    assert m, f"{name} not found in INTEGRATION.md"
    return re.findall(r'\("(\w+)",\s*([\w.]+(?:\([\w.]+\))?)\)', m.group(1))


def test_documented_binding_structs_match_the_library_structs():
    # a maintainer copies INTEGRATION.md's ctypes structs; a missing or reordered
    # field would shift every later pointer the library reads
    for doc_name, lib_struct in (("_Geom", _abi.Geometry), ("_Layer", _abi.Layer)):
        doc = [(f, eval(t, {"ctypes": ctypes, "_Geom": _abi.Geometry})) for f, t in _documented_struct(doc_name)]
        assert doc == list(lib_struct._fields_), (doc_name, doc, lib_struct._fields_)
