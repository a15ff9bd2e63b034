"""Tensor-parallel decode on 2 GPUs: the sharded stack (NCCL all-reduce or the
peer-memory push exchange) against the unsharded stack of the same model.

Runs as two spawned processes, one per GPU, with NVLS off; skipped when fewer
than two GPUs are visible.  Each rank builds the same full model from one seed
and keeps its shard, so rank 0 can also build the unsharded model.
"""
from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

TINY_ARGS = dict(layers=2, hidden=1024, mlp=2048, heads=8, kv_heads=4, vocab=2048)


def _rank_main(rank: int, size: int, store_path: str, kind: str, batch: int, out) -> None:
    import datetime

    import torch.distributed as dist

    from wal2026_b200.llama import LlamaShape, TPContext, dense_llama, rvq_llama

    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    # a file rendezvous: no TCP port to collide with the previous case's
    dist.init_process_group("nccl", init_method=f"file://{store_path}", rank=rank, world_size=size, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        shape = LlamaShape(**TINY_ARGS)
        ctor = rvq_llama if kind == "rvq" else dense_llama
        tp = TPContext(rank, size, dist.group.WORLD)
        st = ctor(shape, device=dev, seed=4, tp=tp)
        st.allocate_cache(batch, 65, seed=5, consistent=True)
        gen = torch.Generator(device=dev).manual_seed(6)
        tokens = torch.randint(0, shape.vocab, (batch,), device=dev, generator=gen)
        cos, sin = st.rope_tables(64)
        results = {}
        for mode in (["nccl", "push"] if kind == "rvq" else ["nccl"]):
            if mode == "push":
                st.enable_push_exchange(batch)
            st.allocate_cache(batch, 65, seed=5, consistent=True)
            results[mode] = st.decode_step_fused(tokens, 64, cos, sin, exchange=mode).float().cpu()
            # a second step through a CUDA graph gives the same logits
            st.allocate_cache(batch, 65, seed=5, consistent=True)
            g = torch.cuda.CUDAGraph()
            st.decode_step_fused(tokens, 64, cos, sin, exchange=mode)  # warm-up outside capture
            torch.cuda.synchronize()
            st.allocate_cache(batch, 65, seed=5, consistent=True)
            with torch.cuda.graph(g):
                logits = st.decode_step_fused(tokens, 64, cos, sin, exchange=mode)
            g.replay()
            torch.cuda.synchronize()
            results[mode + "_graph"] = logits.float().cpu()
            del g
        if st.exchange is not None:
            st.exchange.check_status()
        st.close()
        if rank == 0:
            full = ctor(shape, device=dev, seed=4)
            full.allocate_cache(batch, 65, seed=5, consistent=True)
            ref = full.decode_step_fused(tokens, 64, cos, sin).float().cpu()
            errs = {k: float((v - ref).abs().max()) / float(ref.abs().max()) for k, v in results.items()}
            out.put(errs)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kind,batch", [("rvq", 1), ("rvq", 5), ("dense", 2)])
def test_tp2_decode_matches_unsharded(kind, batch, tmp_path):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    store = str(tmp_path / "rendezvous")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, store, kind, batch, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = out.get(timeout=5)
    for k, e in errs.items():
        assert e < 2e-2, (k, e)
