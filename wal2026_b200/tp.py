"""Tensor-parallel sharding of packed Block-RVQ linears and the peer-memory exchange.

Megatron-style split of a Llama block, one process per GPU:

* column-parallel (q/k/v, gate/up): every row group's output rows are split
  evenly; a rank keeps whole 16-row tiles of the packed stream, its rows'
  scales and the group's full (small) codebooks.  No communication.
* row-parallel (o, down): the input dimension is split on 16-block chunk
  boundaries; a rank keeps its chunks of every tile, all row scales and the
  codebooks, and produces an fp32 partial output that must be summed over
  ranks.

The sum is the one exchange step.  ``PeerExchange`` gives every rank a device
region (CUDA IPC, mapped by every peer) holding receive slots;
``wal_rvq_gemv_push`` stores each rank's partial straight into every rank's
slot over NVLink as 8-byte words {value, tag} (NCCL's "LL" idea: an aligned
8-byte store arrives whole, so a word whose tag equals the slot's call count
+ 1 is fresh, with no fence or flag), and ``wal_tp_reduce_rmsnorm`` waits
for all ranks' words, adds them in rank order (identical on every rank), the
residual and the next RMSNorm, then advances the slot's call count.  Slots
rotate over ``PeerExchange.SLOTS`` calls; a rank cannot overwrite a slot a
peer has not consumed, because reaching the slot's next use needs that peer's
partials of the calls in between, which the peer produces only after
consuming the slot.

No reference counterpart: the reference runs on one device.  Encoding-level
sharding (``shard_encoding``) is the host restatement used to check the packed
sharding (``shard_packed``) bit for bit.
"""
from __future__ import annotations

import ctypes
from dataclasses import replace

import torch
from torch import Tensor

from . import _abi
from .block_vq import GroupedBlockRVQEncoding
from .packing import PackedArrays
from .runtime import PackedGroupedBlockRVQLinear

COLUMN = "column"  # split output rows
ROW = "row"        # split input blocks


def shard_bounds(n: int, rank: int, size: int, unit: int, what: str) -> tuple[int, int]:
    """[start, end) of an even split of n into `size` parts, each a multiple of `unit`."""
    if n % (size * unit):
        raise ValueError(f"{what} ({n}) does not split into {size} parts of whole {unit}s")
    part = n // size
    return rank * part, (rank + 1) * part


def shard_encoding(enc: GroupedBlockRVQEncoding, rank: int, size: int, mode: str) -> GroupedBlockRVQEncoding:
    """Rank `rank`'s shard of a plain grouped encoding (host tensors)."""
    groups, slices, row = [], [], 0
    K = int(enc.original_shape[1])
    for g in enc.groups:
        d = int(g.block_size)
        if mode == COLUMN:
            r0, r1 = shard_bounds(int(g.original_shape[0]), rank, size, 16, "group rows")
            ng = replace(g, stage_ids=tuple(t[r0:r1].contiguous() for t in g.stage_ids),
                         row_scale=g.row_scale[r0:r1].contiguous(), original_shape=(r1 - r0, K))
        elif mode == ROW:
            k0, k1 = shard_bounds(K, rank, size, 16 * d, "in_features")
            ng = replace(g, stage_ids=tuple(t[:, k0 // d:k1 // d].contiguous() for t in g.stage_ids),
                         original_shape=(int(g.original_shape[0]), k1 - k0), padded_cols=k1 - k0)
        else:
            raise ValueError(f"unknown shard mode {mode!r}")
        groups.append(ng)
        n = int(ng.original_shape[0])
        slices.append((row, row + n))
        row += n
    k_out = K if mode == COLUMN else int(groups[0].original_shape[1])
    return GroupedBlockRVQEncoding(groups=tuple(groups), row_slices=tuple(slices), original_shape=(row, k_out))


def shard_packed(lin: PackedGroupedBlockRVQLinear, rank: int, size: int, mode: str) -> PackedGroupedBlockRVQLinear:
    """Rank `rank`'s shard of a packed linear, cut from its packed buffers (same device).

    Equal, buffer for buffer, to packing ``shard_encoding`` of the encoding the
    module was packed from.  Row-parallel shards drop the bias (partials are
    summed; the caller adds a bias once).
    """
    if getattr(lin, "has_corrections", False):
        raise ValueError("tensor-parallel shards of layers with per-block corrections are not supported")
    d, R = lin.block_size, lin.num_stages
    idw = 1 if lin.num_entries <= 256 else 2
    blocks = -(-lin.in_features // d)
    chunks = -(-blocks // 16)
    V = R * idw
    tile_bytes = chunks * V * 256
    T = lin.num_tiles
    packed = lin.packed_ids.view(T, tile_bytes)
    rows = lin.group_rows()
    dev = lin.packed_ids.device
    if mode == COLUMN:
        keep_tiles, table, rho, new_rows = [], [], [], []
        t0, row_out = 0, 0
        for g, n in enumerate(rows):
            tg = -(-n // 16)
            r0, r1 = shard_bounds(n, rank, size, 16, "group rows")
            lt0, lt1 = r0 // 16, r1 // 16
            keep_tiles.append(torch.arange(t0 + lt0, t0 + lt1, device=dev))
            for j in range(lt1 - lt0):
                table.append([g, row_out + 16 * j, 16, 0])
            g_row0 = sum(rows[:g])
            rho.append(lin.row_scale[g_row0 + r0:g_row0 + r1])
            new_rows.append(r1 - r0)
            row_out += r1 - r0
            t0 += tg
        idx = torch.cat(keep_tiles)
        new_packed = packed.index_select(0, idx).reshape(-1).contiguous()
        geom = _abi.Geometry(out_features=row_out, in_features=lin.in_features, block_size=d, num_stages=R,
                             num_entries=lin.num_entries, num_groups=lin.num_groups)
        arrays = PackedArrays(geom, len(table), new_packed, torch.tensor(table, dtype=torch.int32, device=dev),
                              lin.codebooks, torch.cat(rho).contiguous(), lin.stage_scales)
        bias = None
        if lin.bias is not None:
            parts, r = [], 0
            for n in rows:
                a, b = shard_bounds(n, rank, size, 16, "group rows")
                parts.append(lin.bias[r + a:r + b])
                r += n
            bias = torch.cat(parts)
        return PackedGroupedBlockRVQLinear.from_packed(arrays, new_rows, bias=bias)
    if mode == ROW:
        k0, k1 = shard_bounds(lin.in_features, rank, size, 16 * d, "in_features")
        c0, c1 = k0 // (16 * d), k1 // (16 * d)
        new_packed = packed.view(T, chunks, V * 256)[:, c0:c1].reshape(-1).contiguous()
        geom = _abi.Geometry(out_features=lin.out_features, in_features=k1 - k0, block_size=d, num_stages=R,
                             num_entries=lin.num_entries, num_groups=lin.num_groups)
        arrays = PackedArrays(geom, T, new_packed, lin.tile_table, lin.codebooks, lin.row_scale, lin.stage_scales)
        return PackedGroupedBlockRVQLinear.from_packed(arrays, rows, bias=None)
    raise ValueError(f"unknown shard mode {mode!r}")


class PeerExchange:
    """Receive slots in every rank's memory for row-parallel partial outputs.

    Region layout (bytes) on every rank:
      [0, 512)           epoch[s]: the slot's call count (one 128-byte line per slot)
      [1024, 1536)       done[s]: CTA counter of the receiving kernel
      [4096, ...)        recv[s][p][max_rows][width] 8-byte words, written by rank p
    All of it starts at zero (the region is zero-filled when created).
    """

    SLOTS = 4

    def __init__(self, rank: int, size: int, max_rows: int, width: int, device: torch.device, group=None):
        import torch.distributed as dist

        if not 1 <= size <= _abi.WAL_MAX_RANKS:
            raise ValueError(f"tensor-parallel size {size} is outside 1..{_abi.WAL_MAX_RANKS}")
        self.rank, self.size, self.max_rows, self.width = int(rank), int(size), int(max_rows), int(width)
        self.device = torch.device(device)
        self.slot_elems = self.max_rows * self.width
        self.bytes = 4096 + self.SLOTS * self.size * self.slot_elems * 8
        lib = _abi.load()
        self._lib = lib
        handle = (ctypes.c_uint8 * _abi.WAL_IPC_HANDLE_BYTES)()
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _abi.check(lib.wal_peer_region_create(self.bytes, ctypes.byref(own), handle), "wal_peer_region_create")
        self.own = int(own.value)
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        parts = [torch.empty_like(mine) for _ in range(self.size)]
        if self.size > 1:
            dist.all_gather(parts, mine, group=group)
        else:
            parts = [mine]
        self.base: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            for p, h in enumerate(parts):
                if p == self.rank:
                    self.base.append(self.own)
                    continue
                raw = (ctypes.c_uint8 * _abi.WAL_IPC_HANDLE_BYTES)(*h.cpu().tolist())
                ptr = ctypes.c_void_p()
                _abi.check(lib.wal_peer_region_open(raw, ctypes.byref(ptr)), "wal_peer_region_open")
                self.base.append(int(ptr.value))
                self._opened.append(int(ptr.value))
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._group = group
        self._pushes = [self._make_push(s) for s in range(self.SLOTS)]
        if self.size > 1:
            dist.barrier(group=group)

    # -- offsets -----------------------------------------------------------
    def _recv_off(self, slot: int, src: int) -> int:
        return 4096 + ((slot * self.size + src) * self.slot_elems) * 8

    def epoch_ptr(self, slot: int) -> int:
        return self.own + slot * 128

    def done_ptr(self, slot: int) -> int:
        return self.own + 1024 + slot * 128

    def recv_ptr(self, slot: int) -> int:
        return self.own + self._recv_off(slot, 0)

    def _make_push(self, slot: int) -> _abi.TPPush:
        push = _abi.TPPush()
        push.num_ranks, push.rank, push.ld_dst = self.size, self.rank, self.width
        for p in range(self.size):
            push.dst[p] = self.base[p] + self._recv_off(slot, self.rank)
        push.epoch = self.epoch_ptr(slot)
        return push

    # -- the two halves of one exchange ------------------------------------
    def push_gemv(self, lin: PackedGroupedBlockRVQLinear, x2: Tensor, slot: int) -> None:
        """Row-parallel GEMV whose fp32 partial lands in `slot` on every rank."""
        if x2.shape[0] > self.max_rows or lin.out_features != self.width:
            raise ValueError("push GEMV shape exceeds the exchange's slot")
        st = self._lib.wal_rvq_gemv_push(ctypes.byref(lin.layer_struct(lin._active_stages(), lin.sum_mode())), x2.data_ptr(), x2.shape[0],
                                         x2.stride(0), ctypes.byref(self._pushes[slot]),
                                         _abi.stream_handle(x2.device))
        _abi.check(st, "wal_rvq_gemv_push")

    def push_rows(self, y: Tensor, slot: int) -> None:
        """Send an already computed output (fp32 or bf16 [M, width], e.g. a dense GEMM's) into `slot` on every rank."""
        if y.shape[0] > self.max_rows or y.shape[1] != self.width or y.stride(1) != 1:
            raise ValueError("pushed rows do not match the exchange's slot")
        st = self._lib.wal_tp_push_rows(y.data_ptr(), y.stride(0), _abi.DTYPE_CODE[y.dtype], y.shape[0], y.shape[1],
                                        ctypes.byref(self._pushes[slot]), _abi.stream_handle(y.device))
        _abi.check(st, "wal_tp_push_rows")

    def reduce_residual_norm(self, slot: int, h: Tensor, norm_w: Tensor, eps: float, x_out: Tensor) -> None:
        """h += sum of the slot's partials (rank order); x_out = RMSNorm(h) * norm_w."""
        M, N = h.shape
        st = self._lib.wal_tp_reduce_rmsnorm(self.recv_ptr(slot), self.size, self.slot_elems, self.width,
                                             self.epoch_ptr(slot), self.done_ptr(slot), h.data_ptr(), h.stride(0),
                                             norm_w.data_ptr(), float(eps), x_out.data_ptr(), x_out.stride(0), M, N,
                                             self.status.data_ptr(), _abi.stream_handle(h.device))
        _abi.check(st, "wal_tp_reduce_rmsnorm")

    def check_status(self) -> None:
        """Raise if any bounded wait of this exchange timed out (synchronises the device)."""
        v = int(self.status.item())
        if v != 0:
            raise _abi.WalError(v, "tensor-parallel exchange")

    def close(self) -> None:
        import torch.distributed as dist

        if self.own == 0:
            return
        torch.cuda.synchronize(self.device)
        if self.size > 1:
            dist.barrier(group=self._group)  # no peer writes into this region any more
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._lib.wal_peer_region_close(p)
            self._lib.wal_peer_region_free(self.own)
        self.own = 0
        self._opened = []


def all_reduce_partial(y: Tensor, group=None) -> Tensor:
    """NCCL sum of fp32 partials (the library-collective baseline of the exchange)."""
    import torch.distributed as dist

    dist.all_reduce(y, group=group)
    return y


__all__ = ["COLUMN", "ROW", "shard_bounds", "shard_encoding", "shard_packed", "PeerExchange", "all_reduce_partial"]
