"""ID-route runtime linear: one int16 id per weight into a scalar fp16 route table.

``PackedIDRouteLinear`` keeps the constructor, ``from_encoded``,
``reconstruct_weight`` and forward contract of the reference module of the
same name (reference ``src/runtime.py:52-97``): ``ids`` int16/int32 ``[N, K]``,
``codebook_w`` fp16 ``[routes, L_max]`` whose row sums form the route table
``codebook_sum`` (computed with the same PyTorch reduction the reference
uses), ``row_scale`` fp16 ``[N, 1]``, optional bias.  The forward runs the
sm_100a ID-route GEMV (``wal_idroute_gemv``) on the packed id stream; its
weight is bit-identical to the reference's
``reconstruct_weight().to(torch.bfloat16)``.  ``FusedIDRouteLinear`` (the
reference's Triton path, which rounds differently) is accepted as an alias
with this module's numerics.

There is no CPU path: the forward raises on CPU input.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch
from torch import Tensor, nn

from . import _abi


def pack_ids(ids: Tensor, num_routes: int) -> Tensor:
    """Host re-layout of int16 ids [N, K] into the packed stream (``wal_idroute_pack``)."""
    lib = _abi.load()
    N, K = (int(v) for v in ids.shape)
    t = ids.detach().cpu()
    if t.dtype != torch.int16:
        t64 = t.to(torch.int64)
        if int(t64.min()) < 0 or int(t64.max()) >= num_routes:
            raise ValueError("id out of range of the route table")
        t = t64.to(torch.int16)
    a = np.ascontiguousarray(t.numpy())
    nbytes = ctypes.c_size_t(0)
    _abi.check(lib.wal_idroute_packed_size(N, K, ctypes.byref(nbytes)), "wal_idroute_packed_size")
    packed = torch.empty(int(nbytes.value), dtype=torch.uint8)
    _abi.check(lib.wal_idroute_pack(N, K, int(num_routes), a.ctypes.data, packed.data_ptr(), nbytes.value),
               "wal_idroute_pack")
    return packed


class PackedIDRouteLinear(nn.Module):
    """Drop-in for reference ``PackedIDRouteLinear`` over the fused CUDA ID-route GEMV."""

    def __init__(self, ids: Tensor, codebook_w: Tensor, row_scale: Tensor, bias: Optional[Tensor] = None) -> None:
        super().__init__()
        if ids.dim() != 2:
            raise ValueError("ids must be [out_features, in_features]")
        routes = int(codebook_w.shape[0])
        if routes > 32767:
            raise ValueError("route tables larger than 32767 entries are not supported (int16 ids)")
        if int(ids.shape[1]) % 8:
            raise ValueError("in_features must be a multiple of 8")
        self.out_features, self.in_features = (int(v) for v in ids.shape)
        self.num_routes = routes
        # the route table: the same reduction and cast as reference src/runtime.py:65-67
        self.register_buffer("codebook_sum", codebook_w.sum(dim=-1).contiguous().to(torch.float16))
        self.register_buffer("row_scale", row_scale.to(torch.float16).reshape(-1).contiguous())
        self.register_buffer("packed_ids", pack_ids(ids, routes))
        if bias is not None:
            # reference keeps an fp16 bias and casts it to x.dtype in the forward
            self.register_buffer("bias", bias.to(torch.float16).to(torch.bfloat16).reshape(-1).contiguous())
        else:
            self.bias = None
        self._layer_cache = None

    @classmethod
    def from_encoded(cls, ids: Tensor, codebook_digits: Tensor, ladder: Tensor, row_scale: Tensor,
                     bias: Optional[Tensor] = None, **_: object) -> "PackedIDRouteLinear":
        """Same folding of digits and ladder as reference ``src/runtime.py:77-87``."""
        codebook_w = (codebook_digits.to(torch.float32) * ladder.to(torch.float32)).to(torch.float16)
        return cls(ids, codebook_w, row_scale.to(torch.float16), bias)

    @classmethod
    def random(cls, out_features: int, in_features: int, *, routes: int = 1536, L: int = 12,
               generator: Optional[torch.Generator] = None, device: torch.device | str = "cuda") -> "PackedIDRouteLinear":
        """Seeded random ID-route linear built directly on ``device`` (benchmark stacks).

        Uniform ids are written straight into the packed stream (any
        permutation of uniform ids is uniform; padding positions too, which
        only meet zero activations), so no [N, K] host tensor is materialised.
        """
        if in_features % 8:
            raise ValueError("in_features must be a multiple of 8")
        device = torch.device(device)
        obj = cls.__new__(cls)
        nn.Module.__init__(obj)
        obj.out_features, obj.in_features, obj.num_routes = int(out_features), int(in_features), int(routes)
        tiles, chunks = -(-out_features // 16), -(-in_features // 128)
        ids = torch.randint(0, routes, (tiles * chunks * 2048,), device=device, generator=generator, dtype=torch.int32)
        obj.register_buffer("packed_ids", ids.to(torch.int16).view(torch.uint8).contiguous())
        book = (torch.randn(routes, L, device=device, generator=generator) * 0.01).to(torch.float16)
        obj.register_buffer("codebook_sum", book.sum(dim=-1).to(torch.float16).contiguous())
        rho = (torch.rand(out_features, device=device, generator=generator) + 0.5).to(torch.float16)
        obj.register_buffer("row_scale", rho.contiguous())
        obj.bias = None
        obj._layer_cache = None
        return obj

    def layer_struct(self) -> _abi.IDRouteLayer:
        key = (self.packed_ids.data_ptr(), self.codebook_sum.data_ptr(), self.row_scale.data_ptr(),
               None if self.bias is None else self.bias.data_ptr())
        if self._layer_cache is not None and self._layer_cache[0] == key:
            return self._layer_cache[1]
        layer = _abi.IDRouteLayer(out_features=self.out_features, in_features=self.in_features,
                                  num_routes=self.num_routes, packed_ids=key[0], codebook_sum=key[1],
                                  row_scale=key[2], bias=key[3])
        self._layer_cache = (key, layer)
        return layer

    def _require_cuda(self, t: Tensor) -> None:
        if not t.is_cuda:
            raise ValueError("PackedIDRouteLinear runs on CUDA only (no CPU path); move the input and the module "
                             "to a CUDA device")
        if self.packed_ids.device != t.device:
            raise ValueError(f"input on {t.device} but module buffers on {self.packed_ids.device}")

    def gemv_into(self, x2: Tensor, y: Tensor) -> None:
        lib = _abi.load()
        with torch.cuda.device(x2.device):
            st = lib.wal_idroute_gemv(ctypes.byref(self.layer_struct()), x2.data_ptr(), x2.shape[0], x2.stride(0),
                                      y.data_ptr(), y.stride(0), _abi.DTYPE_CODE[y.dtype],
                                      _abi.stream_handle(x2.device))
        _abi.check(st, "wal_idroute_gemv")

    def forward(self, x: Tensor) -> Tensor:
        self._require_cuda(x)
        if x.dtype != torch.bfloat16:
            raise ValueError(f"PackedIDRouteLinear expects bfloat16 activations, got {x.dtype}")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"Feature mismatch: {x.shape[-1]} != {self.in_features}")
        orig = x.shape
        x2 = x.reshape(-1, self.in_features)
        if x2.stride(-1) != 1 or x2.stride(0) % 4 != 0 or x2.data_ptr() % 8 != 0:
            x2 = x2.contiguous()
        y = torch.empty((x2.shape[0], self.out_features), device=x.device, dtype=torch.bfloat16)
        if x2.shape[0] > 0:
            self.gemv_into(x2, y)
        return y.reshape(*orig[:-1], self.out_features)

    def reconstruct_weight(self, out_dtype: torch.dtype = torch.float16) -> Tensor:
        """fp16: the reference's ``reconstruct_weight``; bf16: the forward's weight."""
        if out_dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("reconstruct_weight supports torch.float16 and torch.bfloat16")
        dev = self.packed_ids.device
        if dev.type != "cuda":
            raise ValueError("reconstruct_weight runs on CUDA only; move the module to a CUDA device")
        w = torch.empty((self.out_features, self.in_features), device=dev, dtype=out_dtype)
        lib = _abi.load()
        with torch.cuda.device(dev):
            st = lib.wal_idroute_dequant(ctypes.byref(self.layer_struct()), w.data_ptr(), w.stride(0),
                                         _abi.DTYPE_CODE[out_dtype], _abi.stream_handle(dev))
        _abi.check(st, "wal_idroute_dequant")
        return w

    def compressed_bytes(self) -> int:
        return self.out_features * self.in_features * 2 + self.num_routes * 2 + self.out_features * 2

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, routes={self.num_routes}"


# The reference's fused class runs its own Triton kernel with different rounding;
# here both names run the one kernel above (reference numerics of the packed path).
FusedIDRouteLinear = PackedIDRouteLinear
