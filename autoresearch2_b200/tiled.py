"""The 128x128 (vals, meta) variant of the tiled format.

Mirrors old/full_matmul/sparse_pack.py:95-146 (dense_to_tilesparse(dense,
BLOCK_M=128, BLOCK_N=128) -> (vals, meta)) and old/full_matmul/sparse_unpack.py:44-73
(bitsparse_unpack(vals, meta, shape) -> float32 dense).  It shares its name
with the flat bitsparse_unpack, so it lives in its own namespace.
"""
import torch

from . import _lib
from .bitsparse import BitsparseTensor, dense_to_tilesparse as _pack, tile_unpack

__all__ = ["dense_to_tilesparse", "bitsparse_unpack"]


def dense_to_tilesparse(dense: torch.Tensor, BLOCK_M: int = 128, BLOCK_N: int = 128):
    """Returns (vals, meta) with meta keys bitmask, prefix, grid_m, grid_n,
    BLOCK_M, BLOCK_N, shape; vals has exactly nnz elements (one device sync,
    like the reference's .item() at sparse_pack.py:128)."""
    _lib.require_cuda(dense)
    M, N = dense.shape
    arena = torch.empty(M * N, dtype=dense.dtype, device=dense.device)
    offset = torch.zeros(1, dtype=torch.int32, device=dense.device)
    x = _pack(dense, arena, offset, BLOCK_M, BLOCK_N)
    nnz = int(offset.item())
    meta = {"bitmask": x.bitmask, "prefix": x.prefix, "grid_m": x.grid_m, "grid_n": x.grid_n,
            "BLOCK_M": BLOCK_M, "BLOCK_N": BLOCK_N, "shape": (M, N)}
    return arena[:nnz], meta


def bitsparse_unpack(vals: torch.Tensor, meta: dict, shape) -> torch.Tensor:
    """float32 dense [shape] from (vals, meta) (the reference always returns float32)."""
    _lib.require_cuda(vals)
    zero = torch.zeros(1, dtype=torch.int32, device=vals.device)
    x = BitsparseTensor(vals.contiguous(), meta["bitmask"], meta["prefix"], zero, meta["grid_m"],
                        meta["grid_n"], meta["BLOCK_M"], meta["BLOCK_N"], tuple(shape))
    return tile_unpack(x, out_dtype=torch.float32)
