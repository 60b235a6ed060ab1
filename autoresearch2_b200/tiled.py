"""The 128x128 (vals, meta) variant of the tiled format.

Mirrors old/full_matmul/sparse_pack.py:95-146 (dense_to_tilesparse(dense,
BLOCK_M=128, BLOCK_N=128) -> (vals, meta)) and old/full_matmul/sparse_unpack.py:44-73
(bitsparse_unpack(vals, meta, shape) -> float32 dense).  It shares its name
with the flat bitsparse_unpack, so it lives in its own namespace.
"""
import torch

from . import _lib
from ._lib import call, dtype_code, ptr, stream_ptr
from .bitsparse import BitsparseTensor, tile_unpack

__all__ = ["dense_to_tilesparse", "bitsparse_unpack"]


def dense_to_tilesparse(dense: torch.Tensor, BLOCK_M: int = 128, BLOCK_N: int = 128):
    """Returns (vals, meta) with meta keys bitmask, prefix, grid_m, grid_n,
    BLOCK_M, BLOCK_N, shape; vals is allocated with exactly nnz elements:
    the mask and counts first, one device sync for the total (like the
    reference's .item() at sparse_pack.py:128), then the values."""
    _lib.require_cuda(dense)
    if dense.dim() != 2:
        raise ValueError("dense must be 2-D")
    if dense.stride(1) != 1:
        dense = dense.contiguous()
    M, N = dense.shape
    dev = dense.device
    gm, gn = -(-M // BLOCK_M), -(-N // BLOCK_N)
    code = dtype_code(dense)
    bitmask = torch.empty(gm * gn * BLOCK_M * BLOCK_N // 8, dtype=torch.uint8, device=dev)
    prefix = torch.empty(gm * gn + 1, dtype=torch.int32, device=dev)
    offset = torch.zeros(1, dtype=torch.int32, device=dev)
    vals_offset = torch.empty(1, dtype=torch.int32, device=dev)
    status = ptr(_lib.status_word(dev))
    ws = _lib.workspace(_lib.load().sffn_tile_workspace_bytes(M, N, BLOCK_M, BLOCK_N), dev)
    call("sffn_tile_pack", ptr(dense), code, M, N, dense.stride(0), BLOCK_M, BLOCK_N, ptr(bitmask), ptr(prefix),
         None, 0, ptr(offset), ptr(vals_offset), ptr(ws), ws.numel(), status, stream_ptr(dev))
    nnz = int(offset.item())
    vals = torch.empty(nnz, dtype=dense.dtype, device=dev)
    if nnz:
        call("sffn_tile_pack_values", ptr(dense), code, M, N, dense.stride(0), BLOCK_M, BLOCK_N, ptr(bitmask),
             ptr(prefix), ptr(vals), nnz, ptr(vals_offset), status, stream_ptr(dev))
    meta = {"bitmask": bitmask, "prefix": prefix, "grid_m": gm, "grid_n": gn,
            "BLOCK_M": BLOCK_M, "BLOCK_N": BLOCK_N, "shape": (M, N)}
    return vals, meta


def bitsparse_unpack(vals: torch.Tensor, meta: dict, shape) -> torch.Tensor:
    """float32 dense [shape] from (vals, meta) (the reference always returns float32)."""
    _lib.require_cuda(vals)
    zero = torch.zeros(1, dtype=torch.int32, device=vals.device)
    x = BitsparseTensor(vals.contiguous(), meta["bitmask"], meta["prefix"], zero, meta["grid_m"],
                        meta["grid_n"], meta["BLOCK_M"], meta["BLOCK_N"], tuple(shape))
    return tile_unpack(x, out_dtype=torch.float32)
