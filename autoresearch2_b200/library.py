"""torch.library custom ops (namespace ``sparseffn``) over the CUDA library.

torch.compile and torch.export trace through these ops without graph breaks;
the reference's own attempt to register its kernels as ops is commented out
(old/lib_sparse/sparse.py:212-298).  Each op's kernel is this package's
eager API, so it runs the same CUDA code; each fake kernel gives only the
outputs' shapes and dtypes, so tracing needs no device.

    sparseffn::bitsparse_pack(dense) -> (vals, packed_mask)
        old/sparse_pack.py:66-106; len(vals) = nnz is data-dependent (an
        unbacked size while tracing)
    sparseffn::bitsparse_unpack(vals, packed_mask, shape) -> dense
        old/sparse_unpack.py:57-97
    sparseffn::tile_pack(dense, vals!, offset!, block_m, block_n) -> (bitmask, prefix, vals_offset)
        dense_to_tilesparse, old/lib_sparse/sparse.py:154-210; writes the vals
        arena and advances its cursor in place
    sparseffn::tile_unpack(vals, bitmask, prefix, vals_offset, shape, block_m, block_n, square)
        -> dense, old/lib_sparse/sparse_unpack.py:5-55
    sparseffn::ffn_fwd(x, W1, W2, b1?, vals!, offset!, act)
        -> (out, bitmask, prefix, vals_offset, row_offsets, kb_list, kb_count)
    sparseffn::ffn_bwd(grad_output, x, W1, W2, vals, bitmask, prefix, vals_offset, row_offsets,
                       kb_list, kb_count, fused, has_bias, act) -> (grad_x, grad_W1, grad_W2, grad_b1)
        the forward and backward of FFNSparse / FFNSpRelu2 (sparse.py:56-151),
        which call them; act is 0 (ReLU) or 1 (ReLU^2).  The ops that write the
        arena carry no autograd formula (torch.library allows none on a
        mutating op): the autograd.Function classes in ffn.py hold that.
    sparseffn::codec15_compress(data) -> stream
    sparseffn::codec15_uncompress(stream, shape, dtype) -> data
        the 15-bit sign-strip codec, bitshifting/code.py:129-177

The fused bf16 path (ffn._fused_ok, decided from dtypes, contiguity and
shapes alone) keeps z in 128x128 tiles and returns per-row value offsets and
K-block lists; the float32 / float16 path keeps 64x64 tiles and returns
those three as empty tensors, as it does grad_b1 when there is no bias.
"""
from typing import Optional

import torch
from torch import Tensor

from . import bitshift
from . import bitsparse as bs
from . import ffn

__all__ = ["OPS"]

OPS = ("bitsparse_pack", "bitsparse_unpack", "tile_pack", "tile_unpack", "ffn_fwd", "ffn_bwd",
       "codec15_compress", "codec15_uncompress")


def _cdiv(a, b):
    return (a + b - 1) // b


def _i32(like, *shape):
    return torch.empty(shape, dtype=torch.int32, device=like.device)


# ---------------------------------------------------------------------------
# Flat format
# ---------------------------------------------------------------------------
@torch.library.custom_op("sparseffn::bitsparse_pack", mutates_args=())
def bitsparse_pack(dense: Tensor) -> tuple[Tensor, Tensor]:
    return bs.bitsparse_pack(dense)


@bitsparse_pack.register_fake
def _(dense):
    nnz = torch.library.get_ctx().new_dynamic_size()
    return dense.new_empty(nnz), dense.new_empty(_cdiv(dense.numel(), 8), dtype=torch.uint8)


@torch.library.custom_op("sparseffn::bitsparse_unpack", mutates_args=())
def bitsparse_unpack(vals: Tensor, packed_mask: Tensor, shape: list[int]) -> Tensor:
    return bs.bitsparse_unpack(vals, packed_mask, shape)


@bitsparse_unpack.register_fake
def _(vals, packed_mask, shape):
    return vals.new_empty(shape)


# ---------------------------------------------------------------------------
# Tiled format
# ---------------------------------------------------------------------------
@torch.library.custom_op("sparseffn::tile_pack", mutates_args=("vals", "offset"))
def tile_pack(dense: Tensor, vals: Tensor, offset: Tensor, block_m: int,
              block_n: int) -> tuple[Tensor, Tensor, Tensor]:
    x = bs.dense_to_tilesparse(dense, vals, offset, block_m, block_n)
    return x.bitmask, x.prefix, x.vals_offset


@tile_pack.register_fake
def _(dense, vals, offset, block_m, block_n):
    nt = _cdiv(dense.shape[0], block_m) * _cdiv(dense.shape[1], block_n)
    return (dense.new_empty(nt * block_m * block_n // 8, dtype=torch.uint8), _i32(dense, nt + 1),
            _i32(dense, 1))


@torch.library.custom_op("sparseffn::tile_unpack", mutates_args=())
def tile_unpack(vals: Tensor, bitmask: Tensor, prefix: Tensor, vals_offset: Tensor, shape: list[int],
                block_m: int, block_n: int, square: bool) -> Tensor:
    M, N = shape
    x = bs.BitsparseTensor(vals, bitmask, prefix, vals_offset, _cdiv(M, block_m), _cdiv(N, block_n),
                           block_m, block_n, (M, N))
    return bs.tile_unpack(x, square=square)


@tile_unpack.register_fake
def _(vals, bitmask, prefix, vals_offset, shape, block_m, block_n, square):
    return vals.new_empty(shape)


# ---------------------------------------------------------------------------
# FFN forward / backward
# ---------------------------------------------------------------------------
@torch.library.custom_op("sparseffn::ffn_fwd", mutates_args=("vals", "offset"))
def ffn_fwd(x: Tensor, W1: Tensor, W2: Tensor, b1: Optional[Tensor], vals: Tensor, offset: Tensor,
            act: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    if ffn._fused_ok(x, W1, W2, b1, vals):
        return ffn._fused_forward(x, W1, W2, vals, offset, b1, act)
    out, z = ffn._unfused_forward(x, W1, W2, vals, offset, b1, act)
    return out, z.bitmask, z.prefix, z.vals_offset, _i32(x, 0), _i32(x, 0, 0), _i32(x, 0)


@ffn_fwd.register_fake
def _(x, W1, W2, b1, vals, offset, act):
    T, Fd, D = x.shape[0], W1.shape[0], W2.shape[0]
    fused = ffn._fused_ok(x, W1, W2, b1, vals)
    bm = 128 if fused else 64
    nt = _cdiv(T, bm) * _cdiv(Fd, bm)
    out = x.new_empty(T, D)
    bitmask = x.new_empty(nt * bm * bm // 8, dtype=torch.uint8)
    if fused:
        aux = (_i32(x, nt * 128), _i32(x, _cdiv(T, 256), _cdiv(Fd, 64)), _i32(x, _cdiv(T, 256)))
    else:
        aux = (_i32(x, 0), _i32(x, 0, 0), _i32(x, 0))
    return (out, bitmask, _i32(x, nt + 1), _i32(x, 1)) + aux


@torch.library.custom_op("sparseffn::ffn_bwd", mutates_args=())
def ffn_bwd(grad_output: Tensor, x: Tensor, W1: Tensor, W2: Tensor, vals: Tensor, bitmask: Tensor,
            prefix: Tensor, vals_offset: Tensor, row_offsets: Tensor, kb_list: Tensor,
            kb_count: Tensor, fused: bool, has_bias: bool,
            act: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    T, Fd = x.shape[0], W1.shape[0]
    bm = 128 if fused else 64
    z = bs.BitsparseTensor(vals, bitmask, prefix, vals_offset, _cdiv(T, bm), _cdiv(Fd, bm), bm, bm,
                           (T, Fd))
    if fused:
        grads = ffn._fused_backward(grad_output, x, W1, W2, z, row_offsets, kb_list, kb_count,
                                    has_bias, act)
    else:
        grads = ffn._unfused_backward(grad_output, x, W1, W2, z, has_bias, act)
    grad_x, grad_W1, grad_W2, grad_b1 = grads
    if grad_b1 is None:
        grad_b1 = x.new_empty(0)
    return grad_x, grad_W1, grad_W2, grad_b1


@ffn_bwd.register_fake
def _(grad_output, x, W1, W2, vals, bitmask, prefix, vals_offset, row_offsets, kb_list, kb_count,
      fused, has_bias, act):
    return (x.new_empty(x.shape), W1.new_empty(W1.shape), W2.new_empty(W2.shape),
            x.new_empty(W1.shape[0] if has_bias else 0))


# ---------------------------------------------------------------------------
# 15-bit sign-strip codec
# ---------------------------------------------------------------------------
@torch.library.custom_op("sparseffn::codec15_compress", mutates_args=())
def codec15_compress(data: Tensor) -> Tensor:
    return bitshift.compress_fn(data)


@codec15_compress.register_fake
def _(data):
    return data.new_empty(bitshift.padded_bytes(data.numel()), dtype=torch.uint8)


@torch.library.custom_op("sparseffn::codec15_uncompress", mutates_args=())
def codec15_uncompress(compressed: Tensor, shape: list[int], dtype: torch.dtype) -> Tensor:
    return bitshift.uncompress_fn(compressed, shape, dtype)


@codec15_uncompress.register_fake
def _(compressed, shape, dtype):
    return compressed.new_empty(shape, dtype=dtype)
