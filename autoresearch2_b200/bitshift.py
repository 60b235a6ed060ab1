"""15-bit sign-strip codec with the reference's API (bitshifting/code.py).

    compress_fn(data, dtype=None, device=None) -> uint8 stream
    uncompress_fn(compressed, shape, dtype, device=None) -> data

Non-negative bf16 / fp16 values carry a sign bit that is always 0; the codec
drops it and packs the remaining 15 bits of each value into one continuous
little-endian bit stream (value i at bits [15 i, 15 i + 15)), saving 1/16 of
the bytes.  Both directions run on the CUDA library (sffn_codec15_*); the
bytes equal the reference's for every input, including its handling of a set
sign bit (OR-ed into the next value's bit 0 unless that value starts a byte).
"""
import math

import torch

from . import _lib
from ._lib import call, ptr, require_cuda, stream_ptr

__all__ = ["compress_fn", "uncompress_fn", "compressed_bytes", "padded_bytes"]


def compressed_bytes(numel: int) -> int:
    """ceil(15 numel / 8), the stream's length (code.py:135)."""
    return (numel * 15 + 7) // 8


def padded_bytes(numel: int) -> int:
    """Length of compress_fn's buffer: the stream plus 8 bytes, rounded up to
    even (code.py:139-144)."""
    n = compressed_bytes(numel) + 8
    return n + n % 2


def compress_fn(data: torch.Tensor, dtype=None, device=None) -> torch.Tensor:
    """Pack the 16-bit values of `data` (any shape, 2-byte dtype) into a uint8
    buffer of padded_bytes(numel) bytes (code.py:129-160).  The first
    compressed_bytes(numel) bytes are the stream; the padding is left unset, as
    in the reference.  `dtype` and `device` are accepted for the reference's
    signature; the buffer is allocated on data's device (the reference
    allocates it on `device`, the CPU when that is None)."""
    require_cuda(data)
    if data.element_size() != 2:
        raise ValueError("compress_fn packs 16-bit data (bfloat16 / float16)")
    src = data.contiguous().view(-1)
    n = src.numel()
    out = torch.empty(padded_bytes(n), dtype=torch.uint8, device=data.device)
    call("sffn_codec15_compress", ptr(src), n, ptr(out), out.numel(), stream_ptr(data.device))
    return out


def uncompress_fn(compressed_tensor: torch.Tensor, shape, dtype, device=None) -> torch.Tensor:
    """Restore the values of `shape` and 16-bit `dtype` from the stream
    (code.py:163-177); every value comes back with sign bit 0."""
    require_cuda(compressed_tensor)
    if compressed_tensor.dtype != torch.uint8:
        raise ValueError("compressed_tensor must be uint8")
    if torch.empty(0, dtype=dtype).element_size() != 2:
        raise ValueError("uncompress_fn restores 16-bit data (bfloat16 / float16)")
    shape = tuple(int(s) for s in shape)
    n = math.prod(shape)
    src = compressed_tensor.contiguous().view(-1)
    if src.numel() < compressed_bytes(n):
        raise ValueError(f"compressed_tensor holds {src.numel()} bytes; {compressed_bytes(n)} needed")
    out = torch.empty(shape, dtype=dtype, device=compressed_tensor.device)
    call("sffn_codec15_uncompress", ptr(src), src.numel(), n, ptr(out), stream_ptr(out.device))
    return out
