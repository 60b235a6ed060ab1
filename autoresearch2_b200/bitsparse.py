"""Bitmask-sparse formats with the reference's Python API, on the CUDA library.

Flat format (old/sparse_pack.py, old/sparse_unpack.py):
    bitsparse_pack(dense, block=2048) -> (vals, packed_mask)
    bitsparse_unpack(vals, packed_mask, shape, block=8192) -> dense
Tiled format (old/lib_sparse/sparse.py):
    BitsparseTensor, dense_to_tilesparse(dense, vals, offset, BLOCK_M=64, BLOCK_N=64),
    spAx(x_sparse, W, square=False), mask_with_bitmask_(grad, x_sparse),
    grad_relu2_(grad, x_sparse, square=True)
Vals arena (old/lib_sparse/prepare.py:15-33, testing/test.py:68-70):
    init_sparse_buffer, reset_sparse_globals, get_globals, TensorBuffer

`block=` arguments are accepted for signature compatibility and ignored: the
single-pass kernels do not depend on them, and neither do the output bytes
(in the reference they do not either).
"""
import math

import torch

from . import _lib
from ._lib import call, dtype_code, ptr, require_cuda, stream_ptr

__all__ = [
    "bitsparse_pack", "bitsparse_pack_async", "bitsparse_unpack", "BitsparseTensor", "dense_to_tilesparse", "tile_unpack",
    "spAx", "mask_with_bitmask_", "grad_relu2_", "init_sparse_buffer", "reset_sparse_globals",
    "get_globals", "TensorBuffer", "check_status",
]

check_status = _lib.check_status


# ---------------------------------------------------------------------------
# Flat format
# ---------------------------------------------------------------------------
def bitsparse_pack(dense: torch.Tensor, block: int = 2048, vals_out: torch.Tensor = None):
    """Pack a dense CUDA tensor into (vals, packed_mask).

    Follows old/sparse_pack.py:66-106: packed_mask is uint8[ceil(N/8)] with
    element f at byte f//8, bit f%8 (set iff x != 0); vals holds the nonzeros
    in row-major order.  Two kernels (mask, counts and the values staged per
    tile, then the values moved to their offsets); between them the call
    waits for the count, as the reference does to size vals
    (old/sparse_pack.py:98), so that vals holds exactly nnz elements.
    `vals_out` (optional, 1-D, same dtype, >= nnz elements) receives the
    values instead of a fresh buffer (a view of its first nnz is returned);
    bitsparse_pack_async skips the wait."""
    require_cuda(dense)
    code = dtype_code(dense)
    flat = dense.contiguous().view(-1)
    n = flat.numel()
    dev = dense.device
    L = _lib.load()
    mask = torch.empty((n + 7) // 8, dtype=torch.uint8, device=dev)
    out = torch.zeros(2, dtype=torch.int64, device=dev)  # [nnz, status]
    ws = _lib.workspace(L.sffn_flat_pack_workspace_bytes(n, code), dev)
    nnz_p, status_p = _lib.ctypes.c_void_p(out.data_ptr()), _lib.ctypes.c_void_p(out.data_ptr() + 8)
    st = stream_ptr(dev)
    call("sffn_flat_pack_count", ptr(flat), code, n, ptr(mask), nnz_p, ptr(ws), ws.numel(), st)
    nnz = int(out[0].item())
    if vals_out is not None:
        if vals_out.dtype != dense.dtype or not vals_out.is_contiguous() or vals_out.numel() < nnz:
            raise ValueError("vals_out must be a contiguous tensor of the input's dtype with >= nnz elements")
        vals = vals_out
    else:
        vals = torch.empty(nnz, dtype=dense.dtype, device=dev)
    call("sffn_flat_pack_values", code, n, ptr(vals), vals.numel(), nnz_p, ptr(ws), ws.numel(), status_p, st)
    return vals[:nnz], mask


def bitsparse_pack_async(dense: torch.Tensor, vals_out: torch.Tensor):
    """bitsparse_pack without a host wait: the values go to `vals_out` (a
    caller-sized upper bound, e.g. an arena), and the count stays on the
    device.  Returns (vals_out, packed_mask, nnz) with nnz an int64 [1] CUDA
    tensor; more nonzeros than vals_out holds are clipped and flag
    SFFN_STATUS_VALS_OVERFLOW in the device status word (check_status)."""
    require_cuda(dense, vals_out)
    code = dtype_code(dense)
    if vals_out.dtype != dense.dtype or not vals_out.is_contiguous():
        raise ValueError("vals_out must be a contiguous tensor of the input's dtype")
    flat = dense.contiguous().view(-1)
    n = flat.numel()
    dev = dense.device
    mask = torch.empty((n + 7) // 8, dtype=torch.uint8, device=dev)
    nnz = torch.zeros(1, dtype=torch.int64, device=dev)
    ws = _lib.workspace(_lib.load().sffn_flat_pack_workspace_bytes(n, code), dev)
    call("sffn_flat_pack", ptr(flat), code, n, ptr(mask), ptr(vals_out), vals_out.numel(), ptr(nnz),
         ptr(ws), ws.numel(), ptr(_lib.status_word(dev)), stream_ptr(dev))
    return vals_out, mask, nnz


def compress_dense(dense: torch.Tensor, shape, block: int = 2048):
    """The flat pack under its earlier name and signature
    (old/bitpack/train.py:65-103): dense [rows, cols] with shape = (rows,
    cols) -> (vals, packed_mask), as bitsparse_pack."""
    rows, cols = (int(d) for d in shape)
    if dense.numel() != rows * cols:
        raise ValueError(f"dense has {dense.numel()} elements, shape {tuple(shape)} needs {rows * cols}")
    return bitsparse_pack(dense.reshape(rows, cols), block)


def reconstruct_bitmask(vals: torch.Tensor, packed_mask: torch.Tensor, shape, block: int = 8192):
    """The flat unpack under its earlier name (old/bitunpack/train.py:55-90),
    as bitsparse_unpack."""
    return bitsparse_unpack(vals, packed_mask, shape, block)


def bitsparse_unpack(vals: torch.Tensor, packed_mask: torch.Tensor, shape, block: int = 8192):
    """Rebuild the dense tensor of `shape` (old/sparse_unpack.py:57-97)."""
    require_cuda(vals, packed_mask)
    if packed_mask.dtype != torch.uint8:
        raise ValueError("packed_mask must be uint8")
    code = dtype_code(vals)
    shape = tuple(int(s) for s in shape)
    n = math.prod(shape)
    if packed_mask.numel() < (n + 7) // 8:
        raise ValueError("packed_mask is shorter than ceil(N/8) bytes")
    vals = vals.contiguous()
    packed_mask = packed_mask.contiguous()
    dev = vals.device
    out = torch.empty(shape, dtype=vals.dtype, device=dev)
    ws = _lib.workspace(_lib.load().sffn_flat_workspace_bytes(n), dev)
    call("sffn_flat_unpack", ptr(vals), vals.numel(), ptr(packed_mask), code, n, ptr(out),
         ptr(ws), ws.numel(), ptr(_lib.status_word(dev)), stream_ptr(dev))
    return out


# ---------------------------------------------------------------------------
# Tiled format
# ---------------------------------------------------------------------------
class BitsparseTensor:
    """Tiled bitmask-sparse matrix (old/lib_sparse/sparse.py:16-53).

    vals: the vals arena (1-D); bitmask: uint8, BLOCK_M*BLOCK_N/8 bytes per
    tile; prefix: int32[num_tiles + 1]; vals_offset: int32[1] device copy of
    the arena cursor when this matrix was packed; tile t = tm*grid_n + tn
    keeps its values at vals[vals_offset + prefix[t]:...]."""

    def __init__(self, vals, bitmask, prefix, vals_offset, grid_m, grid_n, BLOCK_M, BLOCK_N, shape):
        self.vals = vals
        self.bitmask = bitmask
        self.prefix = prefix
        self.vals_offset = vals_offset
        self.grid_m = grid_m
        self.grid_n = grid_n
        self.BLOCK_M = BLOCK_M
        self.BLOCK_N = BLOCK_N
        self.shape = tuple(shape)

    def __repr__(self):
        return f"BitsparseTensor(shape={list(self.shape)}, nnz={self.vals.numel()})\n"

    def vram_size(self):
        """MB held by vals, bitmask and prefix (sparse.py:46-50)."""
        tot = sum(t.element_size() * t.nelement() for t in (self.vals, self.bitmask, self.prefix))
        return tot / 1024 ** 2

    def sparsity_ratio(self):
        """1 - len(vals)/numel (sparse.py:52-53; with an arena, len(vals) is
        the arena's length, exactly as in the reference)."""
        return 1 - self.vals.numel() / (self.shape[0] * self.shape[1])

    def nnz(self):
        """Number of stored values of this matrix (device sync)."""
        return int(self.prefix[-1].item())

    def to_dense(self, square=False, dtype=None):
        return tile_unpack(self, square=square, out_dtype=dtype)


def _grid(M, N, BM, BN):
    return (M + BM - 1) // BM, (N + BN - 1) // BN


def dense_to_tilesparse(dense: torch.Tensor, vals: torch.Tensor, offset: torch.Tensor,
                        BLOCK_M: int = 64, BLOCK_N: int = 64) -> BitsparseTensor:
    """Pack `dense` [M, N] into the tiled format (old/lib_sparse/sparse.py:154-210).

    Mutates the arena: values go to vals[offset + prefix[t] ...] and `offset`
    (int32[1], device) advances by the number of values, with no host sync.
    vals may instead be a callable alloc(n) -> vals (offset zero on entry):
    the tiles are counted first, the total read back (one device sync), and
    the values packed into alloc(nnz), a tensor of exactly nnz elements."""
    exact = callable(vals)
    require_cuda(dense, offset, *(() if exact else (vals,)))
    if dense.dim() != 2:
        raise ValueError("dense must be 2-D")
    if not exact and (vals.dtype != dense.dtype or vals.dim() != 1 or not vals.is_contiguous()):
        raise ValueError("vals must be a contiguous 1-D tensor of dense's dtype")
    if offset.dtype != torch.int32 or offset.numel() != 1:
        raise ValueError("offset must be an int32 tensor with one element")
    code = dtype_code(dense)
    if dense.stride(1) != 1:
        dense = dense.contiguous()
    M, N = dense.shape
    gm, gn = _grid(M, N, BLOCK_M, BLOCK_N)
    dev = dense.device
    bitmask = torch.empty(gm * gn * BLOCK_M * BLOCK_N // 8, dtype=torch.uint8, device=dev)
    prefix = torch.empty(gm * gn + 1, dtype=torch.int32, device=dev)
    vals_offset = torch.empty(1, dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = _lib.workspace(lib.sffn_tile_workspace_bytes(M, N, BLOCK_M, BLOCK_N), dev)
    status = ptr(_lib.status_word(dev))
    if exact:
        # mask, prefix and cursor first (no values), then exactly nnz values
        call("sffn_tile_pack", ptr(dense), code, M, N, dense.stride(0), BLOCK_M, BLOCK_N, ptr(bitmask),
             ptr(prefix), None, 0, ptr(offset), ptr(vals_offset), ptr(ws), ws.numel(), status, stream_ptr(dev))
        n = int(offset.item())
        vals = vals(n)
        if n:
            call("sffn_tile_pack_values", ptr(dense), code, M, N, dense.stride(0), BLOCK_M, BLOCK_N,
                 ptr(bitmask), ptr(prefix), ptr(vals), n, ptr(vals_offset), status, stream_ptr(dev))
        return BitsparseTensor(vals, bitmask, prefix, vals_offset, gm, gn, BLOCK_M, BLOCK_N, (M, N))
    call("sffn_tile_pack", ptr(dense), code, M, N, dense.stride(0), BLOCK_M, BLOCK_N, ptr(bitmask),
         ptr(prefix), ptr(vals), vals.numel(), ptr(offset), ptr(vals_offset), ptr(ws), ws.numel(),
         status, stream_ptr(dev))
    return BitsparseTensor(vals, bitmask, prefix, vals_offset, gm, gn, BLOCK_M, BLOCK_N, (M, N))


def tile_unpack(x: BitsparseTensor, row_start: int = 0, row_end: int = None, square=False,
                out=None, out_dtype=None, round_tf32=False):
    """Dense rows [row_start, row_end) of a BitsparseTensor (row_start a
    multiple of BLOCK_M), optionally squared in the storage dtype; float32
    output rounded to the nearest TF32 values with round_tf32 (the operand
    of a TF32 product).  Follows old/lib_sparse/sparse_unpack.py:5-55 with
    column bounds."""
    M, N = x.shape
    row_end = M if row_end is None else min(row_end, M)
    BM, BN = x.BLOCK_M, x.BLOCK_N
    if row_start % BM:
        raise ValueError("row_start must be a multiple of BLOCK_M")
    code = dtype_code(x.vals)
    out_dtype = x.vals.dtype if out_dtype is None else out_dtype
    ocode = dtype_code(torch.empty(0, dtype=out_dtype))
    rows = row_end - row_start
    if out is None:
        out = torch.empty(rows, N, dtype=out_dtype, device=x.vals.device)
    if out.shape[0] < rows or out.shape[1] != N or out.stride(1) != 1 or out.dtype != out_dtype:
        raise ValueError("out must be a row-major [rows, N] tensor of out_dtype")
    tr0 = row_start // BM
    trows = (row_end + BM - 1) // BM - tr0
    # Passing row_end as the row count makes the kernel skip rows past it.
    call("sffn_tile_unpack", ptr(x.vals), x.vals.numel(), ptr(x.bitmask), ptr(x.prefix),
         ptr(x.vals_offset), code, row_end, N, BM, BN, tr0, trows, int(bool(square)) | 2 * int(bool(round_tf32)),
         ptr(out),
         ocode, out.stride(0), stream_ptr(x.vals.device))
    return out


def spAx(x_sparse: BitsparseTensor, W: torch.Tensor, square: bool = False,
         row_batch: int = 4096) -> torch.Tensor:
    """y = W @ x_sparse (or W @ x_sparse**2) as in old/lib_sparse/sparse.py:305-351:
    x_sparse [M, N], W [K, M] -> [K, N], unpacked in row batches of `row_batch`
    rows (a multiple of BLOCK_M), each batch's product on this library's
    tcgen05 GEMM, accumulated in fp32: bf16 batches add straight into the
    float32 result in the GEMM's epilogue, float32 / float16 ones run as
    split-bf16 products."""
    from .gemm import matmul, mm_f32acc
    M, N = x_sparse.shape
    if W.shape[1] != M:
        raise ValueError(f"W.shape must be [K, {M}] for W @ sparse_x, got {tuple(W.shape)}")
    require_cuda(W)
    BM = x_sparse.BLOCK_M
    row_batch = max(BM, (row_batch // BM) * BM)
    K = W.shape[0]
    if M <= row_batch:
        return matmul(W, tile_unpack(x_sparse, 0, M, square=square).to(W.dtype))
    acc = torch.empty(K, N, device=W.device, dtype=torch.float32)
    for m0 in range(0, M, row_batch):
        m1 = min(m0 + row_batch, M)
        dense = tile_unpack(x_sparse, m0, m1, square=square).to(W.dtype)
        if W.dtype == torch.bfloat16:
            mm_f32acc(W[:, m0:m1], dense, acc, accumulate=m0 > 0)
        elif m0 == 0:
            acc.copy_(matmul(W[:, m0:m1], dense).float())
        else:
            acc += matmul(W[:, m0:m1], dense).float()
    return acc.to(W.dtype)


def mask_with_bitmask_(grad: torch.Tensor, x_sparse: BitsparseTensor) -> torch.Tensor:
    """In place grad = bit ? grad : 0 (old/lib_sparse/sparse_unpack.py:72-107)."""
    require_cuda(grad)
    M, N = x_sparse.shape
    if tuple(grad.shape) != (M, N) or grad.stride(1) != 1:
        raise ValueError("grad must be a row-major [M, N] tensor matching the sparse matrix")
    call("sffn_tile_mask_grad", ptr(grad), dtype_code(grad), M, N, grad.stride(0),
         ptr(x_sparse.bitmask), x_sparse.BLOCK_M, x_sparse.BLOCK_N, stream_ptr(grad.device))
    return grad


def grad_relu2_(grad: torch.Tensor, x_sparse: BitsparseTensor, square: bool = True) -> torch.Tensor:
    """In place grad = (grad*2)*z, z from the sparse matrix; if `square`,
    its stored values become z*z (old/lib_sparse/sparse_unpack.py:110-147)."""
    require_cuda(grad)
    M, N = x_sparse.shape
    if tuple(grad.shape) != (M, N) or grad.stride(1) != 1:
        raise ValueError("grad must be a row-major [M, N] tensor matching the sparse matrix")
    if grad.dtype != x_sparse.vals.dtype:
        raise ValueError("grad and the sparse values must share a dtype")
    call("sffn_tile_grad_relu2", ptr(grad), dtype_code(grad), M, N, grad.stride(0),
         ptr(x_sparse.vals), x_sparse.vals.numel(), ptr(x_sparse.bitmask), ptr(x_sparse.prefix),
         ptr(x_sparse.vals_offset), x_sparse.BLOCK_M, x_sparse.BLOCK_N, int(bool(square)),
         stream_ptr(grad.device))
    return grad


# ---------------------------------------------------------------------------
# Vals arena (old/lib_sparse/prepare.py:15-33; testing/test.py:68-70)
# ---------------------------------------------------------------------------
class TensorBuffer:
    """One preallocated vals buffer plus an int32 device cursor shared by all
    layers of a step; reset_buffer() rewinds the cursor."""

    def __init__(self, n, device, dtype):
        self.n, self.device, self.dtype = int(n), torch.device(device), dtype
        self.vals = None
        self.offset = None

    def init_buffer(self):
        self.vals = torch.empty(self.n, device=self.device, dtype=self.dtype)
        self.offset = torch.zeros(1, device=self.device, dtype=torch.int32)
        return self

    def reset_buffer(self):
        if self.offset is not None:
            self.offset.zero_()
        return self

    def used(self):
        """Values written since the last reset (device sync)."""
        return int(self.offset.item())

    def as_sparse_data(self):
        return self.vals, self.offset


_global = TensorBuffer(0, "cpu", torch.float32)


def init_sparse_buffer(size: int, device, dtype):
    """Allocate the global vals arena (old/lib_sparse/prepare.py:19-24)."""
    global _global
    _global = TensorBuffer(size, device, dtype).init_buffer()
    return _global


def reset_sparse_globals():
    _global.reset_buffer()


def get_globals():
    return _global.vals, _global.offset
