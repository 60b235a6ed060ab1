"""2:4 structured products on the sparse tensor cores (tcgen05.mma.sp).

A sparse bf16 matrix A [M, K] (here: the FFN activations or their gradients,
~90% zeros in no fixed pattern) is split by ``compress`` into its 2:4 part --
per group of four consecutive K elements the first two non-zeros, which the
sparse tensor cores multiply at twice the dense rate -- and its overflow (the
3rd and 4th non-zero of a group, a fraction of a percent of the groups at 90%
zeros), which ``mm`` adds on the CUDA cores.  The reference has no such path:
its products are dense cuBLAS matmuls (old/lib_sparse/sparse.py:75,95-100,
118,136-139), and ``mm`` returns the same product to bf16 rounding.
"""
import ctypes

import torch

from . import _lib
from ._lib import call, ptr, stream_ptr

__all__ = ["Sp24", "compress", "mm", "transpose"]


class Sp24:
    """A [M, K] in 2:4 form: vals [M, K/2], meta (tensor-memory lane order,
    int32 [M/128, K/128, 128, 4]), overflow per row: cols/vals [M, K/2],
    count [M]."""

    def __init__(self, vals, meta, ovf_cols, ovf_vals, ovf_count, shape):
        self.vals, self.meta = vals, meta
        self.ovf_cols, self.ovf_vals, self.ovf_count = ovf_cols, ovf_vals, ovf_count
        self.shape = tuple(shape)

    @classmethod
    def empty(cls, M, K, device):
        """Uninitialised storage for an [M, K] matrix (M, K multiples of 128)."""
        if M % 128 or K % 128:
            raise ValueError(f"2:4 form needs both sizes divisible by 128, got {M} x {K}")
        return cls(torch.empty(M, K // 2, dtype=torch.bfloat16, device=device),
                   torch.empty(M // 128, K // 128, 128, 4, dtype=torch.int32, device=device),
                   torch.empty(M, K // 2, dtype=torch.int16, device=device),
                   torch.empty(M, K // 2, dtype=torch.bfloat16, device=device),
                   torch.empty(M, dtype=torch.int32, device=device), (M, K))

    def desc(self):
        """The C struct sffn_sp24_mat of this matrix (keep it alive over the call)."""
        return (ctypes.c_void_p * 5)(ptr(self.vals), ptr(self.meta), ptr(self.ovf_cols), ptr(self.ovf_vals),
                                     ptr(self.ovf_count))


def compress(A: torch.Tensor, trans: bool = False) -> Sp24:
    """2:4 form of A (bf16, row-major [M, K]); with trans=True, of A = X^T for
    the given row-major X [K, M] (no transposed copy is made)."""
    _lib.require_cuda(A)
    if A.dtype != torch.bfloat16 or A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("compress takes a row-major 2-D bfloat16 tensor")
    K, M = A.shape if trans else A.shape[::-1]
    if M % 128 or K % 128:
        raise ValueError(f"2:4 form needs both sizes divisible by 128, got {M} x {K}")
    out = Sp24.empty(M, K, A.device)
    call("sffn_sp24_compress", ptr(A), A.stride(0), 1 if trans else 0, M, K, ptr(out.vals), ptr(out.meta),
         ptr(out.ovf_cols), ptr(out.ovf_vals), ptr(out.ovf_count), stream_ptr(A.device))
    return out


def transpose(X: torch.Tensor) -> torch.Tensor:
    """X^T as a new row-major tensor (16-bit X, row-major, both sizes
    multiples of 8)."""
    _lib.require_cuda(X)
    if X.element_size() != 2 or X.dim() != 2 or X.stride(1) != 1:
        raise ValueError("transpose takes a row-major 2-D 16-bit tensor")
    rows, cols = X.shape
    out = torch.empty(cols, rows, dtype=X.dtype, device=X.device)
    call("sffn_transpose16", ptr(X), X.stride(0), rows, cols, ptr(out), out.stride(0), stream_ptr(X.device))
    return out


def mm(a: Sp24, B: torch.Tensor, out: torch.Tensor = None, bt: torch.Tensor = None,
       trans_out: bool = False, fused: bool = False) -> torch.Tensor:
    """out = A @ B (bf16) for A in 2:4 form and B [K, N] bf16 that is
    row-major or a transposed view of a row-major [N, K] tensor; N a multiple
    of 32.  The 2:4 part runs on the sparse tensor cores; the overflow is
    added from bt, B as a row-major [K, N] tensor (B itself when B is
    row-major; made here if not given), by a second kernel or, with
    fused=True, in the GEMM's epilogue (one launch, bit-identical; faster
    only when rows carry few overflow entries, e.g. 95% zeros).
    trans_out=True returns (A @ B)^T as a row-major [N, M] tensor."""
    M, K = a.shape
    _lib.require_cuda(B)
    if B.dtype != torch.bfloat16 or B.shape[0] != K:
        raise ValueError(f"B must be bfloat16 [{K}, N]")
    N = B.shape[1]
    if B.stride(1) == 1:
        b_mn, ldb = 1, B.stride(0)
        if bt is None:
            bt = B
    elif B.stride(0) == 1:
        b_mn, ldb = 0, B.stride(1)
        if bt is None:
            bt = transpose(B.T)
    else:
        raise ValueError("B must be row-major or a transposed view of a row-major tensor")
    if bt.stride(1) != 1 or tuple(bt.shape) != (K, N):
        raise ValueError("bt must be a row-major [K, N] tensor")
    shape = (N, M) if trans_out else (M, N)
    if out is None:
        out = torch.empty(*shape, dtype=torch.bfloat16, device=B.device)
    elif tuple(out.shape) != shape or out.stride(1) != 1:
        raise ValueError(f"out must be a row-major {shape} tensor")
    dev = B.device
    st = stream_ptr(dev)
    status = ptr(_lib.status_word(dev))
    if fused:
        d = a.desc()
        call("sffn_sp24_mm", ctypes.addressof(d), M, K, ptr(B), ldb, b_mn, ptr(bt), bt.stride(0), ptr(out),
             out.stride(0), 1 if trans_out else 0, N, status, st)
        return out
    c = torch.empty(M, N, dtype=torch.bfloat16, device=dev) if trans_out else out
    call("sffn_gemm_sp24", ptr(a.vals), ptr(a.meta), M, K, ptr(B), ldb, b_mn, ptr(c), c.stride(0), N, status, st)
    call("sffn_sp24_overflow_add", ptr(a.ovf_cols), ptr(a.ovf_vals), ptr(a.ovf_count), M, K, ptr(bt),
         bt.stride(0), N, ptr(c), c.stride(0), st)
    if trans_out:
        call("sffn_transpose16", ptr(c), c.stride(0), M, N, ptr(out), out.stride(0), st)
    return out
