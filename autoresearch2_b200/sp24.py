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
import torch

from . import _lib
from ._lib import call, ptr, stream_ptr

__all__ = ["Sp24", "compress", "mm"]


class Sp24:
    """A [M, K] in 2:4 form: vals [M, K/2], meta (tensor-memory lane order,
    int32 [M/128, K/128, 128, 4]), overflow per row: cols/vals [M, K/2],
    count [M]."""

    def __init__(self, vals, meta, ovf_cols, ovf_vals, ovf_count, shape):
        self.vals, self.meta = vals, meta
        self.ovf_cols, self.ovf_vals, self.ovf_count = ovf_cols, ovf_vals, ovf_count
        self.shape = tuple(shape)


def compress(A: torch.Tensor, trans: bool = False) -> Sp24:
    """2:4 form of A (bf16, row-major [M, K]); with trans=True, of A = X^T for
    the given row-major X [K, M] (no transposed copy is made)."""
    _lib.require_cuda(A)
    if A.dtype != torch.bfloat16 or A.dim() != 2 or A.stride(1) != 1:
        raise ValueError("compress takes a row-major 2-D bfloat16 tensor")
    K, M = A.shape if trans else A.shape[::-1]
    if M % 128 or K % 128:
        raise ValueError(f"2:4 form needs both sizes divisible by 128, got {M} x {K}")
    dev = A.device
    vals = torch.empty(M, K // 2, dtype=torch.bfloat16, device=dev)
    meta = torch.empty(M // 128, K // 128, 128, 4, dtype=torch.int32, device=dev)
    ovf_cols = torch.empty(M, K // 2, dtype=torch.int16, device=dev)
    ovf_vals = torch.empty(M, K // 2, dtype=torch.bfloat16, device=dev)
    ovf_count = torch.empty(M, dtype=torch.int32, device=dev)
    call("sffn_sp24_compress", ptr(A), A.stride(0), 1 if trans else 0, M, K, ptr(vals), ptr(meta),
         ptr(ovf_cols), ptr(ovf_vals), ptr(ovf_count), stream_ptr(dev))
    return Sp24(vals, meta, ovf_cols, ovf_vals, ovf_count, (M, K))


def mm(a: Sp24, B: torch.Tensor, out: torch.Tensor = None, bt: torch.Tensor = None) -> torch.Tensor:
    """out = A @ B (bf16) for A in 2:4 form and B [K, N] bf16 that is
    row-major or a transposed view of a row-major [N, K] tensor.  The overflow
    is added from bt, B as a row-major [K, N] tensor (B itself when B is
    row-major; made here if not given)."""
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
            bt = B.contiguous()
    else:
        raise ValueError("B must be row-major or a transposed view of a row-major tensor")
    if bt.stride(1) != 1 or tuple(bt.shape) != (K, N):
        raise ValueError("bt must be a row-major [K, N] tensor")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=B.device)
    dev = B.device
    st = stream_ptr(dev)
    call("sffn_gemm_sp24", ptr(a.vals), ptr(a.meta), M, K, ptr(B), ldb, b_mn, ptr(out), out.stride(0), N,
         ptr(_lib.status_word(dev)), st)
    call("sffn_sp24_overflow_add", ptr(a.ovf_cols), ptr(a.ovf_vals), ptr(a.ovf_count), M, K, ptr(bt),
         bt.stride(0), N, ptr(out), out.stride(0), st)
    return out
