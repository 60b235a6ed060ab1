"""bf16 tcgen05 GEMM and the fused FFN kernels, called through the C ABI.

mm(A, B) computes A @ B for 2-D bf16 CUDA tensors that are row-major or
transposed views of row-major tensors (the kernel reads either major order
directly, so no transposed copies are made).
"""
import ctypes

import torch

from . import _lib
from ._lib import call, ptr, stream_ptr

ACT_RELU, ACT_RELU2 = 0, 1
FORMAT_TILE = 128


def _operand(t, rows_dim):
    """(ld, mn_major) of a 2-D operand whose row index is dim `rows_dim` of
    the mathematical [rows, K] (A) or [K, cols] (B) view."""
    s0, s1 = t.stride()
    if rows_dim == 0:  # A [M, K]
        if s1 == 1:
            return s0, 0
        if s0 == 1:
            return s1, 1
    else:  # B [K, N]: the kernel wants the [N, K] operand
        if s0 == 1:
            return s1, 0
        if s1 == 1:
            return s0, 1
    raise ValueError("operands must be row-major or transposed views of row-major tensors")


def mm(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor = None, kb_list=None, kb_count=None):
    """C = A @ B (bf16 in, fp32 accumulate, bf16 out) on the tcgen05 kernel.

    kb_list / kb_count (int32, from live_kblocks) restrict 256-row tile m of A
    to the listed 64-wide K blocks (the rest of A's row tile must be zero there)."""
    _lib.require_cuda(A, B)
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
        raise TypeError("mm takes bfloat16 operands")
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    lda, a_mn = _operand(A, 0)
    ldb, b_mn = _operand(B, 1)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=A.device)
    if out.stride(1) != 1 or tuple(out.shape) != (M, N):
        raise ValueError("out must be a row-major [M, N] tensor")
    stride = 0
    if kb_list is not None:
        stride = kb_list.shape[1]
    call("sffn_gemm_bf16", ptr(A), lda, a_mn, ptr(B), ldb, b_mn, ptr(out), out.stride(0), M, N, K,
         ptr(kb_list), ptr(kb_count), stride, ptr(_lib.status_word(A.device)), stream_ptr(A.device))
    return out


def split3(X: torch.Tensor, b_order: bool) -> torch.Tensor:
    """[rows, 6 * cols] bf16: the three-term bf16 split of a 2-D float32 /
    float16 tensor (any strides), blocks hi hi mid hi lo mid (A) or hi mid hi
    lo hi mid (b_order, for B^T)."""
    rows, cols = X.shape
    ld = -(-6 * cols // 8) * 8  # 16-byte aligned rows for the TMA loads
    out = torch.empty(rows, ld, dtype=torch.bfloat16, device=X.device)
    call("sffn_split_bf16x3", ptr(X), _lib.dtype_code(X), rows, cols, X.stride(0), X.stride(1), ptr(out), ld,
         int(bool(b_order)), stream_ptr(X.device))
    return out


def matmul(A: torch.Tensor, B: torch.Tensor, relu: bool = False) -> torch.Tensor:
    """A @ B on this library's tcgen05 GEMM, in A's dtype (max(., 0) of it
    with relu, applied by the epilogue).  bfloat16 runs directly (fp32
    accumulation); float32 and float16 run as the split-bf16 product (three
    bf16 pieces per operand, six cross products, fp32 accumulation and
    output): the float32 product up to terms of relative size 2^-24, where a
    TF32 product keeps 2^-11."""
    _lib.require_cuda(A, B)
    if A.dtype != B.dtype:
        raise TypeError("matmul operands must share a dtype")
    if A.dtype == torch.bfloat16:
        return mm_relu(A, B) if relu else mm(A, B)
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    a3, b3 = split3(A, False), split3(B.T, True)
    C = torch.empty(M, N, dtype=torch.float32, device=A.device)
    call("sffn_gemm_bf16_f32out", ptr(a3), a3.stride(0), 0, ptr(b3), b3.stride(0), 0, ptr(C), C.stride(0), M, N,
         6 * K, int(bool(relu)), ptr(_lib.status_word(A.device)), stream_ptr(A.device))
    return C if A.dtype == torch.float32 else C.to(A.dtype)


def mm_relu(A: torch.Tensor, B: torch.Tensor, out_dtype=torch.bfloat16, kb_list=None, kb_count=None):
    """max(A @ B, 0) (bf16 operands, fp32 accumulation) in bf16 or float32,
    the ReLU applied by the GEMM's epilogue; kb_list / kb_count as in mm."""
    _lib.require_cuda(A, B)
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
        raise TypeError("mm_relu takes bfloat16 operands")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("mm_relu stores bfloat16 or float32")
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    lda, a_mn = _operand(A, 0)
    ldb, b_mn = _operand(B, 1)
    out = torch.empty(M, N, dtype=out_dtype, device=A.device)
    stride = kb_list.shape[1] if kb_list is not None else 0
    call("sffn_gemm_relu", ptr(A), lda, a_mn, ptr(B), ldb, b_mn, ptr(out), int(out_dtype == torch.float32),
         out.stride(0), M, N, K, ptr(kb_list), ptr(kb_count), stride, ptr(_lib.status_word(A.device)),
         stream_ptr(A.device))
    return out


def round_tf32(X: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """X (float32) rounded to the nearest TF32 values (ties away from zero),
    into out (a new tensor by default; out=X rounds in place)."""
    _lib.require_cuda(X)
    if X.dtype != torch.float32:
        raise TypeError("round_tf32 takes float32")
    X = X.contiguous()
    out = torch.empty_like(X) if out is None else out
    if out.shape != X.shape or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor of X's shape")
    call("sffn_round_tf32", ptr(X), ptr(out), X.numel(), stream_ptr(X.device))
    return out


def matmul_tf32(A: torch.Tensor, Bt: torch.Tensor, relu: bool = False, round_inputs: bool = False) -> torch.Tensor:
    """A @ Bt.T in float32 on the tcgen05 kind::tf32 path: A [M, K] and Bt
    [N, K] float32, read as TF32 by the tensor cores, float32 accumulation;
    max(., 0) applied by the epilogue with relu.  The tensor cores keep the
    top 19 bits of each operand (truncation: the products of a Triton tl.dot
    at input_precision="tf32"); round_inputs rounds both operands to the
    nearest TF32 values first (the products of cuBLAS's TF32 GEMMs)."""
    _lib.require_cuda(A, Bt)
    if A.dtype != torch.float32 or Bt.dtype != torch.float32:
        raise TypeError("matmul_tf32 takes float32 operands")
    if A.dim() != 2 or Bt.dim() != 2 or A.shape[1] != Bt.shape[1]:
        raise ValueError(f"A [M, K] and Bt [N, K] expected, got {tuple(A.shape)} and {tuple(Bt.shape)}")
    M, K = A.shape
    N = Bt.shape[0]

    def _rows(X):  # row-major with a 16-byte row stride and base
        if X.stride(1) != 1 or X.stride(0) % 4 or X.data_ptr() % 16:
            Y = torch.zeros(X.shape[0], -(-X.shape[1] // 4) * 4, dtype=X.dtype, device=X.device)
            Y[:, :X.shape[1]] = X
            return Y
        return X

    A, Bt = _rows(A), _rows(Bt)
    if round_inputs:
        A, Bt = round_tf32(A), round_tf32(Bt)
    C = torch.empty(M, N, dtype=torch.float32, device=A.device)
    call("sffn_gemm_tf32", ptr(A), A.stride(0), ptr(Bt), Bt.stride(0), ptr(C), C.stride(0), M, N, K,
         int(bool(relu)), ptr(_lib.status_word(A.device)), stream_ptr(A.device))
    return C


def mm_f32acc(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, accumulate: bool):
    """C (float32 [M, N], row-major) = A @ B, or += with accumulate, bf16
    operands, on the tcgen05 kernel (the epilogue adds into C)."""
    _lib.require_cuda(A, B, C)
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16 or C.dtype != torch.float32:
        raise TypeError("mm_f32acc takes bfloat16 operands and a float32 C")
    M, K = A.shape
    K2, N = B.shape
    if K != K2 or tuple(C.shape) != (M, N) or C.stride(1) != 1:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)} -> {tuple(C.shape)}")
    lda, a_mn = _operand(A, 0)
    ldb, b_mn = _operand(B, 1)
    call("sffn_gemm_bf16_f32acc", ptr(A), lda, a_mn, ptr(B), ldb, b_mn, ptr(C), C.stride(0), M, N, K,
         int(bool(accumulate)), ptr(_lib.status_word(A.device)), stream_ptr(A.device))
    return C


def mm_t(A: torch.Tensor, B: torch.Tensor, kb_list=None, kb_count=None):
    """(A @ B)^T [N, M] (bf16) on the tcgen05 kernel, the product stored
    transposed by its epilogue; kb_list / kb_count as in mm (per 256 rows of A)."""
    _lib.require_cuda(A, B)
    if A.dtype != torch.bfloat16 or B.dtype != torch.bfloat16:
        raise TypeError("mm_t takes bfloat16 operands")
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    lda, a_mn = _operand(A, 0)
    ldb, b_mn = _operand(B, 1)
    out = torch.empty(N, M, dtype=torch.bfloat16, device=A.device)
    stride = kb_list.shape[1] if kb_list is not None else 0
    call("sffn_gemm_bf16_ct", ptr(A), lda, a_mn, ptr(B), ldb, b_mn, ptr(out), out.stride(0), M, N, K,
         ptr(kb_list), ptr(kb_count), stride, ptr(_lib.status_word(A.device)), stream_ptr(A.device))
    return out


def live_kblocks_t(bitmask: torch.Tensor, M: int, N: int):
    """(kb_list [ceil(N/256), ceil(M/64)] int32, kb_count [ceil(N/256)] int32):
    for each 256-column tile of a tiled 128x128 bitmask of [M, N], the 64-row
    blocks holding any set bit (the token-skip lists of dpre^T @ x and
    a^T @ dout)."""
    gp, nkb = -(-N // 256), -(-M // 64)
    kb_list = torch.empty(gp, nkb, dtype=torch.int32, device=bitmask.device)
    kb_count = torch.empty(gp, dtype=torch.int32, device=bitmask.device)
    call("sffn_live_kblocks_t", ptr(bitmask), M, N, ptr(kb_list), ptr(kb_count), stream_ptr(bitmask.device))
    return kb_list, kb_count


def full_kblocks(M, N, device):
    """The (kb_list, kb_count) of live_kblocks for a matrix with every 64-wide
    block of every 256-row tile live: kb_count[m] = ceil(N/64), the list left
    unwritten (the GEMM reads no list whose count is full)."""
    gm, nkb = -(-M // 256), -(-N // 64)
    return (torch.empty(gm, nkb, dtype=torch.int32, device=device),
            torch.full((gm,), nkb, dtype=torch.int32, device=device))


def live_kblocks(bitmask: torch.Tensor, M: int, N: int):
    """(kb_list [ceil(M/256), ceil(N/64)] int32, kb_count [ceil(M/256)] int32):
    per 256-row tile, the 64-column blocks holding any set bit of a tiled
    128x128 bitmask (the K-skip lists of mm)."""
    gm, nkb = -(-M // 256), -(-N // 64)
    kb_list = torch.empty(gm, nkb, dtype=torch.int32, device=bitmask.device)
    kb_count = torch.empty(gm, dtype=torch.int32, device=bitmask.device)
    call("sffn_live_kblocks", ptr(bitmask), M, N, ptr(kb_list), ptr(kb_count),
         stream_ptr(bitmask.device))
    return kb_list, kb_count


def ffn_up(x, W1, b1, act, vals, offset, sp24=False, write_act=True, colmask=None):
    """Fused x @ W1.T (+ b1) -> act(z) dense plus the tiled 128x128 sparse z.

    Returns (act [T, F], bitmask, prefix, vals_offset, row_offsets); act is
    dense, or with sp24=True an ``sp24.Sp24`` (2:4 form, K = F) written by the
    same epilogue (T, F multiples of 128), or None with write_act=False.
    colmask (optional int32 [tiles * 4]) receives each format tile's live
    columns (the OR of its rows' mask words).  vals is the arena, or a
    callable alloc(n) -> vals: then the cursor offset (zero on entry) is read
    back once the tiles are counted (one device sync) and the values are
    copied into alloc(nnz), a tensor of exactly nnz elements."""
    T, D = x.shape
    F = W1.shape[0]
    dev = x.device
    gm, gn = -(-T // 128), -(-F // 128)
    nt = gm * gn
    bitmask = torch.empty(nt * 2048, dtype=torch.uint8, device=dev)
    counts = torch.empty(nt * 4, dtype=torch.int32, device=dev)
    # The epilogue writes each group of 32 rows' z values packed in arena order
    # into its quarter of the tile's slot (and the rows' offsets in that run
    # into row_offsets); one contiguous copy per group then fills the arena.
    slots = torch.empty(nt * 128 * 128, dtype=torch.bfloat16, device=dev)
    prefix = torch.empty(nt + 1, dtype=torch.int32, device=dev)
    vals_offset = torch.empty(1, dtype=torch.int32, device=dev)
    row_offsets = torch.empty(nt * 128, dtype=torch.int32, device=dev)
    status = ptr(_lib.status_word(dev))
    st = stream_ptr(dev)
    if sp24:
        from .sp24 import Sp24
        act_out = Sp24.empty(T, F, dev)
        d = act_out.desc()
        call("sffn_ffn_up_sp24", ptr(x), x.stride(0), ptr(W1), W1.stride(0), ptr(b1), T, D, F, act,
             ctypes.addressof(d), ptr(bitmask), ptr(counts), ptr(slots), ptr(row_offsets), status, st)
    else:
        act_out = torch.empty(T, F, dtype=torch.bfloat16, device=dev) if write_act else None
        call("sffn_ffn_up", ptr(x), x.stride(0), ptr(W1), W1.stride(0), ptr(b1), T, D, F, act,
             ptr(act_out), F, ptr(bitmask), ptr(counts), ptr(slots), ptr(row_offsets), status, st)
    call("sffn_tile_scan_counts", ptr(counts), 4, nt, ptr(prefix), ptr(offset), ptr(vals_offset),
         status, st)
    if callable(vals):
        vals = vals(int(offset.item()))
    call("sffn_tile_copy_slots", ptr(slots), ptr(counts), ptr(prefix), ptr(vals_offset), nt, ptr(vals),
         vals.numel(), ptr(row_offsets), ptr(bitmask), ptr(colmask), status, st)
    return act_out, bitmask, prefix, vals_offset, row_offsets


def tile_row_offsets(z_sparse):
    """Per-row value offsets of a 128x128-tile BitsparseTensor (int32 [tiles*128])."""
    nt = z_sparse.grid_m * z_sparse.grid_n
    ro = torch.empty(nt * 128, dtype=torch.int32, device=z_sparse.bitmask.device)
    call("sffn_tile_row_offsets", ptr(z_sparse.bitmask), ptr(z_sparse.prefix), nt, ptr(ro), None,
         stream_ptr(ro.device))
    return ro


def tile_colmask(z_sparse):
    """Live columns of each format tile of a 128x128-tile BitsparseTensor: the
    OR of the tile's 128 rows of mask words (int32 [tiles * 4])."""
    nt = z_sparse.grid_m * z_sparse.grid_n
    cm = torch.empty(nt * 4, dtype=torch.int32, device=z_sparse.bitmask.device)
    call("sffn_tile_row_offsets", ptr(z_sparse.bitmask), ptr(z_sparse.prefix), nt, None, ptr(cm),
         stream_ptr(cm.device))
    return cm


# ---------------------------------------------------------------------------
# Compacted-K down-projection (and dX): the contraction over F runs over each
# 128-row tile's live columns only.
# ---------------------------------------------------------------------------
def ck_supported(T, D, F):
    """Shapes the compacted-K kernels take."""
    return T % 128 == 0 and F % 128 == 0 and D % 256 == 0 and 0 < F <= 65536 and T * F < 2 ** 31


def ck_lists(colmask, T, F, counts_only=False):
    """(idx [T/128, F] int32, kcount [T/128] int32, colpref [T/128, ceil(F/128)]
    int32): per 128-row tile the ascending live columns (padded to a multiple
    of 64 with a column that is zero in the whole tile), their count, and where
    each 128-column block's live columns start.  counts_only: kcount alone."""
    dev = colmask.device
    gm, gn = T // 128, -(-F // 128)
    kcount = torch.empty(gm, dtype=torch.int32, device=dev)
    if counts_only:
        call("sffn_ck_lists", ptr(colmask), T, F, None, F, ptr(kcount), None, stream_ptr(dev))
        return None, kcount, None
    idx = torch.empty(gm, F, dtype=torch.int32, device=dev)
    colpref = torch.empty(gm, gn, dtype=torch.int32, device=dev)
    call("sffn_ck_lists", ptr(colmask), T, F, ptr(idx), F, ptr(kcount), ptr(colpref), stream_ptr(dev))
    return idx, kcount, colpref


def ck_gather_packed(z_sparse, row_offsets, colmask, colpref, kcount, act):
    """The compacted activation [T, F] (columns past each tile's padded count
    unused): act(z) at the tile's live columns, built from the packed z."""
    T, F = z_sparse.shape
    dev = z_sparse.vals.device
    ac = torch.empty(T, F, dtype=torch.bfloat16, device=dev)
    call("sffn_ck_gather_packed", ptr(z_sparse.vals), z_sparse.vals.numel(), ptr(z_sparse.bitmask),
         ptr(z_sparse.prefix), ptr(row_offsets), ptr(z_sparse.vals_offset), ptr(colmask), ptr(colpref), ptr(kcount), T, F, act,
         ptr(ac), F, ptr(_lib.status_word(dev)), stream_ptr(dev))
    return ac


def ck_compact_rows_(x, idx, kcount):
    """In place: each row of x [T, F] (bf16, row-major) compacted to its tile's
    live columns (x's zeros must follow the activation's, as dpre's do)."""
    T, F = x.shape
    if x.stride(1) != 1 or x.dtype != torch.bfloat16:
        raise ValueError("ck_compact_rows_ takes a row-major bf16 matrix")
    call("sffn_ck_compact_rows", ptr(x), x.stride(0), T, F, ptr(idx), idx.stride(0), ptr(kcount),
         stream_ptr(x.device))
    return x


def ck_mm(ac, B_rows, idx, kcount, out=None):
    """C [T, N] = per 128-row tile tm, ac[rows, :Kp] @ B_rows[idx[tm, :Kp], :]
    (Kp = kcount[tm] rounded up to 64): ac the compacted activation, B_rows
    [F, N] row-major with rows = the contraction index, gathered by TMA."""
    _lib.require_cuda(ac, B_rows)
    T, F = ac.shape
    Fb, N = B_rows.shape
    if ac.stride(1) != 1 or B_rows.stride(1) != 1:
        raise ValueError("ck_mm takes row-major operands")
    if out is None:
        out = torch.empty(T, N, dtype=torch.bfloat16, device=ac.device)
    call("sffn_gemm_ck", ptr(ac), ac.stride(0), F, ptr(B_rows), B_rows.stride(0), Fb, ptr(idx), idx.stride(0),
         ptr(kcount), ptr(out), out.stride(0), T, N, ptr(_lib.status_word(ac.device)), stream_ptr(ac.device))
    return out


def ffn_dgrad(dout, W2, act, z_sparse, row_offsets=None, db1=None, sp24=False, want_act=True):
    """Fused dout @ W2 with the activation gradient; returns (dpre, act2)
    where act2 = z*z (ReLU^2) or z (ReLU), both dense [T, F] (act2 None with
    want_act=False).  z_sparse is a
    128x128-tile BitsparseTensor; row_offsets its per-row offsets (computed
    here if not given).  db1: optional zeroed float32 [F] that receives the
    column sums of dpre (the bias gradient).  With sp24=True the outputs are
    ``sp24.Sp24`` matrices instead: (dpre [T, F], dpre^T [F, T], act2^T
    [F, T]), written by the same epilogue (T, F multiples of 128)."""
    T, D = dout.shape
    F = W2.shape[1]
    dev = dout.device
    if z_sparse.BLOCK_M != 128 or z_sparse.BLOCK_N != 128:
        raise ValueError("the fused activation gradient reads 128x128 tiles")
    if row_offsets is None:
        row_offsets = tile_row_offsets(z_sparse)
    if sp24:
        from .sp24 import Sp24
        outs = (Sp24.empty(T, F, dev), Sp24.empty(F, T, dev), Sp24.empty(F, T, dev))
        ds = [o.desc() for o in outs]
        call("sffn_ffn_dgrad_sp24", ptr(dout), dout.stride(0), ptr(W2), W2.stride(0), T, D, F, act,
             ptr(z_sparse.vals), z_sparse.vals.numel(), ptr(z_sparse.bitmask), ptr(row_offsets),
             ptr(z_sparse.vals_offset), *(ctypes.addressof(d) for d in ds), ptr(db1),
             ptr(_lib.status_word(dev)), stream_ptr(dev))
        return outs
    dpre = torch.empty(T, F, dtype=torch.bfloat16, device=dev)
    act2 = torch.empty(T, F, dtype=torch.bfloat16, device=dev) if want_act else None
    call("sffn_ffn_dgrad", ptr(dout), dout.stride(0), ptr(W2), W2.stride(0), T, D, F, act,
         ptr(z_sparse.vals), z_sparse.vals.numel(), ptr(z_sparse.bitmask), ptr(row_offsets),
         ptr(z_sparse.vals_offset), ptr(dpre), ptr(act2), dpre.stride(0), ptr(db1),
         ptr(_lib.status_word(dev)), stream_ptr(dev))
    return dpre, act2
