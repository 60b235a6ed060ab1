"""The 128x128 (vals, meta) variant of the tiled format.

Mirrors old/full_matmul/sparse_pack.py:95-146 (dense_to_tilesparse(dense,
BLOCK_M=128, BLOCK_N=128) -> (vals, meta)), old/full_matmul/sparse_unpack.py:44-73
(bitsparse_unpack(vals, meta, shape) -> float32 dense; the same function as
old/matmul_bitsparse/sparse_unpack.py) and old/matmul_bitsparse/train.py:69-116
(sparse_relu_Ax(W1, x) -> (vals, meta), the product and its ReLU packed by
one kernel), and the two-layer pipeline's products on the packed activation:
old/full_matmul/train.py:21-76,140-184 (sp_relu_Ax, relu_spAx) and
old/sparse_matmul/train.py:56-76 (relu_sparse_Ax).  bitsparse_unpack shares
its name with the flat one, so these live in their own namespace.
"""
import torch

from . import _lib
from ._lib import call, dtype_code, ptr, stream_ptr
from .bitsparse import BitsparseTensor, tile_unpack

__all__ = ["dense_to_tilesparse", "bitsparse_unpack", "sparse_relu_Ax", "sp_relu_Ax", "relu_spAx",
           "relu_sparse_Ax"]


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


def sparse_relu_Ax(W1: torch.Tensor, x: torch.Tensor, BLOCK_M: int = 128, BLOCK_N: int = 128,
                   input_precision: str = "tf32", _round_tf32: bool = False):
    """relu(x @ W1.T) ([M, N], M = rows of x, N = rows of W1) in x's dtype,
    returned as (vals, meta) of the BLOCK_M x BLOCK_N tiled format
    (meta: bitmask, prefix, grid_m, grid_n, BLOCK_M, BLOCK_N, shape), as
    old/matmul_bitsparse/train.py:69-116.  bf16 with 128x128 tiles: one
    tcgen05 GEMM whose epilogue applies the ReLU and writes the bitmask, the
    counts and the values packed per 32 rows; one device sync for the total
    (the reference's .item(), train.py:96), then one copy per 32 rows into a
    vals of exactly nnz elements.  float32 with input_precision "tf32" (the
    reference's default, Triton's tl.dot input_precision): the tcgen05
    kind::tf32 GEMM with the ReLU in its epilogue, then the tiled pack (the
    operands truncated to TF32 as Triton's are; rounded to nearest first
    with _round_tf32, as cuBLAS's TF32 GEMMs do).
    float32 with "tf32x3" or "ieee", float16, other tile shapes: the product
    on this library's GEMM (float32 and float16 as the split-bf16 product,
    float32 accuracy up to terms of 2^-24), its ReLU, then the tiled pack."""
    from . import gemm as G
    _lib.require_cuda(W1, x)
    if x.dim() != 2 or W1.dim() != 2 or x.shape[1] != W1.shape[1]:
        raise ValueError(f"x [M, K] and W1 [N, K] expected, got {tuple(x.shape)} and {tuple(W1.shape)}")
    if x.dtype != W1.dtype:
        raise TypeError("x and W1 must share a dtype")
    if input_precision not in ("tf32", "tf32x3", "ieee"):
        raise ValueError(f"input_precision must be 'tf32', 'tf32x3' or 'ieee', got {input_precision!r}")
    M, K = x.shape
    N = W1.shape[0]
    dev = x.device
    if x.dtype == torch.float32 and input_precision == "tf32":
        return dense_to_tilesparse(G.matmul_tf32(x, W1, relu=True, round_inputs=_round_tf32), BLOCK_M, BLOCK_N)
    fused = (x.dtype == torch.bfloat16 and BLOCK_M == 128 and BLOCK_N == 128 and K % 8 == 0 and N % 8 == 0
             and M * N < 2 ** 31)
    if not fused:
        z = torch.relu(G.matmul(x.contiguous(), W1.contiguous().T)).to(x.dtype)
        return dense_to_tilesparse(z, BLOCK_M, BLOCK_N)
    x, W1 = x.contiguous(), W1.contiguous()
    gm, gn = -(-M // 128), -(-N // 128)
    nt = gm * gn
    bitmask = torch.empty(nt * 2048, dtype=torch.uint8, device=dev)
    counts = torch.empty(nt * 4, dtype=torch.int32, device=dev)
    slots = torch.empty(nt * 128 * 128, dtype=torch.bfloat16, device=dev)
    row_offsets = torch.empty(nt * 128, dtype=torch.int32, device=dev)
    prefix = torch.empty(nt + 1, dtype=torch.int32, device=dev)
    offset = torch.zeros(1, dtype=torch.int32, device=dev)
    vals_offset = torch.empty(1, dtype=torch.int32, device=dev)
    status = ptr(_lib.status_word(dev))
    st = stream_ptr(dev)
    call("sffn_ffn_up", ptr(x), K, ptr(W1), K, None, M, K, N, G.ACT_RELU, None, N, ptr(bitmask), ptr(counts),
         ptr(slots), ptr(row_offsets), status, st)
    call("sffn_tile_scan_counts", ptr(counts), 4, nt, ptr(prefix), ptr(offset), ptr(vals_offset), status, st)
    nnz = int(offset.item())
    vals = torch.empty(nnz, dtype=x.dtype, device=dev)
    if nnz:
        call("sffn_tile_copy_slots", ptr(slots), ptr(counts), ptr(prefix), ptr(vals_offset), nt, ptr(vals), nnz,
             ptr(row_offsets), ptr(bitmask), None, status, st)
    meta = {"bitmask": bitmask, "prefix": prefix, "grid_m": gm, "grid_n": gn,
            "BLOCK_M": 128, "BLOCK_N": 128, "shape": (M, N)}
    return vals, meta


def _as_bitsparse(vals, meta, shape=None):
    """The (vals, meta) pair as a BitsparseTensor over the whole of vals."""
    zero = torch.zeros(1, dtype=torch.int32, device=vals.device)
    shape = tuple(meta["shape"] if shape is None else shape)
    return BitsparseTensor(vals.contiguous(), meta["bitmask"], meta["prefix"], zero, meta["grid_m"],
                           meta["grid_n"], meta["BLOCK_M"], meta["BLOCK_N"], shape)


def sp_relu_Ax(W1: torch.Tensor, x: torch.Tensor, BLOCK_M: int = 128, BLOCK_N: int = 128):
    """Layer 1 of old/full_matmul/train.py:21-76: relu(x @ W1.T) packed as
    (vals, meta).  The reference's product is F.linear, whose float32
    precision follows torch's global setting: TF32 when
    torch.backends.cuda.matmul.allow_tf32 (set_float32_matmul_precision
    "high"), float32 otherwise; here the kind::tf32 GEMM on operands rounded
    to the nearest TF32 values (cuBLAS's TF32 products) or the split-bf16
    product accordingly (sparse_relu_Ax does the rest)."""
    tf32 = bool(torch.backends.cuda.matmul.allow_tf32)
    return sparse_relu_Ax(W1, x, BLOCK_M, BLOCK_N, input_precision="tf32" if tf32 else "ieee", _round_tf32=tf32)


def relu_spAx(vals: torch.Tensor, meta: dict, W2: torch.Tensor, row_batch: int = 8192) -> torch.Tensor:
    """Layer 2 of old/full_matmul/train.py:140-184: relu(A @ W2.T) [M, N] in
    W2's dtype, A [M, K] = the unpacked (vals, meta) (meta["shape"]), W2
    [N, K]; the rows unpacked in batches of row_batch (the reference: 2048)
    to bound the dense temporary.  bf16: the tcgen05 GEMM with the ReLU in
    its epilogue, 64-wide K blocks that are zero in a 256-row tile skipped
    (128x128 tiles); float32: when torch allows TF32 for float32 matmuls (the
    reference's F.linear runs cuBLAS's TF32 GEMM then) the kind::tf32 GEMM on
    operands rounded to the nearest TF32 values (the unpack rounds A as it
    writes it), else the split-bf16 product; float16: the split-bf16 product
    rounded to float16."""
    from . import gemm as G
    _lib.require_cuda(vals, W2)
    M, K = (int(d) for d in meta["shape"])
    if W2.dim() != 2 or W2.shape[1] != K:
        raise ValueError(f"W2 must be [N, {K}], got {tuple(W2.shape)}")
    if vals.dtype != W2.dtype:
        raise TypeError("vals and W2 must share a dtype")
    z = _as_bitsparse(vals, meta, (M, K))
    # batches start on 256-row boundaries: whole K-block list rows, and whole
    # tile rows for every tile height the format has (32, 64, 128)
    row_batch = max(256, (row_batch // 256) * 256)
    lists = None
    if W2.dtype == torch.bfloat16 and z.BLOCK_M == 128 and z.BLOCK_N == 128:
        lists = G.live_kblocks(z.bitmask, M, K)
    tf32 = W2.dtype == torch.float32 and torch.backends.cuda.matmul.allow_tf32
    W2r = G.round_tf32(W2) if tf32 else None

    def batch(m0, m1):
        a = tile_unpack(z, m0, m1, round_tf32=tf32)
        if W2.dtype == torch.bfloat16:
            kl = kc = None
            if lists is not None:
                kl, kc = lists[0][m0 // 256:], lists[1][m0 // 256:]
            return G.mm_relu(a, W2.T, kb_list=kl, kb_count=kc)
        if tf32:
            return G.matmul_tf32(a, W2r, relu=True)
        return G.matmul(a, W2.T, relu=True)

    if M <= row_batch:
        return batch(0, M)
    out = torch.empty(M, W2.shape[0], dtype=W2.dtype, device=W2.device)
    for m0 in range(0, M, row_batch):
        m1 = min(m0 + row_batch, M)
        out[m0:m1] = batch(m0, m1)
    return out


def relu_sparse_Ax(vals: torch.Tensor, meta: dict, x: torch.Tensor, *, dtype=torch.bfloat16,
                   tf32: bool = False) -> torch.Tensor:
    """old/sparse_matmul/train.py:56-76: relu(A @ x) in float32 [M, N], A
    [M, K] the unpacked (vals, meta) (meta["shape"]) and x [K, N], both taken
    in `dtype` for the product (fp32 accumulation).  bf16: the tcgen05 GEMM
    with the ReLU and a float32 store in its epilogue (the values rounded to
    bf16 before the unpack, which equals rounding the unpacked tensor);
    float16: the split-bf16 product of the float16 operands (exact in
    float32 terms); float32: the kind::tf32 GEMM with tf32=True, else the
    split-bf16 product (float32 accuracy)."""
    from . import gemm as G
    _lib.require_cuda(vals, x)
    M, K = (int(d) for d in meta["shape"])
    if x.dim() != 2 or x.shape[0] != K:
        raise ValueError(f"x must be [{K}, N], got {tuple(x.shape)}")
    if dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError(f"dtype must be bfloat16, float16 or float32, got {dtype}")
    z = _as_bitsparse(vals.to(dtype), meta, (M, K))
    a = tile_unpack(z)
    xd = x.to(dtype)
    if dtype == torch.bfloat16:
        lists = G.live_kblocks(z.bitmask, M, K) if z.BLOCK_M == 128 and z.BLOCK_N == 128 else (None, None)
        return G.mm_relu(a, xd, out_dtype=torch.float32, kb_list=lists[0], kb_count=lists[1])
    if dtype == torch.float16:
        return G.matmul(a.float(), xd.float(), relu=True)
    if tf32:
        return G.matmul_tf32(a, xd.T.contiguous(), relu=True)
    return G.matmul(a, xd, relu=True)
