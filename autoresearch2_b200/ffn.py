"""Sparse FFN autograd functions with the reference's forward/backward contract.

FFNSparse   -- out = relu(x @ W1.T) @ W2.T      (old/lib_sparse/sparse.py:56-109)
FFNSpRelu2  -- out = relu(x @ W1.T)^2 @ W2.T    (old/lib_sparse/sparse.py:112-151)

Contract kept from the reference: forward(ctx, x, W1, W2, sparse_data) saves
(x, W1, W2) with save_for_backward and keeps z = relu(x @ W1.T) only as a
tiled BitsparseTensor on ctx.z_sparse (the activation-memory saving);
backward clears it and returns one gradient per input (None for the arena).
Weights use nn.Linear layout: W1 [F, D], W2 [D, F]; x [T, D].

bf16 inputs run the fused tcgen05 path: the up-projection GEMM's epilogue
applies bias + ReLU/ReLU^2 and emits the bitmask, counts and compacted z (a
128x128-tile BitsparseTensor); the down-projection skips 64-wide K blocks
that are zero in a whole 128-row tile; the backward's dout @ W2 epilogue
applies the mask / 2z gradient from the packed z and emits the activation
for dW2, so no dense z is kept between forward and backward.  float32 and
float16 inputs run their products as split-bf16 products on the same tcgen05
GEMM (three bf16 pieces per operand, fp32 accumulation: float32 accuracy)
with this library's pack/mask kernels (64x64 tiles, as in the reference).  Forward and backward each run as one
torch.library op (sparseffn::ffn_fwd, sparseffn::ffn_bwd, registered in
library.py), so torch.compile traces these Functions without a graph break.

Differences (documented, not inherited defects): FFNSpRelu2 accepts the vals
arena (the reference's forward omits it and raises TypeError,
sparse.py:120), both accept an optional up-projection bias b1 [F] as a
trailing argument (the reference has none), and the backward leaves the
stored z values unchanged (the reference squares them in place,
sparse.py:136-144; here z^2 is formed where it is read).
"""
import torch
import torch.nn.functional as F
from torch.autograd import Function

from . import bitsparse as bs
from . import gemm as G
from . import sp24
from .parallel import submit_grad

__all__ = ["FFNSparse", "FFNSpRelu2", "set_sparse_mma", "sparse_mma", "set_compact_k", "compact_k",
           "last_path", "down_proj", "packed_backward"]

# The four products with a sparse operand -- forward a @ W2^T, backward
# dpre @ W1, dpre^T @ x and a^T @ dout -- can run on the 2:4 sparse tensor
# cores (sp24): the 2:4 part of the activation at twice the dense rate plus
# its overflow on the CUDA cores.  "off": dense tcgen05 GEMMs; "on": sp24
# whenever the shapes allow it (T and F multiples of 128, up to 65536, D a
# multiple of 32); "auto" (default): sp24 when the same layer's previous step
# had at least AUTO_MIN_SPARSITY zeros in its activation.  Measured on a B200
# at T=16384, D=4096, F=14336 (ReLU^2, step ms, dense / sp24, medians of four
# alternating samples in one process): 85% zeros 8.35 / 9.74; 88% 8.31 / 9.09;
# 90% 8.18 / 8.34; 92% 8.44 / 8.10; and 95% 7.97 / 7.19 -- the overflow of the
# 2:4 split shrinks with the density, the saving of the sparse products does
# not.
_SPARSE_MMA = "auto"
AUTO_MIN_SPARSITY = 0.915
# The down-projection and dX contract over F.  With the compacted-K path
# ("ck") each 128-row tile of tokens contracts over its live columns only --
# the columns of z holding a non-zero in any of the tile's rows -- with the
# activation compacted from the packed z and the rows of W2^T (W1 for dX)
# gathered by TMA.  Its GEMM runs on one SM per 128-row tile, which needs
# 1.5x the operand bytes per flop of the two-SM kernel of the dense path and
# measured at half its rate at the same K (4.81 vs 2.35 ms at 8192 x 8192 x
# 28672, 2.29 vs 1.32 ms at 16384 x 4096 x 14336 on a B200).  The dense path
# skips 64-wide K blocks that are zero across a 256-row tile.  So the
# compacted path pays only where its live fraction is below about half the
# dense path's: on the clustered workload (live 0.50 per 128 rows, 0.74 per
# 256 rows) it does not, at 99% random zeros (0.72 against 1.0) it does not,
# at 99.9% (0.12 against 1.0) it does.  "off" / "on" / "auto" (default): "ck"
# when the same layer's previous step had at most CK_AUTO_MAX_LIVE of its
# (128-row tile, column) pairs live.
_COMPACT_K = "auto"
CK_AUTO_MAX_LIVE = 0.35
# The weight gradients skip 64-token blocks that are zero across 256 columns
# of the activation (dW2 then through a transposed-store epilogue, which
# costs ~4% when nothing is skipped): taken when the layer's previous step
# had at most this fraction of its (128-row tile, column) pairs live.
TOKEN_SKIP_MAX_LIVE = 0.9
# The forward builds no K-block lists when at least this fraction of the
# layer's (128-row tile, column) pairs was live in its previous step.
FULL_KBLOCKS_MIN_LIVE = 0.99
# per layer (keyed by W1's storage and the shapes): pinned [activation count,
# live (tile, column) count], its copy's event, the element count, the last
# sparsity and live fraction read
_observed = {}
_last_path = None


def set_sparse_mma(mode: str):
    """Choose the products' path for the fused bf16 FFN: "off", "on" or "auto".
    Also forgets the sparsities "auto" has observed (they are keyed by weight
    storage and shapes, which a later layer may reuse)."""
    global _SPARSE_MMA
    if mode not in ("off", "on", "auto"):
        raise ValueError("sparse MMA mode is 'off', 'on' or 'auto'")
    _SPARSE_MMA = mode
    _observed.clear()


def sparse_mma() -> str:
    return _SPARSE_MMA


def set_compact_k(mode: str):
    """Choose the contraction of the bf16 down-projection and dX: "off" (dense
    K, 64-wide zero blocks skipped), "on" (compacted live columns of each
    128-row tile) or "auto".  Also forgets the observed statistics."""
    global _COMPACT_K
    if mode not in ("off", "on", "auto"):
        raise ValueError("compact-K mode is 'off', 'on' or 'auto'")
    _COMPACT_K = mode
    _observed.clear()


def compact_k() -> str:
    return _COMPACT_K


# The bf16 backward's activation a (z*z or z) for dW2: "fused" -- written by
# the activation-gradient epilogue beside dpre (two dense [T, F] transients
# live together); "lean" -- rebuilt from the packed z by an unpack first, dW2
# computed and a freed before the activation gradient writes dpre (at most one
# dense [T, F] transient at a time).
_BACKWARD = "fused"


def set_backward(mode: str):
    """Choose how the fused bf16 backward gets the activation for dW2:
    "fused" (beside dpre, in the activation-gradient epilogue) or "lean"
    (unpacked from z first and freed before dpre is written: half the dense
    transients)."""
    global _BACKWARD
    if mode not in ("fused", "lean"):
        raise ValueError("backward mode is 'fused' or 'lean'")
    _BACKWARD = mode


def backward_mode() -> str:
    return _BACKWARD


def last_path():
    """The products' path of the last fused forward: "sp24", "ck" (compacted
    K), "dense" or None."""
    return _last_path


def _stats(T, D, Fd, W1):
    """The layer's last observed (sparsity, live fraction), each None if not
    seen yet; reads a landed copy without waiting."""
    ent = _observed.get((W1.data_ptr(), T, D, Fd))
    if ent is None:
        return None, None
    if ent["event"] is not None and ent["event"].query():  # the counts have landed: no wait
        c = ent["counts"].tolist()
        ent["sparsity"] = 1.0 - c[0] / ent["elems"]
        ent["live"] = c[1] / ent["elems"] if c[1] >= 0 else None
        ent["event"] = None
    return ent["sparsity"], ent["live"]


def _sp24_ok(T, D, Fd, W1):
    if _SPARSE_MMA == "off" or not (T % 128 == 0 and Fd % 128 == 0 and D % 32 == 0 and T <= 65536
                                    and Fd <= 65536):
        return False
    if _SPARSE_MMA == "on":
        return True
    s, _ = _stats(T, D, Fd, W1)
    return s is not None and s >= AUTO_MIN_SPARSITY


def _ck_ok(T, D, Fd, W1):
    if _COMPACT_K == "off" or not G.ck_supported(T, D, Fd):
        return False
    if _COMPACT_K == "on":
        return True
    _, live = _stats(T, D, Fd, W1)
    return live is not None and live <= CK_AUTO_MAX_LIVE


def _token_skip(T, D, Fd, key):
    _, live = _stats(T, D, Fd, key)
    return live is not None and live <= TOKEN_SKIP_MAX_LIVE


def _observe(W1, prefix, kcount, T, D, Fd):
    """Copy this step's activation count (prefix[-1]) and live (tile, column)
    count (the sum of kcount, or -1) to pinned host memory without waiting;
    a later step reads them once the copy's event completed (the auto modes
    and the weight gradients' token skipping decide from them)."""
    key = (W1.data_ptr(), T, D, Fd)
    ent = _observed.get(key)
    if ent is None:
        ent = _observed[key] = {
            "counts": torch.empty(2, dtype=torch.int64, pin_memory=True), "event": None,
            "elems": 1, "sparsity": None, "live": None}
    if ent["event"] is not None:  # the previous copy is still unread
        return
    live = kcount.sum(dtype=torch.int64).view(1) * 128 if kcount is not None else prefix.new_full((1,), -1,
                                                                                                 dtype=torch.int64)
    ent["counts"].copy_(torch.cat([prefix[-1:].to(torch.int64), live]), non_blocking=True)
    ent["elems"] = T * Fd
    ent["event"] = torch.cuda.Event()
    ent["event"].record()


def _fused_ok(x, W1, W2, b1, vals):
    """bf16 tensors laid out for the tcgen05 path (16-byte aligned rows)."""
    ts = [x, W1, W2, vals] + ([b1] if b1 is not None else [])
    if not all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts):
        return False
    if not (x.is_contiguous() and W1.is_contiguous() and W2.is_contiguous()):
        return False
    if b1 is not None and not b1.is_contiguous():
        return False
    D, Fd = x.shape[1], W1.shape[0]
    return D % 8 == 0 and Fd % 8 == 0 and x.shape[0] * Fd < 2 ** 31


def _fused_forward(x, W1, W2, vals, offset, b1, act):
    """bf16 forward on the tcgen05 kernels.  Returns (out, bitmask, prefix,
    vals_offset, row_offsets, kb_list, kb_count): the tiled 128x128 z, its
    per-row value offsets and the live 64-wide K blocks of each 256-row tile."""
    T, D = x.shape
    Fd = W1.shape[0]
    global _last_path
    use_sp24 = _sp24_ok(T, D, Fd, W1)
    use_ck = not use_sp24 and _ck_ok(T, D, Fd, W1)
    _last_path = "sp24" if use_sp24 else "ck" if use_ck else "dense"
    want_live = use_ck or G.ck_supported(T, D, Fd)
    colmask = torch.empty(-(-T // 128) * -(-Fd // 128) * 4, dtype=torch.int32, device=x.device) \
        if want_live else None
    # with sp24 the up-projection epilogue writes a in the 2:4 form directly;
    # with ck it writes no dense activation at all.  (Running the arena fill
    # on a second stream beside the down-projection measured no faster.)
    a, bitmask, prefix, voff, row_offsets = G.ffn_up(x, W1, b1, act, vals, offset, sp24=use_sp24,
                                                     write_act=not use_ck, colmask=colmask)
    if callable(vals):  # exact-size values: the allocator kept the tensor it made
        vals = vals.vals
    if use_ck:
        idx, kcount, colpref = G.ck_lists(colmask, T, Fd)
    elif want_live:
        _, kcount, _ = G.ck_lists(colmask, T, Fd, counts_only=True)
    else:
        kcount = None
    _observe(W1, prefix, kcount, T, D, Fd)
    # the K-block lists also serve dX when the backward takes the dense path;
    # when the layer's last observed step had nearly every (tile, column)
    # pair live, a whole 64-column block of 256 rows is dead only by freak
    # chance: the counts alone say "all live" (the GEMM then reads no list;
    # a block it could have skipped is computed, which changes nothing)
    _, live = _stats(T, D, Fd, W1)
    if live is not None and live >= FULL_KBLOCKS_MIN_LIVE and not use_ck:
        kb_list, kb_count = G.full_kblocks(T, Fd, x.device)
    else:
        kb_list, kb_count = G.live_kblocks(bitmask, T, Fd)
    if use_sp24:
        # 2:4 part on the sparse tensor cores, overflow rows k of W2^T
        out = sp24.mm(a, W2.T, bt=sp24.transpose(W2))
    elif use_ck:
        # the activation compacted to each tile's live columns from the packed
        # z, times the rows of W2^T gathered at the same columns
        zs = bs.BitsparseTensor(vals, bitmask, prefix, voff, T // 128, Fd // 128, 128, 128, (T, Fd))
        ac = G.ck_gather_packed(zs, row_offsets, colmask, colpref, kcount, act)
        out = G.ck_mm(ac, sp24.transpose(W2), idx, kcount)
        del ac
    else:
        out = G.mm(a, W2.T, kb_list=kb_list, kb_count=kb_count)
    del a
    return out, bitmask, prefix, voff, row_offsets, kb_list, kb_count


def _fused_backward(grad_output, x, W1, W2, z_sparse, row_offsets, kb_list, kb_count, has_bias, act,
                    stats_key=None):
    """bf16 backward -> (grad_x, grad_W1, grad_W2, grad_b1 or None).  The
    products' path is chosen again here, by the same rule as the forward's."""
    T, D = x.shape
    Fd = W1.shape[0]
    grad_output = grad_output.contiguous()
    # the bias gradient (column sums of dpre) is summed in the same kernel, in fp32
    db1 = torch.zeros(Fd, dtype=torch.float32, device=x.device) if has_bias else None
    if _sp24_ok(T, D, Fd, W1):
        # the epilogue writes dpre, dpre^T and a^T in the 2:4 form (the
        # transposed ones compressed along the token dimension)
        dpre, dpre_t, a_t = G.ffn_dgrad(grad_output, W2, act, z_sparse, row_offsets, db1=db1, sp24=True)
        del row_offsets
        grad_b1 = submit_grad(db1.to(x.dtype)) if has_bias else None
        # dW2 = (a^T @ dout)^T, stored transposed by the kernel: [D, F] row-major
        grad_W2 = submit_grad(sp24.mm(a_t, grad_output, trans_out=True))
        del a_t
        # dW1 before dX: under data parallelism its all-reduce then overlaps dX
        grad_W1 = submit_grad(sp24.mm(dpre_t, x))
        grad_x = sp24.mm(dpre, W1)
        return grad_x, grad_W1, grad_W2, grad_b1
    use_ck = _ck_ok(T, D, Fd, W1 if stats_key is None else stats_key)
    lean = _BACKWARD == "lean"
    if lean:
        # a rebuilt from the packed z (squared in bf16 for ReLU^2, the forward's rounding)
        a = z_sparse.to_dense(square=act == G.ACT_RELU2)
    else:
        dpre, a = G.ffn_dgrad(grad_output, W2, act, z_sparse, row_offsets, db1=db1)
    # the weight gradients contract over tokens: per 256 columns of the
    # activation, 64-token blocks that are zero there are skipped (dW2 as
    # (a^T @ dout)^T, so that the lists index its M tiles), when the layer's
    # activation leaves enough such blocks
    if _token_skip(T, D, Fd, W1 if stats_key is None else stats_key):
        tl, tc = G.live_kblocks_t(z_sparse.bitmask, T, Fd)
        grad_W2 = submit_grad(G.mm_t(a.T, grad_output, kb_list=tl, kb_count=tc))  # reduced while dW1/dX run
    else:
        tl = tc = None
        grad_W2 = submit_grad(G.mm(grad_output.T, a))
    del a
    if lean:
        dpre, _ = G.ffn_dgrad(grad_output, W2, act, z_sparse, row_offsets, db1=db1, want_act=False)
    del row_offsets
    grad_b1 = submit_grad(db1.to(dpre.dtype)) if has_bias else None
    # dW1 before dX: under data parallelism its all-reduce then overlaps dX, and
    # no weight-gradient reduction is left without compute to hide behind
    grad_W1 = submit_grad(G.mm(dpre.T, x, kb_list=tl, kb_count=tc))
    if use_ck:
        # dpre is zero wherever z is: compact it in place to the live columns
        # and gather the matching rows of W1
        idx, kcount, _ = G.ck_lists(G.tile_colmask(z_sparse), T, Fd)
        grad_x = G.ck_mm(G.ck_compact_rows_(dpre, idx, kcount), W1, idx, kcount)
    else:
        grad_x = G.mm(dpre, W1, kb_list=kb_list, kb_count=kb_count)
    return grad_x, grad_W1, grad_W2, grad_b1


def down_proj(z_sparse, W2, act=G.ACT_RELU2):
    """The bitmask-sparse down-projection from a packed activation:
    out [T, D] = act(z) @ W2^T, act(z) = z*z rounded to bf16 (ReLU^2) or z
    (ReLU), for z a bf16 128x128-tile BitsparseTensor [T, F] -- the forward
    product of FFNSpRelu2 / FFNSparse (old/lib_sparse/sparse.py:75,118) and
    the contraction spAx computes by unpacking (sparse.py:305-351), here
    without a dense z: on the compacted-K path (set_compact_k) each 128-row
    tile contracts over its live columns, otherwise the unpacked activation
    runs through the dense tcgen05 GEMM with zero 64-wide blocks skipped."""
    T, Fd = z_sparse.shape
    D = W2.shape[0]
    if z_sparse.BLOCK_M != 128 or z_sparse.BLOCK_N != 128 or W2.dtype != torch.bfloat16:
        raise ValueError("down_proj takes a bf16 128x128-tile activation and bf16 weights")
    global _last_path
    use_ck = _ck_ok(T, D, Fd, W2)
    if use_ck or G.ck_supported(T, D, Fd):
        # statistics for the auto rule are kept under W2 here
        colmask = G.tile_colmask(z_sparse)
        idx, kcount, colpref = G.ck_lists(colmask, T, Fd, counts_only=not use_ck)
        _observe(W2, z_sparse.prefix, kcount, T, D, Fd)
    if use_ck:
        _last_path = "ck"
        ac = G.ck_gather_packed(z_sparse, G.tile_row_offsets(z_sparse), colmask, colpref, kcount, act)
        return G.ck_mm(ac, sp24.transpose(W2), idx, kcount)
    _last_path = "dense"
    a = bs.tile_unpack(z_sparse, square=act == G.ACT_RELU2)
    kb_list, kb_count = G.live_kblocks(z_sparse.bitmask, T, Fd)
    return G.mm(a, W2.T, kb_list=kb_list, kb_count=kb_count)


def packed_backward(grad_output, x, W1, W2, z_sparse, act=G.ACT_RELU2):
    """The backward of out = act(z) @ W2^T with z = relu(x @ W1^T) kept packed
    (a bf16 128x128-tile BitsparseTensor): (grad_x, grad_W1, grad_W2), the
    reference's FFNSpRelu2 / FFNSparse backward (old/lib_sparse/sparse.py:
    83-109,129-151) on this library's kernels, weight gradients handed to an
    attached GradAllReduce as they are produced."""
    T, Fd = z_sparse.shape
    kb_list, kb_count = G.live_kblocks(z_sparse.bitmask, T, Fd)
    gx, gW1, gW2, _ = _fused_backward(grad_output, x, W1, W2, z_sparse, G.tile_row_offsets(z_sparse), kb_list,
                                      kb_count, False, act, stats_key=W2)
    return gx, gW1, gW2


def _unfused_forward(x, W1, W2, vals, offset, b1, act):
    """float32 / float16 forward: the products on this library's tcgen05 GEMM
    (split-bf16 for these dtypes, gemm.matmul), the reference's elementwise
    steps (bias, ReLU, square) in torch, and the 64x64-tile pack.  Returns
    (out, z_sparse)."""
    preact = G.matmul(x, W1.T)
    if b1 is not None:
        preact += b1
    z = F.relu(preact)
    output = G.matmul(z * z if act == G.ACT_RELU2 else z, W2.T)
    z_sparse = bs.dense_to_tilesparse(z, vals, offset)
    return output, z_sparse


def _unfused_backward(grad_output, x, W1, W2, z_sparse, has_bias, act):
    """-> (grad_x, grad_W1, grad_W2, grad_b1 or None), old/lib_sparse/sparse.py:84-109
    (ReLU) and :129-151 (ReLU^2)."""
    grad_output = grad_output.contiguous()
    grad_z = G.matmul(grad_output, W2)
    if act == G.ACT_RELU2:
        # grad_pre = grad_z * 2z; dW2 takes z^2, which the reference stores over
        # z in place (sparse.py:136-147) -- here it is formed while unpacking, the
        # same rounding, so the stored z stay unchanged
        bs.grad_relu2_(grad_z, z_sparse, square=False)
        grad_W2 = submit_grad(bs.spAx(z_sparse, grad_output.T, square=True))
    else:
        grad_W2 = submit_grad(bs.spAx(z_sparse, grad_output.T))
        bs.mask_with_bitmask_(grad_z, z_sparse)
    grad_b1 = submit_grad(grad_z.sum(0)) if has_bias else None
    grad_W1 = submit_grad(G.matmul(grad_z.T, x))
    grad_x = G.matmul(grad_z, W1)
    return grad_x, grad_W1, grad_W2, grad_b1


def _arena(sparse_data, numel, like):
    if sparse_data is not None:
        return sparse_data
    vals = torch.empty(numel, dtype=like.dtype, device=like.device)
    off = torch.zeros(1, dtype=torch.int32, device=like.device)
    return vals, off


class _ExactVals:
    """Allocator for a layer's own values when no arena is given: called by
    the up-projection with the layer's nnz once its tiles are counted."""

    def __init__(self, like):
        self.like, self.vals = like, None

    def __call__(self, n):
        # at n == 0 a zero-length view of one element: a valid pointer for the
        # copy, which still writes the tiles' live-column masks
        self.vals = torch.empty(max(n, 1), dtype=self.like.dtype, device=self.like.device)[:n]
        return self.vals


def _forward(ctx, x, W1, W2, sparse_data, b1, act):
    exact = (sparse_data is None and not torch.compiler.is_compiling()
             and all(t.is_cuda for t in (x, W1, W2)) and not torch.cuda.is_current_stream_capturing())
    if exact and _fused_ok(x, W1, W2, b1, x):
        # No arena: the layer's values get a tensor of exactly nnz elements
        # (one device sync for the count), owned by this autograd node and
        # freed with it after the layer's backward -- no worst-case buffer,
        # and nothing kept alive for the rest of the backward.  (Traced or
        # captured into a CUDA graph, where the count cannot be read back, the
        # layer takes a worst-case buffer instead.)
        holder = _ExactVals(x)
        offset = torch.zeros(1, dtype=torch.int32, device=x.device)
        out, bitmask, prefix, voff, row_offsets, kb_list, kb_count = _fused_forward(
            x, W1, W2, holder, offset, b1, act)
        vals, fused = holder.vals, True
    elif exact and x.dtype == W1.dtype == W2.dtype and x.dtype in (torch.float32, torch.float16):
        # the float32 / float16 path likewise: the 64x64 pack counts first
        holder = _ExactVals(x)
        offset = torch.zeros(1, dtype=torch.int32, device=x.device)
        out, z = _unfused_forward(x, W1, W2, holder, offset, b1, act)
        vals, bitmask, prefix, voff = z.vals, z.bitmask, z.prefix, z.vals_offset
        # no per-row offsets or K-block lists on this path (the op's empty forms)
        row_offsets, kb_count = (torch.empty(0, dtype=torch.int32, device=x.device) for _ in range(2))
        kb_list = torch.empty(0, 0, dtype=torch.int32, device=x.device)
        fused = False
    else:
        vals, offset = _arena(sparse_data, x.shape[0] * W1.shape[0], x)
        fused = _fused_ok(x, W1, W2, b1, vals)
        # one sparseffn:: op (torch.library), so torch.compile traces through it
        out, bitmask, prefix, voff, row_offsets, kb_list, kb_count = torch.ops.sparseffn.ffn_fwd(
            x, W1, W2, b1, vals, offset, act)
    T, Fd = x.shape[0], W1.shape[0]
    bm = 128 if fused else 64
    ctx.save_for_backward(x, W1, W2)
    # the arena is not saved with save_for_backward: later layers write other
    # parts of it in place, which would fail autograd's version check
    ctx.z_sparse = bs.BitsparseTensor(vals, bitmask, prefix, voff, -(-T // bm), -(-Fd // bm), bm, bm,
                                      (T, Fd))
    ctx.aux = (row_offsets, kb_list, kb_count)
    ctx.fused, ctx.has_bias, ctx.act = fused, b1 is not None, act
    return out


def _backward(ctx, grad_output):
    x, W1, W2 = ctx.saved_tensors
    z = ctx.z_sparse
    ctx.z_sparse = None
    row_offsets, kb_list, kb_count = ctx.aux
    ctx.aux = None
    grad_x, grad_W1, grad_W2, grad_b1 = torch.ops.sparseffn.ffn_bwd(
        grad_output, x, W1, W2, z.vals, z.bitmask, z.prefix, z.vals_offset, row_offsets, kb_list,
        kb_count, ctx.fused, ctx.has_bias, ctx.act)
    return grad_x, grad_W1, grad_W2, None, (grad_b1 if ctx.has_bias else None)


class FFNSparse(Function):
    """ReLU FFN whose backward rebuilds the ReLU mask from the bitmask."""

    @staticmethod
    def forward(ctx, x, W1, W2, sparse_data, b1=None):
        return _forward(ctx, x, W1, W2, sparse_data, b1, G.ACT_RELU)

    @staticmethod
    def backward(ctx, grad_output):
        return _backward(ctx, grad_output)


class FFNSpRelu2(Function):
    """ReLU^2 FFN: saves z = relu(pre) sparsely, rebuilds z^2 and 2z in backward."""

    @staticmethod
    def forward(ctx, x, W1, W2, sparse_data=None, b1=None):
        return _forward(ctx, x, W1, W2, sparse_data, b1, G.ACT_RELU2)

    @staticmethod
    def backward(ctx, grad_output):
        return _backward(ctx, grad_output)
