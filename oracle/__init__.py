"""CPU oracle for the activation-sparse FFN path -- TEST INFRASTRUCTURE ONLY.

This package restates the reference's algorithms on the CPU so that tests,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg can check and
time the CUDA library against them.  The product package never imports it.

Pinning: every function here is checked in ``tests/test_oracle_golden.py``
against golden vectors produced by running the reference's own Triton code
under Triton's CPU interpreter (``tests/golden/make_golden.py``).

Byte/bit work (flat and tiled pack/unpack) is in C (``oracle.c`` ->
``liboracle.so``, built by ``oracle/Makefile``); floating-point work (mask
kernels, spAx, FFN forward/backward) is numpy.

Conventions: arrays are numpy; bfloat16 data is carried as its uint16 bit
pattern.  dtype codes: 0 = float32, 1 = bfloat16, 2 = float16.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32, BF16, F16 = 0, 1, 2

_lib = None


def build():
    """Compile liboracle.so (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    """Load liboracle.so, building it first if it is missing."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_flat_pack.argtypes = [vp, ctypes.c_int, i64, vp, vp, i64, ctypes.c_int]
        L.orc_flat_pack.restype = i64
        L.orc_flat_unpack.argtypes = [vp, i64, vp, ctypes.c_int, i64, vp, ctypes.c_int]
        L.orc_flat_unpack.restype = i64
        L.orc_tile_pack.argtypes = [vp, ctypes.c_int, i64, i64, i64, ctypes.c_int, ctypes.c_int,
                                    vp, vp, vp, i64, i64]
        L.orc_tile_pack.restype = i64
        L.orc_tile_unpack.argtypes = [vp, vp, vp, i64, ctypes.c_int, i64, i64, ctypes.c_int,
                                      ctypes.c_int, i64, i64, vp, i64]
        L.orc_tile_unpack.restype = None
        del i32
        _lib = L
    return _lib


def num_threads():
    return lib().orc_num_threads()


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def dtype_code(a):
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:
        return BF16
    if a.dtype == np.float16:
        return F16
    raise TypeError(f"unsupported oracle dtype {a.dtype}")


# ---------------------------------------------------------------------------
# bf16 helpers (bit patterns <-> float32)
# ---------------------------------------------------------------------------
def bf16_to_f32(u16):
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f):
    """Round-to-nearest-even float32 -> bf16 bits (NaN kept quiet)."""
    f = np.ascontiguousarray(f, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def to_f64(a, code):
    if code == BF16:
        return bf16_to_f32(a).astype(np.float64)
    return np.asarray(a, dtype=np.float64)


def from_f64(x, code):
    """Round a float64 array to the storage dtype (via float32 for bf16)."""
    if code == BF16:
        return f32_to_bf16(np.asarray(x, dtype=np.float32))
    if code == F16:
        return np.asarray(x, dtype=np.float16)
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# Flat format (old/sparse_pack.py:66-106, old/sparse_unpack.py:57-97)
# ---------------------------------------------------------------------------
def pack_bool_mask(mask):
    """Golden packer of old/bitpack/prepare.py:6-23: bit i -> byte i//8, bit i%8."""
    mask = np.asarray(mask, dtype=bool).ravel()
    n = mask.size
    nb = (n + 7) // 8
    padded = np.zeros(nb * 8, dtype=np.uint8)
    padded[:n] = mask
    return (padded.reshape(nb, 8) << np.arange(8, dtype=np.uint8)).sum(axis=1).astype(np.uint8)


def flat_pack(dense, nthreads=1):
    """(vals, packed_mask) for a dense array (any shape, row-major)."""
    d = np.ascontiguousarray(dense).ravel()
    code = dtype_code(d)
    n = d.size
    mask = np.zeros((n + 7) // 8, dtype=np.uint8)
    vals = np.empty(n, dtype=d.dtype)
    nnz = lib().orc_flat_pack(_ptr(d), code, n, _ptr(mask), _ptr(vals), n, nthreads)
    assert nnz >= 0
    return vals[:nnz].copy(), mask


def flat_unpack(vals, packed_mask, shape, nthreads=1):
    vals = np.ascontiguousarray(vals)
    mask = np.ascontiguousarray(packed_mask, dtype=np.uint8)
    n = int(np.prod(shape))
    out = np.empty(n, dtype=vals.dtype)
    used = lib().orc_flat_unpack(_ptr(vals), vals.size, _ptr(mask), dtype_code(vals), n,
                                 _ptr(out), nthreads)
    if used < 0:
        raise ValueError("packed mask has more set bits than vals holds")
    return out.reshape(shape)


# ---------------------------------------------------------------------------
# Tiled format (old/lib_sparse/sparse.py:154-210, sparse_pack.py, sparse_unpack.py)
# ---------------------------------------------------------------------------
def tile_pack(dense, BM, BN, vals_arena, offset):
    """Pack ``dense`` [M, N] into (bitmask, prefix) and write its values into
    ``vals_arena`` from ``offset``.  Returns (bitmask, prefix, total)."""
    d = np.ascontiguousarray(dense)
    M, N = d.shape
    gm, gn = -(-M // BM), -(-N // BN)
    bitmask = np.zeros(gm * gn * BM * BN // 8, dtype=np.uint8)
    prefix = np.zeros(gm * gn + 1, dtype=np.int32)
    assert vals_arena.dtype == d.dtype and vals_arena.flags.c_contiguous
    total = lib().orc_tile_pack(_ptr(d), dtype_code(d), M, N, N, BM, BN, _ptr(bitmask),
                                _ptr(prefix), _ptr(vals_arena), vals_arena.size, int(offset))
    if total < 0:
        raise ValueError("vals arena too small")
    return bitmask, prefix, total


def tile_unpack(vals, bitmask, prefix, offset, shape, BM, BN, row0=0, rows=None):
    vals = np.ascontiguousarray(vals)
    M, N = shape
    rows = M - row0 if rows is None else rows
    out = np.zeros((rows, N), dtype=vals.dtype)
    lib().orc_tile_unpack(_ptr(vals), _ptr(np.ascontiguousarray(bitmask)),
                          _ptr(np.ascontiguousarray(prefix, dtype=np.int32)), int(offset),
                          dtype_code(vals), M, N, BM, BN, row0, rows, _ptr(out), N)
    return out


def tile_bits(bitmask, shape, BM, BN):
    """Boolean [M, N] mask from a tiled bitmask."""
    M, N = shape
    gm, gn = -(-M // BM), -(-N // BN)
    bits = np.unpackbits(np.asarray(bitmask, dtype=np.uint8), bitorder="little")
    bits = bits.reshape(gm, gn, BM, BN).transpose(0, 2, 1, 3).reshape(gm * BM, gn * BN)
    return bits[:M, :N].astype(bool)


def mask_with_bitmask(grad, bitmask, BM, BN):
    """K7 (old/lib_sparse/sparse_unpack.py:72-107): where(bit, grad, 0)."""
    code = dtype_code(grad)
    bits = tile_bits(bitmask, grad.shape, BM, BN)
    g = grad.copy()
    g[~bits] = 0
    return g if code != F32 else g.astype(np.float32)


def grad_relu2(grad, vals, bitmask, prefix, offset, BM, BN):
    """K8 (old/lib_sparse/sparse_unpack.py:110-147) with square=True:
    returns (grad * 2 * z rounded to the storage dtype, vals with z -> z*z).
    Off-mask z is 0, so grad*0 (NaN/Inf grad gives NaN there, as in the reference)."""
    code = dtype_code(grad)
    M, N = grad.shape
    z = tile_unpack(vals, bitmask, prefix, offset, (M, N), BM, BN)
    g = to_f64(grad, code)
    zf = to_f64(z, code)
    # Triton evaluates (gz * 2.0) * z in the storage dtype; 2.0 scaling is exact.
    out = from_f64(to_f64(from_f64(g * 2.0, code), code) * zf, code)
    v = vals.copy()
    nnz = int(prefix[-1])
    seg = to_f64(v[offset:offset + nnz], code)
    v[offset:offset + nnz] = from_f64(seg * seg, code)
    return out, v


def spAx(vals, bitmask, prefix, offset, shape, BM, BN, W, square=False):
    """spAx (old/lib_sparse/sparse.py:305-351): W @ unpack(x) (optionally squared),
    computed in float64 and rounded to W's dtype."""
    code = dtype_code(W)
    dense = to_f64(tile_unpack(vals, bitmask, prefix, offset, shape, BM, BN), code)
    if square:
        dense = to_f64(from_f64(dense * dense, code), code)
    return from_f64(to_f64(W, code) @ dense, code)


def relu_matmul(A, B, code=F32):
    """relu(A @ B) in float64 from operands of dtype `code`: the product of
    sparse_relu_Ax / sp_relu_Ax (relu(x @ W1.T), old/matmul_bitsparse/train.py:
    45-52, old/full_matmul/train.py:35), relu_spAx (relu(unpack @ W2.T),
    old/full_matmul/train.py:177-178) and relu_sparse_Ax (relu(A @ x),
    old/sparse_matmul/train.py:44-50)."""
    return np.maximum(to_f64(A, code) @ to_f64(B, code), 0.0)


def relu_ax_pack(x, W1, BM=128, BN=128):
    """sparse_relu_Ax (old/matmul_bitsparse/train.py:70-116) for float32: the
    float64 product rounded to float32, then the tiled pack of its positive
    entries -> (vals, bitmask, prefix)."""
    z = relu_matmul(x, np.ascontiguousarray(W1).T).astype(np.float32)
    arena = np.zeros(z.size, dtype=np.float32)
    bitmask, prefix, total = tile_pack(z, BM, BN, arena, 0)
    return arena[:total], bitmask, prefix


# ---------------------------------------------------------------------------
# FFN forward / backward (sparse.py:56-151, prepare_layer.py:12-29,117-162)
# ---------------------------------------------------------------------------
def ffn_fwd_bwd(x, W1, W2, dout, act="relu2", b1=None, code=F32, compute=np.float64, mask=None):
    """Forward and backward of out = act(x @ W1.T [+ b1]) @ W2.T.

    act = "relu" follows FFNSparse / FFNv3; act = "relu2" follows FFNSpRelu2 /
    FFNrelu2 (a = relu(pre)^2, d pre = d a * 2 z on the mask).  Products are
    accumulated in float64; every intermediate that the reference stores in
    the storage dtype (pre, z, a, d a, d pre) is rounded to it.
    `compute` = np.float32 runs the products in float32 (the timed CPU
    baseline); the default float64 is the checker.  `mask` (bool [T, F])
    overrides the ReLU mask, so a device result can be checked with the mask
    it actually produced (elements whose pre-activation rounds across zero
    differently in another GEMM flip the ReLU derivative).
    Returns dict(out, dx, dW1, dW2, z, mask)."""
    def r(t):  # round to the storage dtype
        return to_f64(from_f64(t, code), code).astype(compute, copy=False)
    xf, W1f, W2f, gf = (to_f64(t, code).astype(compute, copy=False) for t in (x, W1, W2, dout))
    pre = xf @ W1f.T
    if b1 is not None:
        pre = pre + to_f64(b1, code).astype(compute, copy=False)
    pre = r(pre)
    if mask is None:
        mask = pre > 0
    z = np.where(mask, np.maximum(pre, 0.0), np.zeros((), dtype=compute))
    a = r(z * z) if act == "relu2" else z
    out = a @ W2f.T
    dA = r(gf @ W2f)
    dW2 = gf.T @ a
    if act == "relu2":
        dpre = r(r(dA * 2.0) * z)
    else:
        dpre = np.where(mask, dA, np.zeros((), dtype=compute))
    dx = dpre @ W1f
    dW1 = dpre.T @ xf
    res = dict(out=out, dx=dx, dW1=dW1, dW2=dW2, z=z, mask=mask, dpre=dpre, a=a, pre=pre)
    if b1 is not None:
        res["db1"] = dpre.sum(axis=0)
    return res


# ------------------------------------------------------------------ 2:4 ----
# The 2:4 structured form used by the library's sparse tensor-core GEMMs.  It
# has no counterpart in the reference (whose products are dense cuBLAS
# matmuls, old/lib_sparse/sparse.py:75,95-100,118,136-139); what must match
# the reference is the product, checked end to end against dense products.
# Here: A [M, K] (uint16 bf16 bits), K % 128 == 0, M % 128 == 0.
#   vals [M, K/2]: per group of 4 (k = 4q..4q+3) the first two non-zero
#     elements by position (non-zero: magnitude bits != 0); a group with
#     fewer keeps zero slots so that idx0 < idx1 (one non-zero at p: p and 3,
#     or 2 and 3 when p == 3; none: 0 and 1).  A slot holds the bits of the
#     element at its index, so a kept zero keeps its sign (+0 or -0).
#   nib [M, K/4]: idx0 | idx1 << 2.
#   meta [M/128, K/128, 128 lanes, 4 words]: word j of lane
#     dp = m0 + 8*k1 + 16*m2 holds the nibbles of K-half k1 (4 groups) of the
#     j-th 32-wide K step for row 16*m2 + m0 (bits 0-15) and row
#     16*m2 + m0 + 8 (bits 16-31), group g at bits 4g.
#   overflow: the 3rd and 4th non-zero of each group, (row, col, value).
def _sp24_lut():
    k0 = np.zeros(16, np.int64)
    k1 = np.zeros(16, np.int64)
    ov = np.zeros(16, np.uint8)
    for p in range(16):
        idx = [i for i in range(4) if (p >> i) & 1]
        keep = idx[:2]
        if not keep:
            keep = [0, 1]
        elif len(keep) == 1:
            keep = sorted([keep[0], 3 if keep[0] != 3 else 2])
        k0[p], k1[p] = keep
        for i in idx[2:]:
            ov[p] |= 1 << i
    return k0, k1, ov


_SP24 = _sp24_lut()


def sp24_compress(a_bits):
    """-> (vals [M, K/2] uint16, nib [M, K/4] uint8, ovf_rows, ovf_cols, ovf_vals)
    with the overflow in row-major order."""
    a_bits = np.ascontiguousarray(a_bits, dtype=np.uint16)
    M, K = a_bits.shape
    g = a_bits.reshape(M, K // 4, 4)
    nzm = (g & 0x7FFF) != 0
    pat = (nzm * (1 << np.arange(4))).sum(-1)
    k0, k1, ov = _SP24[0][pat], _SP24[1][pat], _SP24[2][pat]
    v0 = np.take_along_axis(g, k0[..., None], -1)[..., 0]
    v1 = np.take_along_axis(g, k1[..., None], -1)[..., 0]
    vals = np.stack([v0, v1], -1).reshape(M, K // 2).astype(np.uint16)
    nib = (k0 | (k1 << 2)).astype(np.uint8)
    ovm = ((ov[..., None] >> np.arange(4)) & 1).astype(bool).reshape(M, K)
    rows, cols = np.nonzero(ovm)
    return vals, nib, rows, cols, a_bits[rows, cols]


def sp24_meta(nib):
    """nib [M, K/4] -> uint32 [M/128, K/128, 128, 4] in tensor-memory lane order."""
    M, G = nib.shape
    K = 4 * G
    n = nib.astype(np.uint32).reshape(M // 128, 128, K // 128, 4, 2, 4)  # tm, row, kb, j, k1, g
    half = (n << (4 * np.arange(4, dtype=np.uint32))).sum(-1, dtype=np.uint32)  # tm, row, kb, j, k1
    r = half.reshape(M // 128, 8, 2, 8, K // 128, 4, 2)  # tm, m2, m1, m0, kb, j, k1
    w = r[:, :, 0] | (r[:, :, 1] << 16)  # tm, m2, m0, kb, j, k1
    w = w.transpose(0, 3, 1, 5, 2, 4)  # tm, kb, m2, k1, m0, j  -> lane = m0 + 8*k1 + 16*m2
    return np.ascontiguousarray(w.reshape(M // 128, K // 128, 128, 4), dtype=np.uint32)


def sp24_project(vals, nib):
    """The dense [M, K] matrix (uint16 bits) that vals/nib represent."""
    M, half = vals.shape
    K = 2 * half
    out = np.zeros((M, K // 4, 4), np.uint16)
    v = vals.reshape(M, K // 4, 2)
    i0 = (nib & 3).astype(np.int64)
    i1 = (nib >> 2).astype(np.int64)
    np.put_along_axis(out, i0[..., None], v[..., 0:1], -1)
    np.put_along_axis(out, i1[..., None], v[..., 1:2], -1)
    return out.reshape(M, K)


# ---------------------------------------------------------------------------
# 15-bit sign-strip codec (bitshifting/code.py)
# ---------------------------------------------------------------------------
def codec15_bytes(n):
    """Length of the packed stream of n values: ceil(15 n / 8) bytes (code.py:135)."""
    return (15 * n + 7) // 8


def codec15_compress(bits):
    """Pack 16-bit words into a stream of 15-bit fields, value i at stream bits
    [15 i, 15 i + 15), bytes little-endian.  Follows the reference's byte
    formula (code.py:39-69): byte b starts at stream bit 8 b, inside value
    i = 8 b // 15 at offset o = 8 b % 15, and is ((v[i] >> o) | (v[i+1] << (15 - o)))
    & 0xFF with v[n] = 0.  The full 16-bit words enter that formula, so a set
    sign bit of v[i] lands on stream bit 15 (i + 1) whenever the byte holding
    that bit starts inside v[i] (15 (i + 1) % 8 != 0); for non-negative data,
    the codec's intended input, the stream is exactly the 15-bit fields."""
    v = np.asarray(bits, dtype=np.uint16).reshape(-1).astype(np.uint32)
    n = v.size
    b = np.arange(codec15_bytes(n), dtype=np.int64)
    i = (8 * b) // 15
    o = ((8 * b) % 15).astype(np.uint32)
    vp = np.concatenate([v, np.zeros(1, np.uint32)])
    return (((vp[i] >> o) | (vp[i + 1] << (15 - o))) & 0xFF).astype(np.uint8)


def codec15_uncompress(stream, n):
    """Value i = stream bits [15 i, 15 i + 15), sign bit 0 (code.py:98-122)."""
    s = np.zeros(codec15_bytes(n) + 4, np.uint8)
    s[:codec15_bytes(n)] = np.asarray(stream, dtype=np.uint8).reshape(-1)[:codec15_bytes(n)]
    k = 15 * np.arange(n, dtype=np.int64)
    byte, sh = k // 8, (k % 8).astype(np.uint32)
    w = (s[byte].astype(np.uint32) | (s[byte + 1].astype(np.uint32) << 8)
         | (s[byte + 2].astype(np.uint32) << 16))
    return ((w >> sh) & 0x7FFF).astype(np.uint16)
