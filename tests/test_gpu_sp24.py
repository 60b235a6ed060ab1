"""2:4 structured path: compression bit-exact against the oracle, the sparse
tensor-core GEMM exact on integer-valued data, and the full product (2:4 part
plus overflow) against dense products."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def sparse_bf16(rows, cols, p_zero, seed, ints=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    if ints:
        v = torch.randint(-3, 4, (rows, cols), device=DEV, generator=g).float()
    else:
        v = torch.randn(rows, cols, device=DEV, generator=g)
    keep = torch.rand(rows, cols, device=DEV, generator=g) >= p_zero
    return torch.where(keep, v, torch.zeros((), device=DEV)).to(torch.bfloat16)


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("p_zero", [0.0, 0.5, 0.9])
def test_compress_matches_oracle(trans, p_zero):
    from autoresearch2_b200 import sp24
    X = sparse_bf16(256, 384, p_zero, seed=3)  # trans: A = X^T is [384, 256]
    a = sp24.compress(X, trans=trans)
    A_bits = bits(X).T.copy() if trans else bits(X)
    vals, nib, rows, cols, ovals = oracle.sp24_compress(A_bits)
    assert np.array_equal(bits(a.vals), vals)
    assert np.array_equal(a.meta.cpu().numpy().view(np.uint32), oracle.sp24_meta(nib))
    cnt = a.ovf_count.cpu().numpy()
    assert np.array_equal(cnt, np.bincount(rows, minlength=A_bits.shape[0]))
    oc = a.ovf_cols.cpu().numpy().view(np.uint16)
    ov = bits(a.ovf_vals)
    got = sorted((r, int(oc[r, i]), int(ov[r, i])) for r in range(len(cnt)) for i in range(cnt[r]))
    assert got == sorted(zip(rows.tolist(), cols.tolist(), ovals.tolist()))


@pytest.mark.parametrize("b_mn", [1, 0])
@pytest.mark.parametrize("shape", [(256, 256, 256), (512, 384, 640)])
def test_sp24_gemm_exact_on_integers(b_mn, shape):
    """The 2:4 part alone: integer data makes the fp32 sums exact, so the
    result must equal bf16(exact product) bit for bit."""
    from autoresearch2_b200 import _lib, sp24
    M, K, N = shape
    A = sparse_bf16(M, K, 0.7, seed=5, ints=True)
    Bkn = sparse_bf16(K, N, 0.0, seed=6, ints=True)
    a = sp24.compress(A)
    vals, nib, _, _, _ = oracle.sp24_compress(bits(A))
    P = torch.from_numpy(oracle.sp24_project(vals, nib).view(np.int16)).to(DEV).view(torch.bfloat16)
    want = (P.float() @ Bkn.float()).to(torch.bfloat16)
    B = Bkn if b_mn else Bkn.t().contiguous().t()  # [K, N] view of a row-major [N, K]
    out = torch.full((M, N), 7.0, dtype=torch.bfloat16, device=DEV)
    L = _lib.load()
    st = _lib.stream_ptr(DEV)
    ldb = B.stride(0) if b_mn else B.stride(1)
    _lib.call("sffn_gemm_sp24", _lib.ptr(a.vals), _lib.ptr(a.meta), M, K, _lib.ptr(B), ldb, b_mn,
              _lib.ptr(out), out.stride(0), N, _lib.ptr(_lib.status_word(DEV)), st)
    _lib.check_status(DEV)
    assert torch.equal(out, want)


@pytest.mark.parametrize("p_zero", [0.5, 0.9])
@pytest.mark.parametrize("b_mn", [1, 0])
def test_sp24_mm_matches_dense(p_zero, b_mn):
    from autoresearch2_b200 import sp24
    M, K, N = 384, 512, 640
    A = sparse_bf16(M, K, p_zero, seed=7)
    Bkn = sparse_bf16(K, N, 0.0, seed=8)
    B = Bkn if b_mn else Bkn.t().contiguous().t()
    out = sp24.mm(sp24.compress(A), B)
    from autoresearch2_b200 import _lib
    _lib.check_status(DEV)
    want = A.float() @ Bkn.float()
    err = (out.float() - want).abs().max() / want.abs().max()
    assert err < 2e-2, err


def test_sp24_transposed_operand_matches_dense():
    """dW-style product: A = X^T compressed along X's rows (the token dim)."""
    from autoresearch2_b200 import sp24
    T, F, D = 512, 384, 256
    X = sparse_bf16(T, F, 0.9, seed=9)   # [T, F]
    Y = sparse_bf16(T, D, 0.0, seed=10)  # [T, D]
    out = sp24.mm(sp24.compress(X, trans=True), Y)  # X^T @ Y  [F, D]
    want = X.float().t() @ Y.float()
    err = (out.float() - want).abs().max() / want.abs().max()
    assert err < 2e-2, err
