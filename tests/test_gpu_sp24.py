"""2:4 structured path: compression bit-exact against the oracle, the sparse
tensor-core GEMM exact on integer-valued data, and the full product (2:4 part
plus overflow) against dense products."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def sparse_bf16(rows, cols, p_zero, seed, ints=False, neg_zero=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    if ints:
        v = torch.randint(-3, 4, (rows, cols), device=DEV, generator=g).float()
    else:
        v = torch.randn(rows, cols, device=DEV, generator=g)
    keep = torch.rand(rows, cols, device=DEV, generator=g) >= p_zero
    zero = torch.zeros((), device=DEV)
    if neg_zero:  # zeros of both signs (a kept zero slot keeps its sign)
        zero = torch.where(torch.rand(rows, cols, device=DEV, generator=g) < 0.5, zero, -zero)
    return torch.where(keep, v, zero).to(torch.bfloat16)


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("p_zero", [0.0, 0.5, 0.9])
def test_compress_matches_oracle(trans, p_zero):
    from autoresearch2_b200 import sp24
    X = sparse_bf16(256, 384, p_zero, seed=3, neg_zero=True)  # trans: A = X^T is [384, 256]
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


@pytest.mark.parametrize("b_mn", [1, 0])
def test_sp24_mm_fused_overflow_equals_two_kernels(b_mn):
    """The overflow added in the GEMM epilogue is bit-identical to the 2:4
    GEMM followed by sffn_sp24_overflow_add, and trans_out stores exactly the
    transpose."""
    from autoresearch2_b200 import _lib, sp24
    M, K, N = 384, 512, 640
    A = sparse_bf16(M, K, 0.6, seed=11, neg_zero=True)
    Bkn = sparse_bf16(K, N, 0.0, seed=12)
    B = Bkn if b_mn else Bkn.t().contiguous().t()
    a = sp24.compress(A)
    assert int(a.ovf_count.sum()) > 0
    fused = sp24.mm(a, B, bt=Bkn, fused=True)
    fused_t = sp24.mm(a, B, bt=Bkn, trans_out=True, fused=True)
    unfused_t = sp24.mm(a, B, bt=Bkn, trans_out=True)
    two = torch.empty(M, N, dtype=torch.bfloat16, device=DEV)
    st = _lib.stream_ptr(DEV)
    ldb = B.stride(0) if b_mn else B.stride(1)
    _lib.call("sffn_gemm_sp24", _lib.ptr(a.vals), _lib.ptr(a.meta), M, K, _lib.ptr(B), ldb, b_mn,
              _lib.ptr(two), two.stride(0), N, _lib.ptr(_lib.status_word(DEV)), st)
    _lib.call("sffn_sp24_overflow_add", _lib.ptr(a.ovf_cols), _lib.ptr(a.ovf_vals), _lib.ptr(a.ovf_count), M, K,
              _lib.ptr(Bkn), Bkn.stride(0), N, _lib.ptr(two), two.stride(0), st)
    _lib.check_status(DEV)
    assert torch.equal(fused.view(torch.int16), two.view(torch.int16))
    assert torch.equal(fused_t.view(torch.int16), two.t().contiguous().view(torch.int16))
    assert torch.equal(unfused_t.view(torch.int16), fused_t.view(torch.int16))


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


def assert_same_sp24(got, want):
    """Two 2:4 forms are equal: kept values and metadata bit for bit, the
    overflow entries of each row as sets (they are written in no fixed order)."""
    assert got.shape == want.shape
    assert torch.equal(got.vals.view(torch.int16), want.vals.view(torch.int16))
    assert torch.equal(got.meta, want.meta)
    assert torch.equal(got.ovf_count, want.ovf_count)
    cnt = got.ovf_count.cpu().numpy()

    def entries(a):
        oc, ov = a.ovf_cols.cpu().numpy().view(np.uint16), bits(a.ovf_vals)
        return sorted((r, int(oc[r, i]), int(ov[r, i])) for r in np.nonzero(cnt)[0] for i in range(cnt[r]))
    assert entries(got) == entries(want)


@pytest.mark.parametrize("act", [0, 1])
def test_fused_up_writes_the_compressed_activation(act):
    """The up-projection epilogue's 2:4 output equals compress() of the dense
    activation the same kernel writes without it; the sparse z is unchanged."""
    from autoresearch2_b200 import gemm, sp24
    T, D, F = 384, 256, 640
    g = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=DEV, generator=g) * D ** -0.5).to(torch.bfloat16)
    b1 = torch.full((F,), -0.6, device=DEV, dtype=torch.bfloat16)  # ~75% zeros
    outs = []
    for flag in (False, True):
        arena = torch.zeros(T * F, device=DEV, dtype=torch.bfloat16)
        off = torch.zeros(1, dtype=torch.int32, device=DEV)
        a, bitmask, prefix, voff, _ = gemm.ffn_up(x, W1, b1, act, arena, off, sp24=flag)
        outs.append((a, bitmask, prefix, arena))
    (a, bm0, pf0, ar0), (a24, bm1, pf1, ar1) = outs
    from autoresearch2_b200 import _lib
    _lib.check_status(DEV)
    assert torch.equal(bm0, bm1) and torch.equal(pf0, pf1)
    assert torch.equal(ar0.view(torch.int16), ar1.view(torch.int16))
    assert_same_sp24(a24, sp24.compress(a))
    assert int(a24.ovf_count.sum()) > 0  # the overflow path is exercised


@pytest.mark.parametrize("act", [0, 1])
def test_fused_dgrad_writes_the_compressed_gradients(act):
    """The activation-gradient epilogue's three 2:4 outputs equal compress()
    of its dense dpre (rows), dpre^T and act^T (token-dimension K); the bias
    gradient it sums on the way matches."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm, sp24
    T, D, F = 512, 256, 384
    g = torch.Generator(device=DEV).manual_seed(22)
    x = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=DEV, generator=g) * D ** -0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, device=DEV, generator=g) * F ** -0.5).to(torch.bfloat16)
    dout = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    b1 = torch.full((F,), -0.5, device=DEV, dtype=torch.bfloat16)
    arena = torch.empty(T * F, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    _, bitmask, prefix, voff, _ = gemm.ffn_up(x, W1, b1, act, arena, off)
    zs = sf.BitsparseTensor(arena, bitmask, prefix, voff, T // 128, F // 128, 128, 128, (T, F))
    db0 = torch.zeros(F, dtype=torch.float32, device=DEV)
    db1 = torch.zeros(F, dtype=torch.float32, device=DEV)
    dpre, act2 = gemm.ffn_dgrad(dout, W2, act, zs, db1=db0)
    d24, dt24, at24 = gemm.ffn_dgrad(dout, W2, act, zs, db1=db1, sp24=True)
    from autoresearch2_b200 import _lib
    _lib.check_status(DEV)
    assert_same_sp24(d24, sp24.compress(dpre))
    assert_same_sp24(dt24, sp24.compress(dpre, trans=True))
    assert_same_sp24(at24, sp24.compress(act2, trans=True))
    torch.testing.assert_close(db1, db0, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("shape", [(64, 64), (4096, 136), (200, 8), (8, 1000)])
def test_transpose16_exact(shape):
    from autoresearch2_b200 import sp24
    X = sparse_bf16(*shape, 0.3, seed=13, neg_zero=True)
    assert torch.equal(sp24.transpose(X).view(torch.int16), X.t().contiguous().view(torch.int16))
