"""GPU parity of the sparse FFN autograd functions against the reference's
golden vectors and the float64 oracle.

Tolerances (elementwise, with an absolute floor scaled to the tensor's
largest magnitude): fp32 rtol = atol/max|ref| = 1e-5; bf16 2e-2."""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def close(got, want, tol):
    got = got.detach().double().cpu().numpy()
    want = np.asarray(want, dtype=np.float64)
    np.testing.assert_allclose(got, want, rtol=tol, atol=tol * np.abs(want).max())


@pytest.fixture(autouse=True)
def _fp32_exact():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev
    import autoresearch2_b200 as sf
    sf.check_status()


@pytest.mark.parametrize("act", ["relu", "relu2"])
def test_ffn_fp32_golden(act):
    import autoresearch2_b200 as sf
    g = golden(f"ffn_{act}")
    x, W1, W2, dout = (torch.from_numpy(g[k]).to(DEV).requires_grad_(k != "dout")
                       for k in ("x", "W1", "W2", "dout"))
    fn = sf.FFNSparse if act == "relu" else sf.FFNSpRelu2
    T, F = x.shape[0], W1.shape[0]
    arena = torch.empty(T * F, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = fn.apply(x, W1, W2, (arena, off))
    out.backward(dout)
    close(out, g["out"], 1e-5)
    close(x.grad, g["dx"], 1e-5)
    close(W1.grad, g["dW1"], 1e-5)
    close(W2.grad, g["dW2"], 1e-5)
    assert int(off.item()) == int(g["nnz"][0])


@pytest.mark.parametrize("mma", ["off", "on"])
@pytest.mark.parametrize("act", ["relu", "relu2"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,D,F", [(256, 128, 384), (512, 256, 1024)])
def test_ffn_against_oracle(act, dtype, T, D, F, mma):
    """mma = "on": the bf16 products with a sparse operand run on the 2:4
    sparse tensor cores (plus the overflow); the results must not change."""
    import autoresearch2_b200 as sf
    if mma == "on" and dtype != torch.bfloat16:
        pytest.skip("the sparse tensor-core path is bf16-only")
    prev = sf.ffn.sparse_mma()
    sf.ffn.set_sparse_mma(mma)
    try:
        _ffn_against_oracle(sf, act, dtype, T, D, F)
    finally:
        sf.ffn.set_sparse_mma(prev)


def _ffn_against_oracle(sf, act, dtype, T, D, F):
    g = torch.Generator().manual_seed(T + D + F)
    x = torch.randn(T, D, generator=g)
    W1 = torch.randn(F, D, generator=g) / D ** 0.5
    W2 = torch.randn(D, F, generator=g) / F ** 0.5
    b1 = torch.full((F,), -0.8)
    dout = torch.randn(T, D, generator=g)
    cast = [t.to(dtype) for t in (x, W1, W2, b1, dout)]
    xg, W1g, W2g, b1g = (t.to(DEV).requires_grad_() for t in cast[:4])
    fn = sf.FFNSparse if act == "relu" else sf.FFNSpRelu2
    out = fn.apply(xg, W1g, W2g, None, b1g)
    gpu_mask = (out.grad_fn.z_sparse.to_dense() > 0).cpu().numpy()
    out.backward(cast[4].to(DEV))
    np_in = [oracle.f32_to_bf16(t.float().numpy()) if dtype == torch.bfloat16 else t.numpy()
             for t in cast]
    code = oracle.BF16 if dtype == torch.bfloat16 else oracle.F32
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    # The device mask may differ from the oracle's only where the
    # pre-activation is within rounding of zero (a few ulps of bf16/fp32).
    r0 = oracle.ffn_fwd_bwd(np_in[0], np_in[1], np_in[2], np_in[4], act=act, b1=np_in[3], code=code)
    flips = gpu_mask != r0["mask"]
    ulp_bound = 2.0 ** -6 if dtype == torch.bfloat16 else 2.0 ** -14
    assert np.all(np.abs(r0["pre"][flips]) <= ulp_bound), np.abs(r0["pre"][flips]).max()
    assert flips.mean() < 1e-2
    r = oracle.ffn_fwd_bwd(np_in[0], np_in[1], np_in[2], np_in[4], act=act, b1=np_in[3], code=code,
                           mask=gpu_mask)
    close(out, r["out"], tol)
    close(xg.grad, r["dx"], tol)
    close(W1g.grad, r["dW1"], tol)
    close(W2g.grad, r["dW2"], tol)
    close(b1g.grad, r["db1"], tol)


@pytest.mark.parametrize("shift,expect", [(-3.2, "sp24"), (-0.5, "dense")])
def test_auto_mode_follows_observed_sparsity(shift, expect):
    """Auto mode: the first step runs dense and records the activation's
    non-zero count without waiting; later steps take the 2:4 products when
    that step had >= AUTO_MIN_SPARSITY zeros.  Both paths give the same result
    within the bf16 bar."""
    import autoresearch2_b200 as sf
    prev = sf.ffn.sparse_mma()
    sf.ffn.set_sparse_mma("auto")
    try:
        T, D, F = 512, 256, 512
        g = torch.Generator(device="cuda").manual_seed(31)
        x = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
        W1 = (torch.randn(F, D, device="cuda", generator=g) * D ** -0.5).to(torch.bfloat16)
        W2 = (torch.randn(D, F, device="cuda", generator=g) * F ** -0.5).to(torch.bfloat16)
        b1 = torch.full((F,), shift, device="cuda", dtype=torch.bfloat16)
        outs, paths = [], []
        for _ in range(3):
            arena = (torch.empty(T * F, device="cuda", dtype=torch.bfloat16),
                     torch.zeros(1, dtype=torch.int32, device="cuda"))
            outs.append(sf.FFNSpRelu2.apply(x, W1, W2, arena, b1).float())
            paths.append(sf.ffn.last_path())
            torch.cuda.synchronize()
        assert paths[0] == "dense" and paths[-1] == expect, paths
        scale = outs[0].abs().max().item() + 1e-6
        assert (outs[-1] - outs[0]).abs().max().item() <= 2e-2 * scale
    finally:
        sf.ffn.set_sparse_mma(prev)


@pytest.mark.parametrize("act", ["relu", "relu2"])
@pytest.mark.parametrize("T,D,F", [(384, 256, 640), (1024, 512, 2048)])
def test_lean_backward_gives_the_same_bits(act, T, D, F):
    """The lean backward rebuilds the activation from the packed z by an
    unpack (squared in bf16 for ReLU^2) instead of taking it from the
    activation-gradient epilogue; the activation is the same bits either way,
    so every gradient must be bit-identical between the two modes."""
    import autoresearch2_b200 as sf
    prev_mma, prev_bw = sf.sparse_mma(), sf.backward_mode()
    sf.set_sparse_mma("off")
    g = torch.Generator(device=DEV).manual_seed(T + F)
    x = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=DEV, generator=g) * D ** -0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, device=DEV, generator=g) * F ** -0.5).to(torch.bfloat16)
    b1 = torch.full((F,), -0.8, device=DEV, dtype=torch.bfloat16)
    dout = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    fn = sf.FFNSparse if act == "relu" else sf.FFNSpRelu2
    res = {}
    try:
        for mode in ("fused", "lean"):
            sf.set_backward(mode)
            ps = [t.clone().requires_grad_() for t in (x, W1, W2, b1)]
            out = fn.apply(ps[0], ps[1], ps[2], None, ps[3])
            out.backward(dout)
            res[mode] = [out.detach()] + [p.grad for p in ps]
    finally:
        sf.set_sparse_mma(prev_mma)
        sf.set_backward(prev_bw)
    for name, a, b in zip(("out", "dx", "dW1", "dW2", "db1"), res["fused"], res["lean"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16)), name


def test_second_step_without_kblock_lists_gives_the_same_bits():
    """After a step whose activation had (nearly) every (tile, column) pair
    live, the next step builds no K-block lists (full counts only) and the
    GEMMs read none; outputs and gradients must be the same bits as the first
    step's, which ran with the lists."""
    import autoresearch2_b200 as sf
    prev = sf.sparse_mma()
    sf.set_sparse_mma("off")
    T, D, F = 1024, 256, 1024
    g = torch.Generator(device=DEV).manual_seed(77)
    x = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=DEV, generator=g) * D ** -0.5).to(torch.bfloat16).requires_grad_()
    W2 = (torch.randn(D, F, device=DEV, generator=g) * F ** -0.5).to(torch.bfloat16).requires_grad_()
    dout = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    runs = []
    try:
        for _ in range(2):
            W1.grad = W2.grad = None
            out = sf.FFNSpRelu2.apply(x, W1, W2)
            out.backward(dout)
            torch.cuda.synchronize()
            runs.append([out.detach().clone(), W1.grad.clone(), W2.grad.clone()])
        _, live = sf.ffn._stats(T, D, F, W1)  # (setting the mode again forgets the statistics)
    finally:
        sf.set_sparse_mma(prev)
    assert live is not None and live >= sf.ffn.FULL_KBLOCKS_MIN_LIVE
    for a, b in zip(*runs):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("act", ["relu", "relu2"])
@pytest.mark.parametrize("backward", ["fused", "lean"])
@pytest.mark.parametrize("T,D,F", [(300, 72, 200), (130, 264, 392), (1000, 136, 136)])
def test_ffn_ragged_shapes_against_oracle(act, backward, T, D, F):
    """Shapes whose tokens and hidden width are not multiples of the 128x128
    format tile: the last tiles are partial (rows past T, columns past F), so
    the up-projection's warp-packed slots, the per-group copy into the arena,
    the activation gradient's prefetched z tile and the K-block lists all
    meet their edge cases.  bf16 against the float64 oracle, both backward
    modes."""
    import autoresearch2_b200 as sf
    prev_mma, prev_bw = sf.ffn.sparse_mma(), sf.backward_mode()
    sf.ffn.set_sparse_mma("off")
    sf.set_backward(backward)
    try:
        _ffn_against_oracle(sf, act, torch.bfloat16, T, D, F)
    finally:
        sf.ffn.set_sparse_mma(prev_mma)
        sf.set_backward(prev_bw)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_exact_size_values_on_the_64x64_path(dtype):
    """float32 / float16 layers given no arena: the 64x64 pack counts first
    and keeps exactly nnz values; output and gradients the same bits as the
    same layer over an arena, the packed values equal."""
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(91)
    T, D, F = 300, 64, 200
    x = torch.randn(T, D, device=DEV, generator=g).to(dtype).requires_grad_()
    W1 = (torch.randn(F, D, device=DEV, generator=g) * D ** -0.5).to(dtype).requires_grad_()
    W2 = (torch.randn(D, F, device=DEV, generator=g) * F ** -0.5).to(dtype).requires_grad_()
    b1 = torch.full((F,), -0.3, device=DEV, dtype=dtype, requires_grad=True)
    dout = torch.randn(T, D, device=DEV, generator=g).to(dtype)
    res = []
    for sd in ((torch.empty(T * F, dtype=dtype, device=DEV), torch.zeros(1, dtype=torch.int32, device=DEV)),
               None):
        out = sf.FFNSpRelu2.apply(x, W1, W2, sd, b1)
        z = out.grad_fn.z_sparse
        n = int(z.prefix[-1].item())
        if sd is None:
            assert z.vals.numel() == n > 0 and z.BLOCK_M == 64
        vals = z.vals[int(z.vals_offset.item()):][:n].clone()
        grads = torch.autograd.grad(out, (x, W1, W2, b1), dout)
        res.append((out.detach(), vals, grads))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
    for a, b in zip(res[0][2], res[1][2]):
        assert torch.equal(a, b)
    sf.check_status()
