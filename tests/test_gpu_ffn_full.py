"""GPU parity of the fused bf16 FFN at the shapes that are benchmarked.

* d_model=4096, d_ff=14336 with 1024 tokens: outputs and every gradient
  against the float64 oracle (oracle.ffn_fwd_bwd, the reference's
  FFNSpRelu2 / FFNrelu2, old/lib_sparse/sparse.py:112-151 and
  prepare_layer.py:12-29), driven by the device's own ReLU mask.
* The same layer with the full 16384 tokens of the headline workload: the
  forward's tiled bitmask, prefix and vals arena bit for bit against
  dense_to_tilesparse applied to the kernel's own z, z against torch, and
  outputs and gradients against torch float32 products of the same bf16
  operands (cuBLAS in fp32, TF32 off).
* The single-layer CPU configuration (8192 tokens, d_model=768, d_ff=3072,
  float32, bias -1.3) on the GPU against the oracle at 1e-5.

Every case runs with the dense products, with the 2:4 sparse tensor-core
products and with the compacted-K down-projection and dX, at 80%, 90% and
99% zeros.  Tolerances (elementwise,
absolute floor scaled to the tensor's largest magnitude): bf16 2e-2,
float32 1e-5."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
D, F = 4096, 14336
BF16_TOL, F32_TOL = 2e-2, 1e-5


def close(got, want, tol, what):
    got = got.detach().double()
    want = want.detach().double() if isinstance(want, torch.Tensor) else torch.from_numpy(
        np.asarray(want, dtype=np.float64))
    want = want.to(got.device)
    floor = tol * want.abs().max().item()
    bad = (got - want).abs() > tol * want.abs() + floor
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} elements off, max |diff| " \
                                f"{(got - want).abs().max().item():.3g} (floor {floor:.3g})"


@pytest.fixture(autouse=True)
def _fp32_exact_and_status():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev
    import autoresearch2_b200 as sf
    sf.check_status()


@pytest.fixture
def path(request):
    """The products' path: dense tcgen05 GEMMs, 2:4 sparse tensor cores, or
    the compacted-K down-projection and dX."""
    import autoresearch2_b200 as sf
    prev = sf.sparse_mma(), sf.compact_k()
    sf.set_sparse_mma("on" if request.param == "sp24" else "off")
    sf.set_compact_k("on" if request.param == "ck" else "off")
    yield request.param
    sf.set_sparse_mma(prev[0])
    sf.set_compact_k(prev[1])


def _inputs(T, s, seed):
    """bf16 x ~ N(0,1), W1 ~ N(0,1/D), W2 ~ N(0,1/F), dout ~ N(0,1) and the
    scalar bias that leaves a fraction s of zeros after the ReLU."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=DEV, generator=g) / D ** 0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, device=DEV, generator=g) / F ** 0.5).to(torch.bfloat16)
    dout = torch.randn(T, D, device=DEV, generator=g).to(torch.bfloat16)
    pre = (x[:512].float() @ W1.float().T).flatten()
    bias = float(-torch.quantile(pre[::16], s))
    b1 = torch.full((F,), bias, device=DEV, dtype=torch.bfloat16)
    return x, W1, W2, b1, dout


def _run(x, W1, W2, b1, dout):
    import autoresearch2_b200 as sf
    T = x.shape[0]
    xg, W1g, W2g, b1g = (t.clone().requires_grad_() for t in (x, W1, W2, b1))
    arena = torch.full((T * F,), 3.0, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = sf.FFNSpRelu2.apply(xg, W1g, W2g, (arena, off), b1g)
    zs = out.grad_fn.z_sparse
    z = zs.to_dense()
    snap = {"bitmask": zs.bitmask.clone(), "prefix": zs.prefix.clone(), "arena": arena.clone(),
            "off": int(off.item()), "vals_offset": int(zs.vals_offset.item())}
    out.backward(dout)
    torch.cuda.synchronize()
    return out, z, snap, (xg.grad, W1g.grad, W2g.grad, b1g.grad)


@pytest.mark.parametrize("path", ["dense", "sp24", "ck"], indirect=True)
@pytest.mark.parametrize("s", [0.8, 0.9, 0.99])
def test_headline_shape_against_oracle(s, path):
    """1024 tokens of the d=4096/14336 layer against the float64 oracle."""
    import autoresearch2_b200 as sf
    x, W1, W2, b1, dout = _inputs(1024, s, seed=int(s * 100))
    out, z, _, (dx, dW1, dW2, db1) = _run(x, W1, W2, b1, dout)
    assert sf.ffn.last_path() == path
    mask = (z > 0).cpu().numpy()
    assert abs(1 - mask.mean() - s) < 0.02
    bits = [oracle.f32_to_bf16(t.float().cpu().numpy()) for t in (x, W1, W2, dout, b1)]
    r0 = oracle.ffn_fwd_bwd(bits[0], bits[1], bits[2], bits[3], act="relu2", b1=bits[4], code=oracle.BF16)
    # the device mask may differ only where the pre-activation rounds to within
    # bf16 rounding of zero
    flips = mask != r0["mask"]
    assert np.all(np.abs(r0["pre"][flips]) <= 2.0 ** -6)
    assert flips.mean() < 1e-3
    r = oracle.ffn_fwd_bwd(bits[0], bits[1], bits[2], bits[3], act="relu2", b1=bits[4], code=oracle.BF16,
                           mask=mask)
    close(z.float(), r["z"], BF16_TOL, "z")
    close(out, r["out"], BF16_TOL, "out")
    close(dx, r["dx"], BF16_TOL, "dx")
    close(dW1, r["dW1"], BF16_TOL, "dW1")
    close(dW2, r["dW2"], BF16_TOL, "dW2")
    close(db1, r["db1"], BF16_TOL, "db1")


@pytest.mark.parametrize("path", ["dense", "sp24", "ck"], indirect=True)
@pytest.mark.parametrize("s", [0.8, 0.9, 0.99])
def test_headline_workload_full_tokens(s, path):
    """All 16384 tokens: the tiled format bit for bit, values against torch."""
    import autoresearch2_b200 as sf
    T = 16384
    x, W1, W2, b1, dout = _inputs(T, s, seed=7 + int(s * 100))
    out, z, snap, (dx, dW1, dW2, db1) = _run(x, W1, W2, b1, dout)
    assert sf.ffn.last_path() == path

    # the forward's format equals dense_to_tilesparse of its own z (128 x 128
    # tiles, the arena written from the same cursor)
    arena2 = torch.full_like(snap["arena"], 3.0)
    off2 = torch.full((1,), snap["vals_offset"], dtype=torch.int32, device=DEV)
    rp = sf.dense_to_tilesparse(z, arena2, off2, 128, 128)
    assert torch.equal(rp.bitmask, snap["bitmask"])
    assert torch.equal(rp.prefix, snap["prefix"])
    assert int(off2.item()) == snap["off"]
    assert torch.equal(arena2.view(torch.int16), snap["arena"].view(torch.int16))
    nnz = int(snap["prefix"][-1].item())
    assert abs(1 - nnz / (T * F) - s) < 0.02

    # z against torch: relu(bf16(x @ W1^T + b1)), mask flips only at zero crossings
    pre = (x.float() @ W1.float().T + b1.float()).to(torch.bfloat16).float()
    zr = torch.relu(pre)
    flips = (z > 0) != (zr > 0)
    assert int(flips.sum()) <= 1e-4 * T * F
    assert bool((pre[flips].abs() <= 2.0 ** -6).all())
    same = ~flips
    close(z.float()[same], zr[same], 2.0 ** -7, "z")

    # outputs and gradients against float32 products of the same bf16 operands,
    # with the device's own z (so that the mask is the one the backward used)
    zf = z.float()
    a = (zf * zf).to(torch.bfloat16).float()
    close(out, a @ W2.float().T, BF16_TOL, "out")
    dA = (dout.float() @ W2.float()).to(torch.bfloat16).float()
    dpre = ((dA * 2.0).to(torch.bfloat16).float() * zf).to(torch.bfloat16).float()
    del dA
    close(dx, dpre @ W1.float(), BF16_TOL, "dx")
    close(dW1, dpre.T @ x.float(), BF16_TOL, "dW1")
    close(db1, dpre.sum(0), BF16_TOL, "db1")
    del dpre
    close(dW2, dout.float().T @ a, BF16_TOL, "dW2")


def test_single_layer_cpu_config_fp32_on_gpu():
    """8192 tokens, d_model=768, d_ff=3072, float32, bias -1.3 (about 90%
    zeros): the configuration the CPU baseline times, on the GPU, against the
    float64 oracle at 1e-5."""
    import autoresearch2_b200 as sf
    T, Dm, Ff = 8192, 768, 3072
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, Dm, generator=g)
    W1 = torch.randn(Ff, Dm, generator=g) / Dm ** 0.5
    W2 = torch.randn(Dm, Ff, generator=g) / Ff ** 0.5
    dout = torch.randn(T, Dm, generator=g)
    b1 = torch.full((Ff,), -1.3)
    xg, W1g, W2g, b1g = (t.to(DEV).requires_grad_() for t in (x, W1, W2, b1))
    arena = torch.empty(T * Ff, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = sf.FFNSpRelu2.apply(xg, W1g, W2g, (arena, off), b1g)
    mask = (out.grad_fn.z_sparse.to_dense() > 0).cpu().numpy()
    out.backward(dout.to(DEV))
    assert 0.85 < 1 - mask.mean() < 0.95
    np_in = [t.numpy() for t in (x, W1, W2, dout, b1)]
    r0 = oracle.ffn_fwd_bwd(*np_in[:4], act="relu2", b1=np_in[4], code=oracle.F32)
    flips = mask != r0["mask"]
    assert np.all(np.abs(r0["pre"][flips]) <= 2.0 ** -14)
    r = oracle.ffn_fwd_bwd(*np_in[:4], act="relu2", b1=np_in[4], code=oracle.F32, mask=mask)
    close(out, r["out"], F32_TOL, "out")
    close(xg.grad, r["dx"], F32_TOL, "dx")
    close(W1g.grad, r["dW1"], F32_TOL, "dW1")
    close(W2g.grad, r["dW2"], F32_TOL, "dW2")
    close(b1g.grad, r["db1"], F32_TOL, "db1")
    assert int(off.item()) == int(mask.sum())
