"""GPU checks of the sparseffn:: torch.library ops: torch.library.opcheck
(schema and mutations, fake kernels against the real outputs' metadata, AOT
dispatch), and torch.compile(fullgraph=True) runs that must give the eager
results -- bit for bit with the aot_eager backend where the kernels are
deterministic (the same kernels run in the same order), within the bf16
tolerance 2e-2 where they sum with atomics and with inductor (which rewrites
the loss's elementwise ops around the ops)."""
import pytest
import torch

import autoresearch2_b200 as sf

pytestmark = pytest.mark.gpu
DEV = "cuda"
ops = torch.ops.sparseffn


@pytest.fixture(autouse=True)
def _status():
    yield
    sf.set_sparse_mma("auto")
    torch._dynamo.reset()
    sf.check_status()


def sparse_dense(shape, p, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    v = torch.rand(shape, generator=g, device=DEV).add_(0.5)  # no zeros, no -0.0
    keep = torch.rand(shape, generator=g, device=DEV) < p
    return torch.where(keep, v, torch.zeros_like(v)).to(dtype)


def ffn_inputs(dtype, T, D, Fd, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(T, D, generator=g, device=DEV).to(dtype)
    W1 = (torch.randn(Fd, D, generator=g, device=DEV) * D ** -0.5).to(dtype)
    W2 = (torch.randn(D, Fd, generator=g, device=DEV) * Fd ** -0.5).to(dtype)
    b1 = torch.full((Fd,), -1.3, device=DEV).to(dtype)  # about 90% zeros
    return x, W1, W2, b1


def test_opcheck_flat_ops():
    d = sparse_dense((48, 96), 0.3, torch.bfloat16, 1)
    vals, mask = ops.bitsparse_pack(d)
    assert torch.equal(vals, d.flatten()[d.flatten() != 0])
    torch.library.opcheck(ops.bitsparse_pack.default, (d,), test_utils=("test_schema",))
    torch.library.opcheck(ops.bitsparse_unpack.default, (vals, mask, [48, 96]))


@pytest.mark.parametrize("bm,bn", [(64, 64), (128, 128)])
def test_opcheck_tile_ops(bm, bn):
    d = sparse_dense((200, 136), 0.2, torch.float16, 2)
    vals = torch.empty(4 * d.numel(), dtype=d.dtype, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.library.opcheck(ops.tile_pack.default, (d, vals, off, bm, bn),
                          test_utils=("test_schema", "test_faketensor"))
    off.zero_()
    bitmask, prefix, voff = ops.tile_pack(d, vals, off, bm, bn)
    assert torch.equal(ops.tile_unpack(vals, bitmask, prefix, voff, [200, 136], bm, bn, False), d)
    torch.library.opcheck(ops.tile_unpack.default, (vals, bitmask, prefix, voff, [200, 136], bm, bn, True))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("bias", [False, True])
def test_opcheck_ffn_ops(dtype, bias):
    T, D, Fd = 256, 128, 384
    x, W1, W2, b1 = ffn_inputs(dtype, T, D, Fd)
    b1 = b1 if bias else None
    vals = torch.empty(4 * T * Fd, dtype=dtype, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    utils = ("test_schema", "test_faketensor")
    torch.library.opcheck(ops.ffn_fwd.default, (x, W1, W2, b1, vals, off, 1), test_utils=utils)
    off.zero_()
    out, bitmask, prefix, voff, ro, kbl, kbc = ops.ffn_fwd(x, W1, W2, b1, vals, off, 1)
    fused = dtype == torch.bfloat16
    dout = torch.randn(T, D, device=DEV).to(dtype)
    args = (dout, x, W1, W2, vals, bitmask, prefix, voff, ro, kbl, kbc, fused, bias, 1)
    torch.library.opcheck(ops.ffn_bwd.default, args, test_utils=utils)


def two_layers(x, W1, W2, W3, W4, b1, vals, off):
    h = sf.FFNSpRelu2.apply(x, W1, W2, (vals, off), b1)
    return sf.FFNSparse.apply(h, W3, W4, (vals, off))


def run_step(fn, dtype, seed=0):
    T, D, Fd = 512, 256, 1024
    x, W1, W2, b1 = ffn_inputs(dtype, T, D, Fd, seed)
    _, W3, W4, _ = ffn_inputs(dtype, T, D, Fd, seed + 1)
    params = [t.requires_grad_() for t in (W1, W2, W3, W4, b1)]
    vals = torch.empty(2 * T * Fd, dtype=dtype, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = fn(x, W1, W2, W3, W4, b1, vals, off)
    out.float().square().sum().backward()
    return [out.detach(), off.clone()] + [p.grad for p in params]


def assert_close(got, want, tol):
    for g, w in zip(got, want):
        err = (g.float() - w.float()).abs().max().item()
        assert err <= tol * w.float().abs().max().item(), err


def test_compiled_two_layer_step_is_bitwise_eager():
    """Two FFN layers over one shared arena on the bf16 fused path with dense
    products.  All but the bias gradient must match bit for bit; that one is
    summed with fp32 atomics (one per 32 rows and column), whose order, and
    so its last bits, vary between runs."""
    sf.set_sparse_mma("off")
    want = run_step(two_layers, torch.bfloat16)
    got = run_step(torch.compile(two_layers, backend="aot_eager", fullgraph=True), torch.bfloat16)
    for g, w in zip(got[:-1], want[:-1]):
        assert torch.equal(g, w)
    assert_close(got[-1:], want[-1:], 2e-2)


def test_compiled_two_layer_step_sp24():
    """The same with the 2:4 products: their overflow entries are appended
    through per-row atomic cursors, so the fp32 order of the overflow sums,
    and the last bits of the results, vary between runs; the arena cursor
    does not."""
    sf.set_sparse_mma("on")
    want = run_step(two_layers, torch.bfloat16)
    got = run_step(torch.compile(two_layers, backend="aot_eager", fullgraph=True), torch.bfloat16)
    assert torch.equal(got[1], want[1])
    assert_close(got[:1] + got[2:], want[:1] + want[2:], 2e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_inductor_two_layer_step(dtype):
    sf.set_sparse_mma("off")
    want = run_step(two_layers, dtype)
    got = run_step(torch.compile(two_layers, fullgraph=True), dtype)
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])  # forward, arena cursor
    assert_close(got[2:], want[2:], 2e-2 if dtype == torch.bfloat16 else 1e-5)


def test_compiled_flat_round_trip():
    d = sparse_dense((300, 4096), 0.1, torch.bfloat16, 3)

    def round_trip(t):
        vals, mask = ops.bitsparse_pack(t)
        return ops.bitsparse_unpack(vals, mask, list(t.shape)), vals.numel()

    got, nnz = torch.compile(round_trip, backend="aot_eager", fullgraph=True)(d)
    assert torch.equal(got, d) and nnz == int((d != 0).sum())
