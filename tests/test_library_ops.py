"""CPU-side checks of the sparseffn:: torch.library ops: their schemas, their
fake kernels (the shapes torch.compile traces with, on fake CUDA tensors),
autograd through FFNSparse / FFNSpRelu2 on meta tensors, a torch.compile
trace with no graph break, and that a real call on CPU tensors still fails
(there is no CPU path).  The real kernels are compared with eager calls in
tests/test_gpu_library.py."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.symbolic_shapes import ShapeEnv

import autoresearch2_b200 as sf

ops = torch.ops.sparseffn


def fake_mode():
    return FakeTensorMode(shape_env=ShapeEnv())


def test_every_op_is_registered_with_its_mutations():
    for name in sf.library.OPS:
        schema = getattr(ops, name).default._schema
        written = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
        want = {"tile_pack": {"vals", "offset"}, "ffn_fwd": {"vals", "offset"}}.get(name, set())
        assert written == want, (name, written)


def test_flat_fake_kernels():
    with fake_mode():
        d = torch.empty(37, 53, device="cuda", dtype=torch.bfloat16)
        vals, mask = ops.bitsparse_pack(d)
        assert mask.shape == ((37 * 53 + 7) // 8,) and mask.dtype == torch.uint8
        assert vals.dtype == torch.bfloat16 and vals.dim() == 1
        assert not isinstance(vals.shape[0], int)  # nnz is data-dependent
        out = ops.bitsparse_unpack(vals, mask, [37, 53])
        assert out.shape == (37, 53) and out.dtype == torch.bfloat16 and out.is_cuda


def test_codec15_fake_kernels():
    with fake_mode():
        d = torch.empty(9, 37, device="cuda", dtype=torch.bfloat16)
        stream = ops.codec15_compress(d)
        nb = (9 * 37 * 15 + 7) // 8 + 8
        assert stream.shape == (nb + nb % 2,) and stream.dtype == torch.uint8
        out = ops.codec15_uncompress(stream, [9, 37], torch.float16)
        assert out.shape == (9, 37) and out.dtype == torch.float16 and out.is_cuda


@pytest.mark.parametrize("bm,bn", [(64, 64), (128, 128), (64, 128)])
def test_tile_fake_kernels(bm, bn):
    with fake_mode():
        d = torch.empty(130, 300, device="cuda", dtype=torch.float16)
        vals = torch.empty(130 * 300, device="cuda", dtype=torch.float16)
        off = torch.zeros(1, device="cuda", dtype=torch.int32)
        bitmask, prefix, voff = ops.tile_pack(d, vals, off, bm, bn)
        nt = -(-130 // bm) * -(-300 // bn)
        assert bitmask.shape == (nt * bm * bn // 8,) and bitmask.dtype == torch.uint8
        assert prefix.shape == (nt + 1,) and voff.shape == (1,) and prefix.dtype == torch.int32
        out = ops.tile_unpack(vals, bitmask, prefix, voff, [130, 300], bm, bn, True)
        assert out.shape == (130, 300) and out.dtype == torch.float16


def _ffn_inputs(dev, dtype, T, D, Fd, bias):
    x = torch.empty(T, D, device=dev, dtype=dtype, requires_grad=True)
    W1 = torch.empty(Fd, D, device=dev, dtype=dtype, requires_grad=True)
    W2 = torch.empty(D, Fd, device=dev, dtype=dtype, requires_grad=True)
    b1 = torch.empty(Fd, device=dev, dtype=dtype, requires_grad=True) if bias else None
    arena = (torch.empty(T * Fd, device=dev, dtype=dtype), torch.zeros(1, device=dev, dtype=torch.int32))
    return x, W1, W2, b1, arena


@pytest.mark.parametrize("dtype,fused", [(torch.bfloat16, True), (torch.float32, False)])
@pytest.mark.parametrize("fn", ["FFNSparse", "FFNSpRelu2"])
@pytest.mark.parametrize("bias", [False, True])
def test_ffn_fake_kernels(dtype, fused, fn, bias):
    """Forward through the autograd.Function, then the backward op on the
    state it kept (the autograd engine itself needs a real CUDA device)."""
    T, D, Fd = 384, 96, 520
    with fake_mode():
        x, W1, W2, b1, arena = _ffn_inputs("cuda", dtype, T, D, Fd, bias)
        out = getattr(sf, fn).apply(x, W1, W2, arena, b1)
        assert out.shape == (T, D) and out.dtype == dtype
        ctx = out.grad_fn
        z = ctx.z_sparse
        bm = 128 if fused else 64
        assert ctx.fused == fused and (z.BLOCK_M, z.BLOCK_N, z.shape) == (bm, bm, (T, Fd))
        assert z.vals is arena[0] and z.bitmask.numel() == -(-T // bm) * -(-Fd // bm) * bm * bm // 8
        row_offsets, kb_list, kb_count = ctx.aux
        if fused:
            assert row_offsets.shape == (z.bitmask.numel() // 2048 * 128,)
            assert kb_list.shape == (2, 9) and kb_count.shape == (2,)
        else:
            assert row_offsets.numel() == kb_list.numel() == kb_count.numel() == 0
        grads = ops.ffn_bwd(out.detach(), x.detach(), W1.detach(), W2.detach(), z.vals, z.bitmask,
                            z.prefix, z.vals_offset, row_offsets, kb_list, kb_count, fused, bias,
                            ctx.act)
        for g, t in zip(grads, (x, W1, W2)):
            assert g.shape == t.shape and g.dtype == dtype and g.is_contiguous()
        assert grads[3].shape == ((Fd,) if bias else (0,))


@pytest.mark.parametrize("fn", ["FFNSparse", "FFNSpRelu2"])
def test_ffn_autograd_on_meta_tensors(fn):
    """The autograd.Function classes drive ffn_fwd / ffn_bwd and release the
    sparse z after backward (meta tensors: the float32 64x64-tile path)."""
    x, W1, W2, b1, arena = _ffn_inputs("meta", torch.float32, 200, 64, 136, True)
    out = getattr(sf, fn).apply(x, W1, W2, arena, b1)
    ctx = out.grad_fn
    assert ctx.z_sparse.BLOCK_M == 64 and not ctx.fused
    out.sum().backward()
    assert ctx.z_sparse is None
    for t in (x, W1, W2, b1):
        assert t.grad is not None and t.grad.shape == t.shape


def test_compile_traces_the_ffn_without_a_graph_break():
    """A two-layer FFN (ReLU^2 then ReLU) over one shared arena compiles with
    fullgraph=True; the forward graph holds two ffn_fwd, the backward graph
    two ffn_bwd.  Meta tensors run the ops' fake kernels, so the compiled
    step (and its backward) runs here without a device."""
    from torch._dynamo.backends.common import aot_autograd

    graphs = []

    def record(gm, example_inputs):
        graphs.append(gm.code)
        return gm

    def two_layers(x, W1, W2, W3, W4, vals, off):
        h = sf.FFNSpRelu2.apply(x, W1, W2, (vals, off))
        return sf.FFNSparse.apply(h, W3, W4, (vals, off)).float().square().sum()

    torch._dynamo.reset()
    f = torch.compile(two_layers, backend=aot_autograd(fw_compiler=record, bw_compiler=record),
                      fullgraph=True)
    shapes = [(64, 32), (96, 32), (32, 96), (80, 32), (32, 80)]
    args = [torch.empty(*s, device="meta", requires_grad=i > 0) for i, s in enumerate(shapes)]
    vals = torch.empty(64 * 96 * 2, device="meta")
    off = torch.zeros(1, device="meta", dtype=torch.int32)
    f(*args, vals, off).backward()
    assert len(graphs) == 2, "forward and backward graphs"
    fw, bw = graphs
    assert fw.count("sparseffn.ffn_fwd") == 2 and "sparseffn.ffn_bwd" not in fw
    assert bw.count("sparseffn.ffn_bwd") == 2
    assert all(a.grad is not None and a.grad.shape == a.shape for a in args[1:])
    torch._dynamo.reset()


def test_real_kernels_refuse_cpu_tensors():
    """The ops' real kernels are the CUDA library: no CPU path."""
    d = torch.ones(8, 8)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        ops.bitsparse_pack(d)
    x, W1, W2 = torch.randn(64, 32), torch.randn(96, 32), torch.randn(32, 96)
    with pytest.raises(ValueError, match="CUDA tensors only"):
        sf.FFNSpRelu2.apply(x, W1, W2, None)
