"""Generate golden input/output vectors by running the reference's own code.

The reference (Maccy-Z/autoresearch2) is Python + Triton.  Its kernels run on
the CPU under Triton's interpreter (``TRITON_INTERPRET=1``), so this script
imports the reference modules from the checkout named by ``--ref`` (required),
calls its public functions and raw kernels on small,
seeded inputs, and stores inputs and outputs as ``.npz`` files next to this
script.  The fixtures are committed; nothing at test time reads the reference.

Shims needed to import the reference unmodified (none of them changes its
arithmetic):
  * ``cprint`` (``requirements.txt:1``) is not installed -> stub module.
  * ``old/lib_sparse/sparse.py:18`` annotates with ``Tensor`` imported only
    under ``TYPE_CHECKING`` -> ``builtins.Tensor = torch.Tensor``.
  * ``old/lib_sparse/sparse.py:202`` hard-codes ``device="cuda"`` -> the
    ``device`` keyword of ``torch.tensor`` is dropped during that call.
  * ``old/sparse_unpack.py:63`` asserts ``is_cuda`` -> its three kernels are
    launched directly in the order ``bitsparse_unpack`` launches them.
  * ``FFNSpRelu2.forward`` (``old/lib_sparse/sparse.py:120``) omits the vals
    arena arguments (TypeError in the reference) -> forward is re-run with the
    arena passed; ``backward`` is the reference's own.
  * ``triton.autotune`` benchmarks its configurations through a GPU driver ->
    the autotuned kernels of ``old/matmul_bitsparse/train.py`` and
    ``old/sparse_matmul/train.py`` keep their first configuration only (a
    single configuration is not benchmarked).
  * ``old/sparse_matmul/sparse_unpack.py:45,58`` assert ``is_cuda`` -> the
    ``bitsparse_unpack`` that ``relu_sparse_Ax`` calls launches its kernel the
    same way without the asserts.
  The (vals, meta) products use shapes whose sides are multiples of 128: the
  reference's 128x128 tile kernels bound rows only, and ragged columns wrote
  out of bounds under the interpreter.

Usage:  python tests/golden/make_golden.py --ref /path/to/reference
"""
import argparse
import builtins
import importlib
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    """Tensor -> numpy; bf16 is stored as its uint16 bit pattern."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def _import_ref(ref):
    sys.modules.setdefault("cprint", types.SimpleNamespace(c_print=lambda *a, **k: None))
    builtins.Tensor = torch.Tensor

    def load(subdir, name, alias):
        path = os.path.join(ref, subdir)
        sys.path.insert(0, path)
        for m in ("sparse_pack", "sparse_unpack", "sparse", "prepare_layer"):
            sys.modules.pop(m, None)
        mod = importlib.import_module(name)
        sys.modules[alias] = mod
        sys.path.remove(path)
        return mod

    mods = types.SimpleNamespace()
    mods.flat_pack = load("old", "sparse_pack", "ref_flat_pack")
    mods.flat_unpack = load("old", "sparse_unpack", "ref_flat_unpack")
    mods.fm_pack = load("old/full_matmul", "sparse_pack", "ref_fm_pack")
    mods.fm_unpack = load("old/full_matmul", "sparse_unpack", "ref_fm_unpack")
    # lib_sparse: sparse.py imports sparse_pack / sparse_unpack by bare name.
    path = os.path.join(ref, "old/lib_sparse")
    sys.path.insert(0, path)
    for m in ("sparse_pack", "sparse_unpack", "sparse", "prepare_layer"):
        sys.modules.pop(m, None)
    mods.lib_pack = importlib.import_module("sparse_pack")
    mods.lib_unpack = importlib.import_module("sparse_unpack")
    mods.lib = importlib.import_module("sparse")
    mods.layer = importlib.import_module("prepare_layer")
    sys.path.remove(path)
    return mods


class _NoCudaDevice:
    """Drops ``device=`` from torch.tensor inside dense_to_tilesparse (sparse.py:202)."""

    def __enter__(self):
        self.orig = torch.tensor

        def tensor(*a, **k):
            k.pop("device", None)
            return self.orig(*a, **k)

        torch.tensor = tensor

    def __exit__(self, *exc):
        torch.tensor = self.orig


def _flat_data(rows, cols, p, dtype, g, specials=True):
    """Data like old/bitpack/prepare.py:26-45 (mask ~ rand<p, values ~ randn,
    exact zeros replaced by 1e-8), plus -0.0 and negative entries."""
    n = rows * cols
    mask = torch.rand(n, generator=g) < p
    nz = torch.randn(int(mask.sum()), generator=g)
    nz = torch.where(nz == 0, torch.tensor(1e-8), nz)
    dense = torch.zeros(n)
    dense[mask] = nz
    if specials:
        zero_idx = torch.nonzero(~mask).flatten()
        if zero_idx.numel() > 4:
            dense[zero_idx[:3]] = -0.0  # -0.0 compares == 0 -> bit 0
    return dense.reshape(rows, cols).to(dtype)


def _ref_flat_unpack(mods, vals, packed_mask, shape, block=8192):
    """Launch old/sparse_unpack.py's three kernels exactly as its
    bitsparse_unpack (old/sparse_unpack.py:57-97) does, minus the is_cuda assert."""
    import triton
    m = mods.flat_unpack
    N = shape[0] * shape[1]
    n_blocks = triton.cdiv(N, block)
    block_counts = torch.empty(n_blocks, dtype=torch.int32)
    m._compute_block_counts_kernel[(n_blocks,)](packed_mask, block_counts, N=N,
                                                BYTE_BLOCK=triton.cdiv(block, 8))
    block_prefix = torch.empty(n_blocks, dtype=torch.int32)
    m._prefix_sum_kernel[(1,)](block_counts, block_prefix, n_blocks=n_blocks,
                               BLOCK_SCAN=triton.next_power_of_2(n_blocks))
    out = torch.empty(N, dtype=vals.dtype)
    m._reconstruct_packed_kernel[(n_blocks,)](vals, packed_mask, block_prefix, out,
                                             N=N, BLOCK=block, num_warps=8, num_stages=2)
    return out.reshape(shape)


def gen_flat(mods, out):
    g = torch.Generator().manual_seed(0)
    cases = [
        ("f32_37x53_p50", 37, 53, 0.5, torch.float32),
        ("f32_64x256_p10", 64, 256, 0.1, torch.float32),
        ("f16_33x100_p20", 33, 100, 0.2, torch.float16),
        ("bf16_48x96_p50", 48, 96, 0.5, torch.bfloat16),
        ("f32_7x9_p0", 7, 9, 0.0, torch.float32),
        ("f32_5x13_p100", 5, 13, 1.0, torch.float32),
    ]
    for name, r, c, p, dt in cases:
        dense = _flat_data(r, c, p, dt, g)
        vals, packed = mods.flat_pack.bitsparse_pack(dense, block=2048)
        vals_b, packed_b = mods.flat_pack.bitsparse_pack(dense, block=256)
        assert torch.equal(packed, packed_b) and torch.equal(vals, vals_b)
        recon = _ref_flat_unpack(mods, vals, packed, (r, c))
        out[f"flat_{name}"] = dict(dense=_np(dense), vals=_np(vals), packed_mask=_np(packed),
                                   unpacked=_np(recon), shape=np.array([r, c]))


def gen_tiled(mods, out):
    g = torch.Generator().manual_seed(1)
    lib = mods.lib
    # (name, M, N, BM, BN, dtype, start_offset)
    cases = [
        ("f32_130x192_64", 130, 192, 64, 64, torch.float32, 17),
        ("f32_96x64_32", 96, 64, 32, 32, torch.float32, 0),
        ("f16_64x128_64", 64, 128, 64, 64, torch.float16, 5),
        ("bf16_128x128_64", 128, 128, 64, 64, torch.bfloat16, 0),
        ("f32_70x100_64", 70, 100, 64, 64, torch.float32, 3),  # ragged N (pack only)
    ]
    for name, M, N, BM, BN, dt, off0 in cases:
        pre = torch.randn(M, N, generator=g) - 0.8
        pre.view(-1)[:5] = torch.tensor([-0.0, 0.0, 1e-30, -1e-30, 3.0])
        z = torch.relu(pre).to(dt)
        if name.startswith("f32_70"):
            z[0, 1] = -2.0  # negative entries are dropped by the tiled `> 0` test
        cap = M * N + off0 + 64
        vals = torch.full((cap,), -7.0, dtype=dt)
        offset = torch.tensor([off0], dtype=torch.int32)
        with _NoCudaDevice():
            bs = lib.dense_to_tilesparse(z, vals, offset, BLOCK_M=BM, BLOCK_N=BN)
        rec = dict(dense=_np(z), bitmask=_np(bs.bitmask), prefix=_np(bs.prefix),
                   vals_offset=_np(bs.vals_offset), offset_after=_np(offset),
                   vals=_np(vals), block=np.array([BM, BN]), shape=np.array([M, N]),
                   start_offset=np.array([off0]))
        if N % BN == 0:
            # unpack through spAx with an identity W (sparse.py:305-351) and a random W
            eye = torch.eye(M, dtype=dt)
            rec["unpacked"] = _np(lib.spAx(bs, eye))
            W = (torch.randn(9, M, generator=g) * 0.1).to(dt)
            rec["spAx_W"] = _np(W)
            rec["spAx"] = _np(lib.spAx(bs, W))
            rec["spAx_sq"] = _np(lib.spAx(bs, W, square=True))
        # K7: mask a gradient in place (sparse.py:96-102)
        grad = torch.randn(M, N, generator=g).to(dt)
        rec["grad"] = _np(grad)
        gm = grad.clone()
        lib._mask_with_bitmask_kernel[(bs.grid_m, bs.grid_n)](
            gm, bs.bitmask, M, N, BLOCK_M=BM, BLOCK_N=BN, TILE_BYTES=BM * BN // 8,
            num_warps=4, num_stages=2)
        rec["grad_masked"] = _np(gm)
        # K8: grad * 2z, vals squared in place (sparse.py:136-144).  Triton's
        # interpreter has no bf16 scalar constants (the `* 2.0`), so bf16 is skipped.
        if dt == torch.bfloat16:
            out[f"tiled_{name}"] = rec
            continue
        gr = grad.clone()
        vals2 = vals.clone()
        lib._grad_relu2_kernel[(bs.grid_m, bs.grid_n)](
            gr, vals2, bs.bitmask, bs.prefix, bs.vals_offset, M, N,
            BLOCK_M=BM, BLOCK_N=BN, TILE_NUMEL=BM * BN, TILE_BYTES=BM * BN // 8,
            num_warps=4, num_stages=2, square=True)
        rec["grad_relu2"] = _np(gr)
        rec["vals_squared"] = _np(vals2)
        out[f"tiled_{name}"] = rec

    # 128x128 (vals, meta) variant: old/full_matmul/sparse_pack.py:95-146 + sparse_unpack.py:44-73
    for name, M, N, dt in [("f32_200x300", 200, 300, torch.float32),
                           ("f16_256x128", 256, 128, torch.float16)]:
        z = torch.relu(torch.randn(M, N, generator=g) - 1.0).to(dt)
        vals, meta = mods.fm_pack.dense_to_tilesparse(z, 128, 128)
        # fm_unpack's bitsparse_unpack asserts is_cuda; launch its kernel the
        # way it does (old/full_matmul/sparse_unpack.py:60-72)
        outd = torch.empty(M, N, dtype=torch.float32)
        mods.fm_unpack._unpack_tiles_kernel[(meta["grid_m"], meta["grid_n"])](
            meta["bitmask"], vals, meta["prefix"], outd, meta["grid_n"], M, N,
            BLOCK_M=128, BLOCK_N=128, TILE_NUMEL=128 * 128, TILE_BYTES=128 * 128 // 8,
            num_warps=8, num_stages=2)
        out[f"tiled128_{name}"] = dict(dense=_np(z), vals=_np(vals), bitmask=_np(meta["bitmask"]),
                                       prefix=_np(meta["prefix"]), unpacked_f32=_np(outd),
                                       shape=np.array([M, N]))


def gen_ffn(mods, out):
    g = torch.Generator().manual_seed(2)
    lib, layer = mods.lib, mods.layer
    T, D, F = 128, 64, 192
    x = torch.randn(T, D, generator=g)
    W1 = torch.randn(F, D, generator=g) / D ** 0.5
    W2 = torch.randn(D, F, generator=g) / F ** 0.5
    dout = torch.randn(T, D, generator=g)
    torch.backends.cuda.matmul.allow_tf32 = False

    # FFNSparse (ReLU), sparse.py:56-109
    xs, W1s, W2s = (t.clone().requires_grad_() for t in (x, W1, W2))
    vals = torch.empty(T * F, dtype=torch.float32)
    off = torch.zeros(1, dtype=torch.int32)
    with _NoCudaDevice():
        o = lib.FFNSparse.apply(xs, W1s, W2s, (vals, off))
    o.backward(dout)
    # dense oracle FFNv3 (prepare_layer.py:117-162)
    xd, W1d, W2d = (t.clone().requires_grad_() for t in (x, W1, W2))
    od = layer.FFNv3.apply(xd, W1d, W2d)
    od.backward(dout)
    out["ffn_relu"] = dict(x=_np(x), W1=_np(W1), W2=_np(W2), dout=_np(dout),
                           out=_np(o), dx=_np(xs.grad), dW1=_np(W1s.grad), dW2=_np(W2s.grad),
                           out_dense=_np(od), dx_dense=_np(xd.grad), dW1_dense=_np(W1d.grad),
                           dW2_dense=_np(W2d.grad), nnz=_np(off))

    # FFNSpRelu2 (ReLU^2), sparse.py:112-151, forward re-run with the arena
    class FFNSpRelu2Arena(lib.FFNSpRelu2):
        @staticmethod
        def forward(ctx, x, W1, W2, sparse_data):
            vals, offset = sparse_data
            preact = x @ W1.T
            z = torch.nn.functional.relu(preact)
            output = (z * z) @ W2.T
            z_sparse = lib.dense_to_tilesparse(z, vals, offset)
            ctx.save_for_backward(x, W1, W2)
            ctx.z_sparse = z_sparse
            return output

        @staticmethod
        def backward(ctx, grad_output):
            return (*lib.FFNSpRelu2.backward(ctx, grad_output), None)

    xs, W1s, W2s = (t.clone().requires_grad_() for t in (x, W1, W2))
    vals = torch.empty(T * F, dtype=torch.float32)
    off = torch.zeros(1, dtype=torch.int32)
    with _NoCudaDevice():
        o = FFNSpRelu2Arena.apply(xs, W1s, W2s, (vals, off))
    o.backward(dout)
    xd, W1d, W2d = (t.clone().requires_grad_() for t in (x, W1, W2))
    od = layer.FFNrelu2.apply(xd, W1d, W2d)  # prepare_layer.py:12-29, torch autograd
    od.backward(dout)
    out["ffn_relu2"] = dict(x=_np(x), W1=_np(W1), W2=_np(W2), dout=_np(dout),
                            out=_np(o), dx=_np(xs.grad), dW1=_np(W1s.grad), dW2=_np(W2s.grad),
                            out_dense=_np(od), dx_dense=_np(xd.grad), dW1_dense=_np(W1d.grad),
                            dW2_dense=_np(W2d.grad), nnz=_np(off))


def _import_codec15(ref):
    """bitshifting/code.py, loaded by path (its module name would shadow the
    standard library's ``code``)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_codec15", os.path.join(ref, "bitshifting", "code.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gen_codec15(ref, out):
    """The 15-bit sign-strip codec (bitshifting/code.py:129-177).  Its kernels
    are autotuned, and the autotuner needs a driver, so each is launched
    through the autotuner's own function with one of its configurations
    (BLOCK_SIZE 256) and the grid its public function computes; the output
    buffer is the one compress_fn allocates, zero-filled so that its padding
    is defined.  Data as bitshifting/prepare.py:8-10 (|randn| bf16), plus raw
    16-bit patterns with the sign bit set, which the reference does not strip
    cleanly (its byte formula ORs the sign into the next value's bit 0)."""
    import math
    import triton
    m = _import_codec15(ref)
    g = torch.Generator().manual_seed(3)
    cases = [("bf16_n1", 1, "abs"), ("bf16_n7", 7, "abs"), ("bf16_n16", 16, "abs"),
             ("bf16_n17", 17, "abs"), ("bf16_n1000", 1000, "abs"), ("f16_n333", 333, "abs16"),
             ("raw_n2187", 2187, "raw")]
    for name, n, kind in cases:
        if kind == "raw":
            bits = torch.randint(0, 1 << 16, (n,), generator=g, dtype=torch.int32).to(torch.int16)
            bits = bits.view(torch.uint16)
        else:
            dt = torch.float16 if kind == "abs16" else torch.bfloat16
            bits = torch.randn(n, generator=g).to(dt).abs().view(torch.uint16)
        cb = (n * 15 + 7) // 8
        padded = cb + 8
        padded += padded & 1
        comp = torch.zeros(padded, dtype=torch.uint8)
        m._compress_15bit_kernel.fn[(triton.cdiv(cb, 256),)](bits, comp, n, cb, BLOCK_SIZE=256)
        restored = torch.empty(n, dtype=torch.uint16)
        m._uncompress_15bit_kernel.fn[(triton.cdiv(n, 256),)](comp.view(torch.uint16), restored, n, cb,
                                                              BLOCK_SIZE=256)
        out[f"codec15_{name}"] = dict(bits=bits.numpy(), compressed=comp[:cb].numpy(),
                                      restored=restored.numpy())
        assert math.prod(restored.shape) == n


def _load_train(ref, subdir):
    """train.py of one of the reference's (vals, meta) experiments, with the
    sparse_pack / sparse_unpack modules it imports by bare name."""
    path = os.path.join(ref, subdir)
    sys.path.insert(0, path)
    for m in ("train", "prepare", "sparse_pack", "sparse_unpack"):
        sys.modules.pop(m, None)
    mod = importlib.import_module("train")
    pack, unpack = sys.modules.get("sparse_pack"), sys.modules.get("sparse_unpack")
    sys.path.remove(path)
    return mod, pack, unpack


def gen_products(ref, out):
    """The (vals, meta) products, float32: sparse_relu_Ax
    (old/matmul_bitsparse/train.py:70-116), sp_relu_Ax + relu_spAx
    (old/full_matmul/train.py:21-184) and relu_sparse_Ax
    (old/sparse_matmul/train.py:56-76)."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(128, 64, generator=g)
    W1 = torch.randn(256, 64, generator=g) / 8.0 + 0.02
    W2 = torch.randn(32, 256, generator=g) / 16.0

    mb, _, _ = _load_train(ref, "old/matmul_bitsparse")
    mb._matmul_sparse_kernel.configs = mb._matmul_sparse_kernel.configs[:1]
    vals, meta = mb.sparse_relu_Ax(W1, x)
    out["products_sparse_relu_Ax_f32"] = dict(
        x=_np(x), W1=_np(W1), vals=_np(vals), bitmask=_np(meta["bitmask"]), prefix=_np(meta["prefix"]),
        grid=np.array([meta["grid_m"], meta["grid_n"]]))

    fm, _, _ = _load_train(ref, "old/full_matmul")
    vals, meta = fm.sp_relu_Ax(W1, x)
    y = fm.relu_spAx(vals, meta, W2)
    out["products_full_matmul_f32"] = dict(
        x=_np(x), W1=_np(W1), W2=_np(W2), vals=_np(vals), bitmask=_np(meta["bitmask"]),
        prefix=_np(meta["prefix"]), y=_np(y))

    sm, sm_pack, sm_unpack = _load_train(ref, "old/sparse_matmul")
    sm._matmul_relu_kernel.configs = sm._matmul_relu_kernel.configs[:1]

    def unpack(vals, meta, shape):  # sparse_matmul/sparse_unpack.py:44-73 without its is_cuda asserts
        outd = torch.empty(*shape, dtype=torch.float32)
        bm, bn = meta["BLOCK_M"], meta["BLOCK_N"]
        sm_unpack._unpack_tiles_kernel[(meta["grid_m"], meta["grid_n"])](
            meta["bitmask"], vals, meta["prefix"], outd, meta["grid_n"], shape[0], shape[1],
            BLOCK_M=bm, BLOCK_N=bn, TILE_NUMEL=bm * bn, TILE_BYTES=bm * bn // 8, num_warps=8, num_stages=2)
        return outd

    sm.bitsparse_unpack = unpack
    A = torch.relu(torch.randn(256, 128, generator=g) + 0.1)
    xs = torch.randn(128, 96, generator=g)
    vals, meta = sm_pack.dense_to_tilesparse(A)
    meta["shape"] = [256, 128]
    y = sm.relu_sparse_Ax(vals, meta, xs, dtype=torch.float32)
    out["products_relu_sparse_Ax_f32"] = dict(
        A=_np(A), x=_np(xs), vals=_np(vals), bitmask=_np(meta["bitmask"]), prefix=_np(meta["prefix"]),
        y=_np(y))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a checkout of the reference")
    ap.add_argument("--only", help="generate only the fixtures whose group starts with this "
                                   "(flat, tiled, ffn, codec15, products)")
    args = ap.parse_args()
    torch.manual_seed(0)
    mods = _import_ref(args.ref)
    out = {}
    want = lambda name: args.only is None or name.startswith(args.only)  # noqa: E731
    if want("flat"):
        gen_flat(mods, out)
    if want("tiled"):
        gen_tiled(mods, out)
    if want("ffn"):
        gen_ffn(mods, out)
    if want("codec15"):
        gen_codec15(args.ref, out)
    if want("products"):
        gen_products(args.ref, out)
    for name, rec in out.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(name, {k: v.shape for k, v in rec.items()})


if __name__ == "__main__":
    main()
