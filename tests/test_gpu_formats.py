"""GPU parity of the bitmask formats against the oracle and the reference's
golden vectors.  Masks, prefixes, vals and unpacked tensors are bit-exact."""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden, golden_names

pytestmark = pytest.mark.gpu

DEV = "cuda"


def to_t(a):
    """numpy (bf16 as uint16 bits) -> CUDA tensor."""
    if a.dtype == np.uint16:
        return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).to(DEV)
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def to_np(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    np.testing.assert_array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.fixture(autouse=True)
def _status_clean():
    import autoresearch2_b200 as sf
    yield
    sf.check_status()  # raises if any kernel flagged a device-side error


def flat_case(rows, cols, p, dtype, seed, specials=True):
    g = torch.Generator().manual_seed(seed)
    n = rows * cols
    mask = torch.rand(n, generator=g) < p
    vals = torch.randn(int(mask.sum()), generator=g).abs() + 1e-3
    d = torch.zeros(n)
    d[mask] = vals
    if specials and n > 16:
        d[0] = -0.0
        d[1] = float("nan")
        d[2] = -3.5
        d[n - 1] = 7.0
    return d.reshape(rows, cols).to(dtype)


# ------------------------------------------------------------------ flat ----
@pytest.mark.parametrize("name", golden_names("flat_"))
def test_flat_pack_unpack_golden(name):
    import autoresearch2_b200 as sf
    g = golden(name)
    dense = to_t(g["dense"])
    vals, mask = sf.bitsparse_pack(dense)
    bits_equal(to_np(mask), g["packed_mask"])
    bits_equal(to_np(vals), g["vals"])
    out = sf.bitsparse_unpack(to_t(g["vals"]), to_t(g["packed_mask"]), tuple(g["shape"]))
    bits_equal(to_np(out), g["unpacked"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols,p", [(1, 1, 1.0), (3, 7, 0.5), (1, 8191, 0.3), (2, 8192, 0.5),
                                          (257, 333, 0.1), (1024, 4099, 0.05), (64, 64, 0.0),
                                          (100, 100, 1.0), (4096, 4096, 0.2)])
def test_flat_against_oracle(dtype, rows, cols, p):
    import autoresearch2_b200 as sf
    d = flat_case(rows, cols, p, dtype, seed=rows * 7 + cols)
    vals, mask = sf.bitsparse_pack(d.to(DEV))
    ov, om = oracle.flat_pack(to_np(d))
    bits_equal(to_np(mask), om)
    bits_equal(to_np(vals), ov)
    out = sf.bitsparse_unpack(vals, mask, d.shape)
    bits_equal(to_np(out), oracle.flat_unpack(ov, om, d.shape))


@pytest.mark.parametrize("rows,cols,p", [(3, 7, 0.5), (257, 333, 0.1)])
def test_flat_under_its_earlier_names(rows, cols, p):
    """compress_dense / reconstruct_bitmask (old/bitpack/train.py:65,
    old/bitunpack/train.py:55) give the oracle's bits, the dense tensor
    passed flat with its shape as the reference's harness does."""
    import autoresearch2_b200 as sf
    d = flat_case(rows, cols, p, torch.bfloat16, seed=rows + cols)
    vals, mask = sf.compress_dense(d.to(DEV).flatten(), (rows, cols))
    ov, om = oracle.flat_pack(to_np(d))
    bits_equal(to_np(mask), om)
    bits_equal(to_np(vals), ov)
    out = sf.reconstruct_bitmask(vals, mask, (rows, cols))
    assert tuple(out.shape) == (rows, cols)
    bits_equal(to_np(out), oracle.flat_unpack(ov, om, d.shape))
    with pytest.raises(ValueError):
        sf.compress_dense(d.to(DEV), (rows, cols + 1))


def test_flat_empty():
    import autoresearch2_b200 as sf
    d = torch.zeros(0, 5, device=DEV, dtype=torch.bfloat16)
    vals, mask = sf.bitsparse_pack(d)
    assert vals.numel() == 0 and mask.numel() == 0
    assert sf.bitsparse_unpack(vals, mask, (0, 5)).shape == (0, 5)


@pytest.mark.parametrize("p", [0.5, 0.1, 0.01])
def test_flat_full_size_round_trip(p):
    """[65536, 4096] bf16 (the pack/unpack benchmark shape): pack -> unpack is
    the identity up to -0.0, nnz equals the count of nonzeros, and the mask
    popcount equals nnz."""
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(0)
    keep = torch.rand(65536, 4096, device=DEV, generator=g) < p
    d = torch.where(keep, torch.randn(65536, 4096, device=DEV, generator=g).abs() + 1e-3,
                    torch.zeros((), device=DEV)).to(torch.bfloat16)
    vals, mask = sf.bitsparse_pack(d)
    assert vals.numel() == int(keep.sum())
    pop = torch.bitwise_and(mask.view(-1, 1).int() >> torch.arange(8, device=DEV), 1).sum()
    assert int(pop) == vals.numel()
    assert torch.equal(sf.bitsparse_unpack(vals, mask, d.shape), d)
    # row-major order of values: compare with torch's boolean indexing
    assert torch.equal(vals, d.view(-1)[keep.view(-1)])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_flat_pack_sizes_vals_exactly_and_the_async_form(dtype):
    """bitsparse_pack returns a vals buffer of exactly nnz elements; the
    sync-free bitsparse_pack_async writes the same values into a caller's
    upper-bound buffer and leaves the count on the device; a bound below the
    count clips and flags SFFN_STATUS_VALS_OVERFLOW.  All against the oracle."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import _lib
    d = flat_case(300, 1111, 0.15, dtype, seed=17).to(DEV)
    ov, om = oracle.flat_pack(to_np(d))
    vals, mask = sf.bitsparse_pack(d)
    assert vals.numel() == len(ov) and vals.untyped_storage().nbytes() == len(ov) * d.element_size()
    bits_equal(to_np(vals), ov)
    bits_equal(to_np(mask), om)
    arena = torch.full((d.numel(),), 5, dtype=dtype, device=DEV)
    va, ma, nnz = sf.bitsparse_pack_async(d, arena)
    assert va is arena and int(nnz.item()) == len(ov)
    bits_equal(to_np(arena[:len(ov)]), ov)
    bits_equal(to_np(ma), om)
    assert bool((arena[len(ov):] == 5).all())
    small = torch.full((len(ov) // 2,), 5, dtype=dtype, device=DEV)
    sf.bitsparse_pack_async(d, small)
    assert _lib.check_status(DEV, raise_on_error=False) == 1  # SFFN_STATUS_VALS_OVERFLOW
    bits_equal(to_np(small), ov[:len(ov) // 2])


def _flat_capi(dtype, n, p, seed):
    from autoresearch2_b200 import _lib
    d = flat_case(1, n, p, dtype, seed=seed).view(-1)
    ov, om = oracle.flat_pack(to_np(d))
    L = _lib.load()
    ws = _lib.workspace(L.sffn_flat_pack_workspace_bytes(n, _lib.dtype_code(d)), DEV)
    return _lib, d.to(DEV), ov, om, ws


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_flat_capi_unaligned_vals_and_short_capacity(dtype):
    """Through the C ABI: `vals` 2 or 4 bytes past a 16-byte boundary (the
    element-wise write-out) gives the oracle's values; a capacity below nnz
    writes exactly the first `cap` values, nothing past them, sets
    SFFN_STATUS_VALS_OVERFLOW and still reports the full nnz."""
    n = 3 * 8192 + 13
    _lib, d, ov, om, ws = _flat_capi(dtype, n, 0.3, seed=41)
    code = _lib.dtype_code(d)
    nnz = len(ov)
    st = _lib.stream_ptr(DEV)
    status = _lib.status_word(DEV)
    mask = torch.empty((n + 7) // 8, dtype=torch.uint8, device=DEV)
    nnz_d = torch.zeros(1, dtype=torch.int64, device=DEV)
    buf = torch.full((nnz + 16,), 7, dtype=dtype, device=DEV)
    vals = buf[1:]  # one element past the allocation's (16-byte aligned) start
    _lib.call("sffn_flat_pack", _lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), nnz, _lib.ptr(nnz_d),
              _lib.ptr(ws), ws.numel(), _lib.ptr(status), st)
    assert _lib.check_status(DEV, raise_on_error=False) == 0
    bits_equal(to_np(mask), om)
    bits_equal(to_np(vals[:nnz]), ov)
    assert int(nnz_d.item()) == nnz
    cap = nnz // 2 + 3
    buf.fill_(7)
    _lib.call("sffn_flat_pack", _lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), cap, _lib.ptr(nnz_d),
              _lib.ptr(ws), ws.numel(), _lib.ptr(status), st)
    assert _lib.check_status(DEV, raise_on_error=False) == 1  # SFFN_STATUS_VALS_OVERFLOW
    bits_equal(to_np(vals[:cap]), ov[:cap])
    assert torch.all(vals[cap:] == 7) and float(buf[0]) == 7
    assert int(nnz_d.item()) == nnz


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_flat_capi_unpack_unaligned_and_short_vals(dtype):
    """Through the C ABI: unpack from `vals` off a 16-byte boundary with a mask
    only 4-byte aligned equals the oracle; with vals_len < nnz the elements
    whose values are missing come out as zero and SFFN_STATUS_VALS_SHORT is
    set."""
    n = 5 * 8192 + 77
    _lib, d, ov, om, ws = _flat_capi(dtype, n, 0.2, seed=43)
    code = _lib.dtype_code(d)
    nnz = len(ov)
    st = _lib.stream_ptr(DEV)
    status = _lib.status_word(DEV)
    vbuf = torch.zeros(nnz + 8, dtype=dtype, device=DEV)
    vals = vbuf[3:3 + nnz]
    vals.copy_(to_t(ov))
    mbuf = torch.zeros(len(om) + 16, dtype=torch.uint8, device=DEV)
    mask = mbuf[4:4 + len(om)]  # 4-byte but not 16-byte aligned
    mask.copy_(torch.from_numpy(om).to(DEV))
    out = torch.full((n,), 5, dtype=dtype, device=DEV)
    _lib.call("sffn_flat_unpack", _lib.ptr(vals), nnz, _lib.ptr(mask), code, n, _lib.ptr(out), _lib.ptr(ws),
              ws.numel(), _lib.ptr(status), st)
    assert _lib.check_status(DEV, raise_on_error=False) == 0
    want = oracle.flat_unpack(ov, om, (n,))
    bits_equal(to_np(out), want)
    short = nnz - 100
    _lib.call("sffn_flat_unpack", _lib.ptr(vals), short, _lib.ptr(mask), code, n, _lib.ptr(out), _lib.ptr(ws),
              ws.numel(), _lib.ptr(status), st)
    assert _lib.check_status(DEV, raise_on_error=False) == 8  # SFFN_STATUS_VALS_SHORT
    ov_short = ov.copy()
    ov_short[short:] = 0
    bits_equal(to_np(out), oracle.flat_unpack(ov_short, om, (n,)))


# ----------------------------------------------------------------- tiled ----
@pytest.mark.parametrize("name", golden_names("tiled_"))
def test_tile_pack_golden(name):
    import autoresearch2_b200 as sf
    g = golden(name)
    BM, BN = (int(v) for v in g["block"])
    off0 = int(g["start_offset"][0])
    arena = to_t(g["vals"]).clone()
    total = int(g["prefix"][-1])
    arena[off0:off0 + total] = 0
    offset = torch.tensor([off0], dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(to_t(g["dense"]), arena, offset, BM, BN)
    bits_equal(to_np(x.bitmask), g["bitmask"])
    bits_equal(to_np(x.prefix), g["prefix"])
    bits_equal(to_np(x.vals_offset), g["vals_offset"])
    bits_equal(to_np(offset), g["offset_after"])
    bits_equal(to_np(arena), g["vals"])  # untouched slots keep the fill value
    if "unpacked" in g:
        bits_equal(to_np(x.to_dense()), g["unpacked"])
    gm = to_t(g["grad"]).clone()
    sf.mask_with_bitmask_(gm, x)
    bits_equal(to_np(gm), g["grad_masked"])
    if "grad_relu2" in g:
        gr = to_t(g["grad"]).clone()
        sf.grad_relu2_(gr, x, square=True)
        bits_equal(to_np(gr), g["grad_relu2"])
        bits_equal(to_np(arena), g["vals_squared"])


@pytest.mark.parametrize("name", golden_names("tiled128_"))
def test_tile128_variant_golden(name):
    import autoresearch2_b200 as sf
    g = golden(name)
    vals, meta = sf.tiled.dense_to_tilesparse(to_t(g["dense"]))
    bits_equal(to_np(vals), g["vals"])
    # vals is its own allocation of exactly nnz values (no dense-size arena behind it)
    assert vals.untyped_storage().nbytes() == vals.numel() * vals.element_size()
    bits_equal(to_np(meta["bitmask"]), g["bitmask"])
    bits_equal(to_np(meta["prefix"]), g["prefix"])
    out = sf.tiled.bitsparse_unpack(to_t(g["vals"]), meta, tuple(g["shape"]))
    bits_equal(to_np(out), g["unpacked_f32"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("BM,BN", [(32, 32), (64, 64), (128, 128), (64, 128), (128, 64)])
@pytest.mark.parametrize("M,N", [(1, 32), (129, 200), (300, 1000), (512, 512)])
def test_tile_against_oracle(dtype, BM, BN, M, N):
    import autoresearch2_b200 as sf
    g = torch.Generator().manual_seed(M * 31 + N + BM)
    z = torch.relu(torch.randn(M, N, generator=g) - 1.0)
    z[0, 0] = -0.0
    z.view(-1)[min(5, M * N - 1)] = float("nan")
    z = z.to(dtype)
    zn = to_np(z)
    off0 = 11
    cap = M * N + off0 + 5
    arena = torch.full((cap,), 3.0, dtype=dtype, device=DEV)
    offset = torch.tensor([off0], dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(z.to(DEV), arena, offset, BM, BN)
    oarena = to_np(torch.full((cap,), 3.0, dtype=dtype))
    obm, opre, total = oracle.tile_pack(zn, BM, BN, oarena, off0)
    bits_equal(to_np(x.bitmask), obm)
    bits_equal(to_np(x.prefix), opre)
    bits_equal(to_np(arena), oarena)
    assert int(offset.item()) == off0 + total
    # unpack (whole, then a row range), squared unpack, float32 output
    bits_equal(to_np(x.to_dense()), oracle.tile_unpack(oarena, obm, opre, off0, (M, N), BM, BN))
    if M > BM:
        part = sf.tile_unpack(x, BM, M)
        bits_equal(to_np(part), oracle.tile_unpack(oarena, obm, opre, off0, (M, N), BM, BN, BM,
                                                   M - BM))
    code = oracle.dtype_code(zn)
    sq = oracle.tile_unpack(oarena, obm, opre, off0, (M, N), BM, BN)
    sqf = oracle.to_f64(sq, code)
    bits_equal(to_np(x.to_dense(square=True)), oracle.from_f64(sqf * sqf, code))
    if dtype != torch.float32:
        f32 = x.to_dense(dtype=torch.float32)
        np.testing.assert_array_equal(to_np(f32), oracle.to_f64(sq, code).astype(np.float32))
    # K7 and K8
    grad = torch.randn(M, N, generator=g).to(dtype)
    gm = grad.to(DEV)
    sf.mask_with_bitmask_(gm, x)
    bits_equal(to_np(gm), oracle.mask_with_bitmask(to_np(grad), obm, BM, BN))
    gr = grad.to(DEV)
    sf.grad_relu2_(gr, x, square=True)
    ogr, ovals = oracle.grad_relu2(to_np(grad), oarena, obm, opre, off0, BM, BN)
    bits_equal(to_np(gr), ogr)
    bits_equal(to_np(arena), ovals)


def test_arena_cursor_chains_layers():
    """Several packs into one arena (the per-layer use in
    old/lib_sparse/prepare.py:71-78): each layer starts where the previous ended."""
    import autoresearch2_b200 as sf
    buf = sf.TensorBuffer(4 * 256 * 384, DEV, torch.bfloat16).init_buffer()
    zs, xs = [], []
    for layer in range(4):
        z = torch.relu(torch.randn(256, 384, device=DEV) - 0.5 * layer).to(torch.bfloat16)
        zs.append(z)
        xs.append(sf.dense_to_tilesparse(z, buf.vals, buf.offset, 64, 64))
    counts = [int((z > 0).sum()) for z in zs]
    assert buf.used() == sum(counts)
    for layer, (z, x) in enumerate(zip(zs, xs)):
        assert int(x.vals_offset.item()) == sum(counts[:layer])
        assert torch.equal(x.to_dense(), torch.where(z > 0, z, torch.zeros_like(z)))
    buf.reset_buffer()
    assert buf.used() == 0


def test_arena_overflow_is_reported_and_clipped():
    import autoresearch2_b200 as sf
    z = torch.ones(128, 128, device=DEV, dtype=torch.bfloat16)
    arena = torch.zeros(1000 + 8, dtype=torch.bfloat16, device=DEV)
    guard = arena[1000:]
    offset = torch.zeros(1, dtype=torch.int32, device=DEV)
    sf.dense_to_tilesparse(z, arena[:1000], offset, 64, 64)
    with pytest.raises(sf._lib.SparseFFNError, match="capacity"):
        sf.check_status()
    assert torch.count_nonzero(guard) == 0  # nothing written past the capacity


def test_spAx_matches_oracle():
    import autoresearch2_b200 as sf
    g = torch.Generator().manual_seed(5)
    z = torch.relu(torch.randn(4096 + 64, 192, generator=g) - 0.5)
    W = torch.randn(48, 4096 + 64, generator=g) * 0.1
    arena = torch.empty(z.numel(), device=DEV)
    offset = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(z.to(DEV), arena, offset, 64, 64)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for square in (False, True):
            got = sf.spAx(x, W.to(DEV), square=square).cpu().double().numpy()
            want = (W.double() @ (z.double() ** (2 if square else 1))).numpy()
            np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(want).max())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("square", [False, True])
def test_spAx_bf16_batches_accumulate_in_fp32(square):
    """bf16 spAx over more rows than one batch (two full batches and a part):
    each batch's product is added into one float32 result by the GEMM's
    epilogue.  Against float64 of the same bf16 operands: the only rounding
    left is the final bf16 one (and the bf16 square of z), so 1e-2."""
    import autoresearch2_b200 as sf
    g = torch.Generator().manual_seed(6)
    M, N, K = 9000, 256, 72
    z = torch.relu(torch.randn(M, N, generator=g) - 1.0).to(torch.bfloat16)
    W = (torch.randn(K, M, generator=g) * 0.05).to(torch.bfloat16)
    arena = torch.empty(z.numel(), device=DEV, dtype=torch.bfloat16)
    offset = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(z.to(DEV), arena, offset, 64, 64)
    got = sf.spAx(x, W.to(DEV), square=square).double().cpu().numpy()
    zz = (z.float() * z.float()).to(torch.bfloat16) if square else z
    want = (W.double() @ zz.double()).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2 * np.abs(want).max())
