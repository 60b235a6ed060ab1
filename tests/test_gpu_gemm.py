"""GPU tests of the tcgen05 GEMM and the fused FFN epilogues.

GEMM numerics are checked against an fp32 torch product of the same bf16
operands (tolerance: 1e-2 relative to the largest |C|, bf16 output rounding
plus accumulation order).  The fused up-projection is checked for
self-consistency bit for bit: its bitmask, prefix and vals must equal what the
standalone packer produces from the z it wrote."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status_clean():
    import autoresearch2_b200 as sf
    yield
    sf.check_status()


def ref_mm(A, B):
    return (A.float() @ B.float())


def assert_close_rel(got, want, tol=1e-2):
    err = (got.float() - want).abs().max().item()
    scale = want.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


def rand(*shape, seed=0, scale=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, device=DEV, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (200, 296, 72), (1000, 776, 520),
                                   (2048, 2048, 4096), (136, 8, 8)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
def test_mm_layouts(M, N, K, a_t, b_t):
    from autoresearch2_b200 import gemm
    A = rand(K, M, seed=1).T if a_t else rand(M, K, seed=1)   # a_t: transposed view
    B = rand(N, K, seed=2).T if b_t else rand(K, N, seed=2)
    C = gemm.mm(A, B)
    assert_close_rel(C, ref_mm(A, B))


def test_mm_out_and_strided_output():
    from autoresearch2_b200 import gemm
    A, B = rand(256, 128, seed=3), rand(128, 256, seed=4)
    big = torch.zeros(256, 320, dtype=torch.bfloat16, device=DEV)
    out = big[:, :256]
    gemm.mm(A, B, out=out)
    assert_close_rel(out, ref_mm(A, B))
    assert torch.count_nonzero(big[:, 256:]) == 0


def test_mm_k_skip_lists():
    """Row tiles skip 64-wide K blocks that are zero in the whole tile."""
    from autoresearch2_b200 import gemm
    M, N, K = 768, 256, 512
    A = rand(M, K, seed=5)
    keep = torch.rand(M // 256, K // 64, generator=torch.Generator().manual_seed(0)) < 0.5
    keep[1] = False  # one 256-row tile with no live block at all
    mask = keep.repeat_interleave(256, 0).repeat_interleave(64, 1).to(DEV)
    A = torch.where(mask, A, torch.zeros((), dtype=A.dtype, device=DEV))
    B = rand(K, N, seed=6)
    kb_list = torch.zeros(M // 256, K // 64, dtype=torch.int32)
    kb_count = torch.zeros(M // 256, dtype=torch.int32)
    for m in range(M // 256):
        live = torch.nonzero(keep[m]).flatten()
        kb_list[m, :live.numel()] = live.int()
        kb_count[m] = live.numel()
    C = gemm.mm(A, B, kb_list=kb_list.to(DEV), kb_count=kb_count.to(DEV))
    assert_close_rel(C, ref_mm(A, B))
    assert torch.count_nonzero(C[256:512]) == 0


def test_live_kblocks_matches_mask():
    """Live lists from a bitmask equal the 64-column blocks with any nonzero
    in each 256-row tile (odd number of 128-row tiles included)."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    T, F = 384, 640
    z = torch.zeros(T, F, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    live = torch.rand(T // 128, F // 64, generator=g) < 0.3
    for tm in range(T // 128):
        for kb in range(F // 64):
            if live[tm, kb]:
                z[tm * 128 + 7, kb * 64 + 5] = 1.0
    arena = torch.empty(T * F, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(z, arena, off, 128, 128)
    kb_list, kb_count = gemm.live_kblocks(x.bitmask, T, F)
    for tp in range(2):
        want = torch.nonzero(live[2 * tp:2 * tp + 2].any(0)).flatten().int()
        n = int(kb_count[tp])
        assert n == want.numel()
        assert torch.equal(kb_list[tp, :n].cpu(), want)


@pytest.mark.parametrize("T,F", [(384, 640), (1024, 256), (256, 1152)])
def test_live_kblocks_transposed_lists(T, F):
    """Token-skip lists: per 256 activation columns, the 64-row blocks with
    any nonzero (odd numbers of 128-column tiles included)."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    z = torch.zeros(T, F, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(T + F)
    live = torch.rand(T // 64, F // 128, generator=g) < 0.3
    for kb in range(T // 64):
        for tn in range(F // 128):
            if live[kb, tn]:
                z[kb * 64 + 13, tn * 128 + 100] = 2.0
    arena = torch.empty(T * F, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = sf.dense_to_tilesparse(z, arena, off, 128, 128)
    kb_list, kb_count = gemm.live_kblocks_t(x.bitmask, T, F)
    for tp in range(-(-F // 256)):
        want = torch.nonzero(live[:, 2 * tp:2 * tp + 2].any(1)).flatten().int()
        n = int(kb_count[tp])
        assert n == want.numel()
        assert torch.equal(kb_list[tp, :n].cpu(), want)


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (640, 256, 1024), (2048, 1024, 4096)])
def test_transposed_store_gemm_with_token_lists(M, N, K):
    """(A @ B)^T stored by the epilogue, A = a^T for an activation a [K, M]
    whose zero 64-row blocks per 256 columns are skipped."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    dead = torch.rand(K // 128, -(-M // 128), device=DEV, generator=g) < 0.5
    keep = ~dead.repeat_interleave(128, 0).repeat_interleave(128, 1)[:K, :M]
    a = torch.where(keep & (torch.rand(K, M, device=DEV, generator=g) < 0.3),
                    torch.randn(K, M, device=DEV, generator=g), 0).to(torch.bfloat16)
    B = torch.randn(K, N, device=DEV, generator=g).to(torch.bfloat16)
    arena = torch.empty(K * M, device=DEV, dtype=torch.bfloat16)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    zs = sf.dense_to_tilesparse(a.abs(), arena, off, 128, 128)
    tl, tc = gemm.live_kblocks_t(zs.bitmask, K, M)
    want = (a.float().T @ B.float()).T
    for lists in ((None, None), (tl, tc)):
        got = gemm.mm_t(a.T, B, kb_list=lists[0], kb_count=lists[1])
        assert got.shape == (N, M)
        err = (got.float() - want).abs().max().item()
        assert err <= 2e-2 * want.abs().max().item() + 1e-3
    sf.check_status()


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("T,D,F,bias", [(256, 128, 384, True), (300, 72, 200, False),
                                        (1024, 512, 1536, True)])
def test_ffn_up_fused(act, T, D, F, bias):
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    x = rand(T, D, seed=7)
    W1 = rand(F, D, seed=8, scale=D ** -0.5)
    b1 = torch.full((F,), -0.7, device=DEV, dtype=torch.bfloat16) if bias else None
    arena = torch.full((T * F + 50,), 9.0, device=DEV, dtype=torch.bfloat16)
    offset = torch.tensor([17], dtype=torch.int32, device=DEV)
    a, bitmask, prefix, voff, _ = gemm.ffn_up(x, W1, b1, act, arena, offset)
    pre = x.float() @ W1.float().T + (b1.float() if bias else 0)
    z_ref = torch.relu(pre)
    # the device z: the kernel's own dense output (ReLU) or the unpacked values
    x_sp = sf.BitsparseTensor(arena, bitmask, prefix, voff, -(-T // 128), -(-F // 128), 128, 128, (T, F))
    z_dev = x_sp.to_dense()
    assert_close_rel(z_dev, z_ref, 1e-2)
    if act == 0:
        assert torch.equal(a, z_dev)
    else:
        assert torch.equal(a, (z_dev.float() * z_dev.float()).to(torch.bfloat16))
    # self-consistency: the standalone packer on z_dev gives the same format
    arena2 = torch.full_like(arena, 9.0)
    off2 = torch.tensor([17], dtype=torch.int32, device=DEV)
    y = sf.dense_to_tilesparse(z_dev, arena2, off2, 128, 128)
    assert torch.equal(y.bitmask, bitmask)
    assert torch.equal(y.prefix, prefix)
    assert torch.equal(arena2.view(torch.int16), arena.view(torch.int16))
    assert int(offset.item()) == int(off2.item()) == 17 + int((z_dev > 0).sum())
    assert int(voff.item()) == 17


@pytest.mark.parametrize("start", range(8))
def test_ffn_up_tile_copy_at_every_alignment(start):
    """The up-projection's tile-packed slots reach the arena by one copy per
    tile; the arena's start offset (0..7 values) sets how the copy's 16-byte
    stores straddle the slot's vectors.  Arena, row offsets and live columns
    must equal the standalone packer's (integer/byte work: exact), and nothing
    outside the written range may change."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    T, D, F = 640, 256, 896
    x = rand(T, D, seed=20 + start)
    W1 = rand(F, D, seed=30 + start, scale=D ** -0.5)
    b1 = torch.full((F,), -0.3 * (start % 4), device=DEV, dtype=torch.bfloat16)
    arena = torch.full((T * F + 64,), 9.0, device=DEV, dtype=torch.bfloat16)
    offset = torch.tensor([start], dtype=torch.int32, device=DEV)
    colmask = torch.empty(-(-T // 128) * -(-F // 128) * 4, dtype=torch.int32, device=DEV)
    a, bitmask, prefix, voff, ro = gemm.ffn_up(x, W1, b1, 1, arena, offset, colmask=colmask)
    zs = sf.BitsparseTensor(arena, bitmask, prefix, voff, -(-T // 128), -(-F // 128), 128, 128, (T, F))
    z_dev = zs.to_dense()
    arena2 = torch.full_like(arena, 9.0)
    off2 = torch.tensor([start], dtype=torch.int32, device=DEV)
    y = sf.dense_to_tilesparse(z_dev, arena2, off2, 128, 128)
    assert torch.equal(arena2.view(torch.int16), arena.view(torch.int16))
    assert torch.equal(ro, gemm.tile_row_offsets(y))
    assert torch.equal(colmask, gemm.tile_colmask(y))
    assert torch.equal(a, (z_dev.float() * z_dev.float()).to(torch.bfloat16))
    sf.check_status()


def test_ffn_up_arena_too_small_flags_and_stays_in_bounds():
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    T, D, F = 256, 128, 512
    x = rand(T, D, seed=41)
    W1 = rand(F, D, seed=42, scale=D ** -0.5)
    big = torch.full((T * F,), 9.0, device=DEV, dtype=torch.bfloat16)
    cap = 1000
    arena = big[:cap]
    offset = torch.tensor([3], dtype=torch.int32, device=DEV)
    gemm.ffn_up(x, W1, None, 1, arena, offset)
    assert sf.check_status(raise_on_error=False) & 1  # SFFN_STATUS_VALS_OVERFLOW
    assert bool((big[cap:] == 9.0).all())


@pytest.mark.parametrize("act", [0, 1])
def test_ffn_dgrad_fused(act):
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    T, D, F = 384, 256, 640
    x = rand(T, D, seed=9)
    W1 = rand(F, D, seed=10, scale=D ** -0.5)
    W2 = rand(D, F, seed=11, scale=F ** -0.5)
    dout = rand(T, D, seed=12)
    b1 = torch.full((F,), -0.5, device=DEV, dtype=torch.bfloat16)
    arena = torch.empty(T * F, device=DEV, dtype=torch.bfloat16)
    offset = torch.zeros(1, dtype=torch.int32, device=DEV)
    _, bitmask, prefix, voff, _ = gemm.ffn_up(x, W1, b1, act, arena, offset)
    zs = sf.BitsparseTensor(arena, bitmask, prefix, voff, -(-T // 128), -(-F // 128), 128, 128, (T, F))
    db1 = torch.zeros(F, dtype=torch.float32, device=DEV)
    dpre, act2 = gemm.ffn_dgrad(dout, W2, act, zs, db1=db1)
    # fused bias gradient: column sums of the bf16 dpre, accumulated in fp32
    torch.testing.assert_close(db1, dpre.float().sum(0), rtol=1e-5, atol=1e-4)
    z = zs.to_dense().float()
    g = (dout.float() @ W2.float()).to(torch.bfloat16).float()
    if act == 1:
        want_d = (g * 2 * z)
        want_a = z * z
    else:
        want_d = torch.where(z > 0, g, torch.zeros_like(g))
        want_a = z
    assert_close_rel(dpre, want_d, 2e-2)
    assert torch.equal(act2, want_a.to(torch.bfloat16))
    # exact: elements off the mask are (signed) zero
    assert torch.count_nonzero(dpre[z == 0]) == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 768), (300, 200, 1000), (8192, 768, 3072), (3072, 768, 8192)])
@pytest.mark.parametrize("trans", ["nn", "nt", "tn"])
def test_split_bf16_float32_product(M, N, K, trans):
    """float32 products on the tcgen05 GEMM as split-bf16 (three pieces per
    operand, six cross products, fp32 accumulation): within 1e-5 of the float64
    product (elementwise, absolute floor 1e-5 x max |ref|), for row-major and
    transposed views, K not a multiple of 64 included."""
    from autoresearch2_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    A = torch.randn(M, K, device=DEV, generator=g) if trans[0] == "n" else \
        torch.randn(K, M, device=DEV, generator=g).T
    B = torch.randn(K, N, device=DEV, generator=g) / K ** 0.5 if trans[1] == "n" else \
        (torch.randn(N, K, device=DEV, generator=g) / K ** 0.5).T
    got = gemm.matmul(A, B)
    want = A.double() @ B.double()
    assert got.dtype == torch.float32
    err = (got.double() - want).abs()
    assert bool((err <= 1e-5 * want.abs() + 1e-5 * want.abs().max()).all()), err.max().item()


def test_split_bf16_float16_product():
    from autoresearch2_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(5)
    A = torch.randn(512, 384, device=DEV, generator=g).half()
    B = (torch.randn(384, 256, device=DEV, generator=g) / 20).half()
    got = gemm.matmul(A, B)
    want = (A.double() @ B.double()).half().double()
    assert got.dtype == torch.float16
    err = (got.double() - want).abs()
    assert bool((err <= 1e-3 * want.abs() + 1e-3 * want.abs().max()).all())


@pytest.mark.parametrize("act", [0, 1])
def test_per_row_slots_route_matches_the_warp_packed_route(act):
    """sffn_ffn_up with slot_rows NULL writes per-row slots, which
    sffn_tile_gather_slots moves into the arena; with slot_rows given it
    writes warp-packed slots for sffn_tile_copy_slots.  Arena, mask, prefix
    and row offsets must be the same bits (integer/byte results)."""
    from autoresearch2_b200 import _lib, gemm
    from autoresearch2_b200._lib import ptr
    T, D, F = 384, 128, 640
    x = rand(T, D, seed=51)
    W1 = rand(F, D, seed=52, scale=D ** -0.5)
    b1 = torch.full((F,), -0.4, device=DEV, dtype=torch.bfloat16)
    arena = torch.full((T * F + 40,), 9.0, device=DEV, dtype=torch.bfloat16)
    offset = torch.tensor([5], dtype=torch.int32, device=DEV)
    a, bitmask, prefix, voff, ro = gemm.ffn_up(x, W1, b1, act, arena, offset)
    nt = -(-T // 128) * -(-F // 128)
    bm2 = torch.empty(nt * 2048, dtype=torch.uint8, device=DEV)
    counts = torch.empty(nt * 4, dtype=torch.int32, device=DEV)
    slots = torch.empty(nt * 16384, dtype=torch.bfloat16, device=DEV)
    act2 = torch.empty(T, F, dtype=torch.bfloat16, device=DEV)
    pf2 = torch.empty(nt + 1, dtype=torch.int32, device=DEV)
    vo2 = torch.empty(1, dtype=torch.int32, device=DEV)
    ro2 = torch.empty(nt * 128, dtype=torch.int32, device=DEV)
    arena2 = torch.full_like(arena, 9.0)
    off2 = torch.tensor([5], dtype=torch.int32, device=DEV)
    status = ptr(_lib.status_word(x.device))
    st = _lib.stream_ptr(x.device)
    _lib.call("sffn_ffn_up", ptr(x), D, ptr(W1), D, ptr(b1), T, D, F, act, ptr(act2), F, ptr(bm2), ptr(counts),
              ptr(slots), None, status, st)
    _lib.call("sffn_tile_scan_counts", ptr(counts), 4, nt, ptr(pf2), ptr(off2), ptr(vo2), status, st)
    _lib.call("sffn_tile_gather_slots", ptr(slots), ptr(bm2), ptr(pf2), ptr(vo2), nt, ptr(arena2),
              arena2.numel(), _lib.BF16, ptr(ro2), None, status, st)
    torch.cuda.synchronize()
    assert torch.equal(bm2, bitmask) and torch.equal(pf2, prefix) and torch.equal(ro2, ro)
    assert torch.equal(arena2.view(torch.int16), arena.view(torch.int16))
    assert torch.equal(act2.view(torch.int16), a.view(torch.int16))
    assert int(off2.item()) == int(offset.item())


@pytest.mark.parametrize("M,K,N", [(512, 128, 384), (1000, 256, 640), (130, 72, 200)])
def test_sparse_relu_Ax_fused_bf16(M, K, N):
    """tiled.sparse_relu_Ax (old/matmul_bitsparse/train.py:69-116) on bf16 with
    128x128 tiles runs the fused up-projection: its (vals, meta) must be the
    same bits as packing relu(x @ W1.T) from this library's plain GEMM (the
    same main loop and the same round-to-nearest of the accumulator), vals of
    exactly nnz elements, and the unpacked result within the bf16 bar of the
    float32 product."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    x = rand(M, K, seed=61)
    W1 = rand(N, K, seed=62, scale=K ** -0.5)
    vals, meta = sf.tiled.sparse_relu_Ax(W1, x)
    z = torch.relu(gemm.mm(x, W1.T))
    want_vals, want_meta = sf.tiled.dense_to_tilesparse(z)
    assert torch.equal(meta["bitmask"], want_meta["bitmask"]) and torch.equal(meta["prefix"], want_meta["prefix"])
    assert torch.equal(vals.view(torch.int16), want_vals.view(torch.int16))
    assert vals.untyped_storage().nbytes() == vals.numel() * 2
    y = sf.tiled.bitsparse_unpack(vals, meta, (M, N))
    assert_close_rel(y, torch.relu(x.float() @ W1.float().T), 1e-2)
    sf.check_status()


@pytest.mark.parametrize("dtype,BM,BN", [(torch.float32, 128, 128), (torch.bfloat16, 64, 64),
                                         (torch.float16, 128, 128)])
def test_sparse_relu_Ax_other_forms(dtype, BM, BN):
    """The unfused route: float32 with input_precision "ieee" (split-bf16
    product, float32 accuracy) and bf16 with 64x64 tiles; unpacked against
    the float32 product."""
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(63)
    M, K, N = 384, 96, 256
    x = torch.randn(M, K, device=DEV, generator=g).to(dtype)
    W1 = (torch.randn(N, K, device=DEV, generator=g) * K ** -0.5).to(dtype)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        vals, meta = sf.tiled.sparse_relu_Ax(W1, x, BLOCK_M=BM, BLOCK_N=BN, input_precision="ieee")
        assert vals.dtype == dtype and meta["BLOCK_M"] == BM
        y = sf.tiled.bitsparse_unpack(vals, meta, (M, N))
        want = torch.relu(x.float() @ W1.float().T)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    tol = 1e-5 if dtype == torch.float32 else 1e-3 if dtype == torch.float16 else 1e-2
    assert_close_rel(y, want, tol)
    sf.check_status()


def _tf32_bound(A, Bt):
    """|C - A @ Bt.T| for TF32 inputs (10 mantissa bits, rounded or
    truncated: relative error below 2^-10 each) and float32 accumulation over
    K terms, from float64 |A| @ |Bt|.T."""
    K = A.shape[1]
    return (2.0 ** -9 + K * 2.0 ** -23) * (A.double().abs() @ Bt.double().abs().T) + 1e-30


@pytest.mark.parametrize("M,K,N", [(384, 96, 256), (130, 70, 200), (700, 1000, 520), (256, 4096, 512)])
def test_matmul_tf32_within_the_tf32_bound(M, K, N):
    """gemm.matmul_tf32 (tcgen05 kind::tf32): ragged M / N, K not a multiple
    of the 32-element k-block (70 also not of 4: the operands are padded),
    several K blocks; within the TF32 error bound of the float64 product and
    clearly coarser than float32 (the inputs really are read as TF32);
    relu=True stores exactly max(C, 0) of the same product."""
    from autoresearch2_b200 import gemm
    g = torch.Generator(device=DEV).manual_seed(M + K + N)
    A = torch.randn(M, K, device=DEV, generator=g)
    Bt = torch.randn(N, K, device=DEV, generator=g) * K ** -0.5
    C = gemm.matmul_tf32(A, Bt)
    want = A.double() @ Bt.double().T
    assert ((C.double() - want).abs() <= _tf32_bound(A, Bt)).all()
    rel = ((C.double() - want).norm() / want.norm()).item()
    assert 1e-5 < rel < 2e-3, rel
    Cr = gemm.matmul_tf32(A, Bt, relu=True)
    assert torch.equal(Cr, torch.clamp_min(C, 0.0))
    from autoresearch2_b200 import _lib
    _lib.check_status()


def test_sparse_relu_Ax_float32_tf32_default():
    """float32 sparse_relu_Ax at the reference's default input_precision
    "tf32" (old/matmul_bitsparse/train.py:45-52): the TF32 GEMM with the ReLU
    in its epilogue and the tiled pack; the unpacked result within the TF32
    bound of relu of the float64 product (relu is 1-Lipschitz), only
    positive values stored, 64x64 tiles too; an unknown precision raises."""
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(64)
    M, K, N = 1000, 512, 640
    x = torch.randn(M, K, device=DEV, generator=g)
    W1 = torch.randn(N, K, device=DEV, generator=g) * K ** -0.5
    want = torch.relu(x.double() @ W1.double().T)
    for BM, BN in ((128, 128), (64, 64)):
        vals, meta = sf.tiled.sparse_relu_Ax(W1, x, BLOCK_M=BM, BLOCK_N=BN)
        assert vals.dtype == torch.float32 and (vals > 0).all()
        assert meta["BLOCK_M"] == BM and meta["BLOCK_N"] == BN
        y = sf.tiled.bitsparse_unpack(vals, meta, (M, N))
        assert ((y.double() - want).abs() <= _tf32_bound(x, W1)).all()
    with pytest.raises(ValueError):
        sf.tiled.sparse_relu_Ax(W1, x, input_precision="fp64")
    sf.check_status()


def test_mm_relu_equals_relu_of_the_product():
    """gemm.mm_relu (sffn_gemm_relu): the ReLU applied by the epilogue gives
    the values of relu(gemm.mm) in bf16 (rounding keeps the sign) and of
    relu(mm_f32acc) in float32, with and without K-block lists; the
    split-bf16 matmul(relu=True) gives relu of matmul (the ReLU after the
    last K chunk's sum)."""
    from autoresearch2_b200 import gemm
    M, K, N = 700, 320, 520
    A = rand(M, K, seed=71)
    B = rand(K, N, seed=72, scale=K ** -0.5)
    got = gemm.mm_relu(A, B)
    assert got.dtype == torch.bfloat16
    assert torch.equal(got.float(), torch.relu(gemm.mm(A, B).float()))
    C = torch.empty(M, N, dtype=torch.float32, device=DEV)
    gemm.mm_f32acc(A, B, C, False)
    assert torch.equal(gemm.mm_relu(A, B, out_dtype=torch.float32), torch.relu(C))
    # zero 64-wide K blocks in every 256-row tile, skipped through the lists
    Az = A.clone()
    Az[:, 64:192] = 0
    import autoresearch2_b200 as sf
    _, meta = sf.tiled.dense_to_tilesparse(Az)
    kl, kc = gemm.live_kblocks(meta["bitmask"], M, K)
    assert int(kc.max()) < -(-K // 64)
    assert torch.equal(gemm.mm_relu(Az, B, kb_list=kl, kb_count=kc).float(), torch.relu(gemm.mm(Az, B).float()))
    g = torch.Generator(device=DEV).manual_seed(73)
    A32 = torch.randn(300, 2100, device=DEV, generator=g)
    B32 = torch.randn(2100, 200, device=DEV, generator=g)
    assert torch.equal(gemm.matmul(A32, B32, relu=True), torch.relu(gemm.matmul(A32, B32)))
    sf.check_status()


def _relu_layer_input(M, K, seed, dtype):
    """relu of shifted xavier-like values, as the reference's two-layer
    harness draws its sparse operand (old/sparse_matmul/prepare.py:7-17)."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    A = torch.randn(M, K, device=DEV, generator=g) * (2.0 / (M + K)) ** 0.5
    return torch.relu(A + 0.1 * A.std()).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_relu_spAx_forms(dtype):
    """tiled.relu_spAx (old/full_matmul/train.py:140-184): relu(A @ W2.T) from
    the packed A.  bf16: the same values as relu of this library's plain GEMM
    on the unpacked A, in one batch and in 256-row batches; float32: within
    the TF32 bound with allow_tf32 and within 1e-5 without; float16 within
    its rounding of the float32 product."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    M, K, N = 1000, 512, 384
    A = _relu_layer_input(M, K, 74, dtype)
    g = torch.Generator(device=DEV).manual_seed(75)
    W2 = (torch.randn(N, K, device=DEV, generator=g) * K ** -0.5).to(dtype)
    vals, meta = sf.tiled.dense_to_tilesparse(A)
    want64 = torch.relu(A.double() @ W2.double().T)
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        if dtype == torch.bfloat16:
            y = sf.tiled.relu_spAx(vals, meta, W2)
            assert y.dtype == dtype and y.shape == (M, N)
            want = torch.relu(gemm.mm(A, W2.T).float())
            assert torch.equal(y.float(), want)
            assert torch.equal(sf.tiled.relu_spAx(vals, meta, W2, row_batch=256).float(), want)
        elif dtype == torch.float32:
            torch.backends.cuda.matmul.allow_tf32 = True
            y = sf.tiled.relu_spAx(vals, meta, W2)
            assert ((y.double() - want64).abs() <= _tf32_bound(A, W2)).all()
            torch.backends.cuda.matmul.allow_tf32 = False
            y = sf.tiled.relu_spAx(vals, meta, W2, row_batch=512)
            assert_close_rel(y, want64.float(), 1e-5)
        else:
            y = sf.tiled.relu_spAx(vals, meta, W2)
            assert y.dtype == dtype
            assert_close_rel(y.float(), want64.float(), 1e-3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    with pytest.raises(ValueError):
        sf.tiled.relu_spAx(vals, meta, W2[:, :-8])
    sf.check_status()


@pytest.mark.parametrize("dtype,tf32", [(torch.bfloat16, False), (torch.float16, False), (torch.float32, False),
                                        (torch.float32, True)])
def test_relu_sparse_Ax_forms(dtype, tf32):
    """tiled.relu_sparse_Ax (old/sparse_matmul/train.py:56-76): relu(A @ x) in
    float32 with both operands taken in `dtype`.  bf16 / float16: the exact
    products of the rounded operands summed in float32 (bound K * 2^-23 of
    |A| |x|); float32: 1e-5 of the float64 product, or the TF32 bound."""
    import autoresearch2_b200 as sf
    M, K, N = 640, 384, 1000
    A = _relu_layer_input(M, K, 76, torch.float32)
    g = torch.Generator(device=DEV).manual_seed(77)
    x = torch.randn(K, N, device=DEV, generator=g)
    vals, meta = sf.tiled.dense_to_tilesparse(A)
    y = sf.tiled.relu_sparse_Ax(vals, meta, x, dtype=dtype, tf32=tf32)
    assert y.dtype == torch.float32 and y.shape == (M, N)
    Ad, xd = A.to(dtype).double(), x.to(dtype).double()
    want = torch.relu(Ad @ xd)
    if dtype == torch.float32 and not tf32:
        assert_close_rel(y, want.float(), 1e-5)
    elif tf32:
        assert ((y.double() - want).abs() <= _tf32_bound(A, x.T)).all()
    else:
        assert ((y.double() - want).abs() <= K * 2.0 ** -23 * (Ad.abs() @ xd.abs()) + 1e-30).all()
    sf.check_status()


def test_sp_relu_Ax_follows_torch_tf32_setting():
    """tiled.sp_relu_Ax (old/full_matmul/train.py:21-76) takes F.linear's
    float32 precision from torch's global setting: with allow_tf32 its vals
    are the pack of the TF32 GEMM on operands rounded to nearest (cuBLAS's
    TF32 products), without it sparse_relu_Ax at "ieee"; sparse_relu_Ax at
    "tf32" keeps Triton's truncated operands."""
    import autoresearch2_b200 as sf
    g = torch.Generator(device=DEV).manual_seed(78)
    x = torch.randn(300, 256, device=DEV, generator=g)
    W1 = torch.randn(512, 256, device=DEV, generator=g) * 256 ** -0.5
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        from autoresearch2_b200 import gemm
        torch.backends.cuda.matmul.allow_tf32 = True
        v1, m1 = sf.tiled.sp_relu_Ax(W1, x)
        v2, m2 = sf.tiled.dense_to_tilesparse(gemm.matmul_tf32(x, W1, relu=True, round_inputs=True))
        assert torch.equal(v1, v2) and torch.equal(m1["bitmask"], m2["bitmask"])
        assert m1["shape"] == (300, 512)
        v3, _ = sf.tiled.sparse_relu_Ax(W1, x)
        v4, _ = sf.tiled.dense_to_tilesparse(gemm.matmul_tf32(x, W1, relu=True))
        assert torch.equal(v3, v4)
        torch.backends.cuda.matmul.allow_tf32 = False
        v1, m1 = sf.tiled.sp_relu_Ax(W1, x)
        v2, m2 = sf.tiled.sparse_relu_Ax(W1, x, input_precision="ieee")
        assert torch.equal(v1, v2) and torch.equal(m1["bitmask"], m2["bitmask"])
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    sf.check_status()


def _tf32_round_np(x):
    """Round-to-nearest TF32 (ties away from zero) of float32 values, on the
    bit patterns: half of the 13 dropped bits' weight added to the
    magnitude, those bits cleared; infinities and NaNs unchanged."""
    import numpy as np
    u = x.view(np.uint32).astype(np.uint64)
    special = (u & 0x7F800000) == 0x7F800000
    r = ((u + 0x1000) & 0xFFFFE000).astype(np.uint32)
    return np.where(special, x.view(np.uint32), r).view(np.float32)


def test_round_tf32_bits_and_fused_unpack_rounding():
    """sffn_round_tf32 against the bit formula on random values, exact ties
    (both signs), the largest finite value (rounds to infinity), subnormals,
    infinities and NaN; an unaligned view takes the scalar path and in-place
    rounding works; tile_unpack(round_tf32=True) equals rounding the plain
    unpack."""
    import numpy as np
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    rng = np.random.default_rng(79)
    x = (rng.standard_normal(100003) * 10.0 ** rng.integers(-30, 30, 100003)).astype(np.float32)
    specials = np.array([1.0 + 2.0 ** -11, -(1.0 + 2.0 ** -11), 1.0 + 3 * 2.0 ** -11, np.finfo(np.float32).max,
                         1e-40, -1e-42, np.inf, -np.inf, np.nan, 0.0, -0.0], dtype=np.float32)
    x[:specials.size] = specials
    want = _tf32_round_np(x)
    X = torch.from_numpy(x).to(DEV)
    got = gemm.round_tf32(X).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.isinf(got[3]) and got[0] == np.float32(1.0 + 2.0 ** -10) and got[2] == np.float32(1.0 + 2.0 ** -9)
    V = torch.empty(X.numel() + 3, device=DEV)[1:1 + X.numel()]  # 4-byte aligned only: the scalar path
    V.copy_(X)
    gemm.round_tf32(V, out=V)
    assert np.array_equal(V.cpu().numpy().view(np.uint32), want.view(np.uint32))
    A = _relu_layer_input(300, 520, 80, torch.float32)
    vals, meta = sf.tiled.dense_to_tilesparse(A)
    z = sf.tiled._as_bitsparse(vals, meta)
    plain = sf.bitsparse.tile_unpack(z)
    assert torch.equal(sf.bitsparse.tile_unpack(z, round_tf32=True), gemm.round_tf32(plain))
    sf.check_status()


def test_relu_spAx_float32_tf32_rounds_its_operands():
    """relu_spAx in float32 with TF32 allowed equals the kind::tf32 GEMM on
    operands rounded to the nearest TF32 values (cuBLAS's TF32 products)."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    M, K, N = 520, 384, 300
    A = _relu_layer_input(M, K, 81, torch.float32)
    g = torch.Generator(device=DEV).manual_seed(82)
    W2 = torch.randn(N, K, device=DEV, generator=g) * K ** -0.5
    vals, meta = sf.tiled.dense_to_tilesparse(A)
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = True
        y = sf.tiled.relu_spAx(vals, meta, W2)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert torch.equal(y, gemm.matmul_tf32(A, W2, relu=True, round_inputs=True))
    sf.check_status()


@pytest.mark.parametrize("BM,BN", [(64, 64), (128, 64)])
def test_relu_products_on_other_tile_shapes(BM, BN):
    """relu_spAx (bf16, no K-block lists off 128x128 tiles) and relu_sparse_Ax
    (bf16 default) from (vals, meta) packed with BM x BN tiles: the values of
    relu of this library's GEMM on the unpacked operand."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    M, K, N = 390, 200, 264
    A = _relu_layer_input(M, K, 83, torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(84)
    W2 = (torch.randn(N, K, device=DEV, generator=g) * K ** -0.5).bfloat16()
    vals, meta = sf.tiled.dense_to_tilesparse(A, BM, BN)
    assert torch.equal(sf.tiled.relu_spAx(vals, meta, W2).float(), torch.relu(gemm.mm(A, W2.T).float()))
    x = torch.randn(K, N, device=DEV, generator=g)
    y = sf.tiled.relu_sparse_Ax(vals.float(), meta, x)
    C = torch.empty(M, N, dtype=torch.float32, device=DEV)
    gemm.mm_f32acc(A, x.bfloat16(), C, False)
    assert torch.equal(y, torch.relu(C))
    sf.check_status()


def _fixture(name):
    from conftest import golden
    return golden(name)


@pytest.mark.parametrize("name", ["products_sparse_relu_Ax_f32", "products_full_matmul_f32"])
def test_relu_Ax_against_the_reference_fixture(name):
    """sparse_relu_Ax / sp_relu_Ax at float32 accuracy ("ieee"; TF32 off) on the
    inputs of the reference's own run (tests/golden): mask and prefix the
    reference's bit for bit (no product lies within 4e-6 of the largest of
    zero there), values within 1e-5 of the largest."""
    import autoresearch2_b200 as sf
    g = _fixture(name)
    x, W1 = torch.from_numpy(g["x"]).to(DEV), torch.from_numpy(g["W1"]).to(DEV)
    prev = torch.backends.cuda.matmul.allow_tf32
    try:
        torch.backends.cuda.matmul.allow_tf32 = False
        if name.endswith("full_matmul_f32"):
            vals, meta = sf.tiled.sp_relu_Ax(W1, x)
        else:
            vals, meta = sf.tiled.sparse_relu_Ax(W1, x, input_precision="ieee")
        assert torch.equal(meta["bitmask"].cpu(), torch.from_numpy(g["bitmask"]))
        assert torch.equal(meta["prefix"].cpu(), torch.from_numpy(g["prefix"]))
        want = torch.from_numpy(g["vals"])
        assert float((vals.cpu() - want).abs().max()) <= 1e-5 * float(want.abs().max())
        if name.endswith("full_matmul_f32"):
            # layer 2 from the reference's own layer-1 values
            W2 = torch.from_numpy(g["W2"]).to(DEV)
            y = sf.tiled.relu_spAx(torch.from_numpy(g["vals"]).to(DEV),
                                   {"bitmask": torch.from_numpy(g["bitmask"]).to(DEV),
                                    "prefix": torch.from_numpy(g["prefix"]).to(DEV), "grid_m": 1,
                                    "grid_n": 2, "BLOCK_M": 128, "BLOCK_N": 128, "shape": (128, 256)}, W2)
            yw = torch.from_numpy(g["y"])
            assert float((y.cpu() - yw).abs().max()) <= 1e-5 * float(yw.abs().max())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    sf.check_status()


def test_relu_sparse_Ax_against_the_reference_fixture():
    """relu_sparse_Ax at float32 ("ieee") on the reference's packed A and x
    (tests/golden): within 1e-5 of the largest output of its run."""
    import autoresearch2_b200 as sf
    g = _fixture("products_relu_sparse_Ax_f32")
    meta = {"bitmask": torch.from_numpy(g["bitmask"]).to(DEV), "prefix": torch.from_numpy(g["prefix"]).to(DEV),
            "grid_m": 2, "grid_n": 1, "BLOCK_M": 128, "BLOCK_N": 128, "shape": [256, 128]}
    y = sf.tiled.relu_sparse_Ax(torch.from_numpy(g["vals"]).to(DEV), meta, torch.from_numpy(g["x"]).to(DEV),
                                dtype=torch.float32)
    yw = torch.from_numpy(g["y"])
    assert y.dtype == torch.float32 and float((y.cpu() - yw).abs().max()) <= 1e-5 * float(yw.abs().max())
    sf.check_status()
