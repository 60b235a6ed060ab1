"""GPU checks of the compacted-K (bitmask-sparse) down-projection.

Each 128-row tile of tokens contracts over its live columns only: the
activation's columns holding a non-zero in any row of the tile, compacted,
times the rows of W2^T (W1 for dX) gathered at the same column indices.
The reference computes the dense product z @ W2.T (old/lib_sparse/sparse.py:
75,118) or unpacks and multiplies (spAx, sparse.py:305-351); the compacted
product must equal it within the bf16 bar.

Lists, the gather from the packed form and the in-place row compaction are
integer/byte work and must be exact; products are compared with float32
torch products of the same bf16 operands (elementwise 2e-2 with an absolute
floor of 2e-2 x max |ref|)."""
import os
import sys

import numpy as np
import pytest
import torch

import oracle
from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402  (the clustered-activation generator of the benchmark)

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


def close(got, want, tol=TOL, what=""):
    got = got.detach().double()
    want = want.detach().double().to(got.device)
    floor = tol * want.abs().max().item()
    bad = (got - want).abs() > tol * want.abs() + floor
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} off, max |diff| {(got - want).abs().max().item():.3g}"


@pytest.fixture(autouse=True)
def _status_and_mode():
    import autoresearch2_b200 as sf
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    prev = sf.compact_k()
    yield
    sf.set_compact_k(prev)
    torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    sf.check_status()


def _pack(z):
    import autoresearch2_b200 as sf
    T, F = z.shape
    arena = torch.empty(T * F, dtype=z.dtype, device=DEV)
    off = torch.zeros(1, dtype=torch.int32, device=DEV)
    return sf.dense_to_tilesparse(z, arena, off, 128, 128)


def _lists_reference(z):
    """Per 128-row tile: the ascending live columns, as numpy arrays."""
    live = (z.view(z.shape[0] // 128, 128, z.shape[1]) != 0).any(dim=1).cpu().numpy()
    return [np.nonzero(r)[0] for r in live]


@pytest.mark.parametrize("T,F,kind", [(256, 1024, "clustered"), (512, 768, "iid99"), (128, 256, "empty"),
                                      (384, 512, "full")])
def test_lists_and_gather_are_exact(T, F, kind):
    from autoresearch2_b200 import gemm as G
    if kind == "clustered":
        z = bench.clustered_activation(T, F, DEV, seed=3)
    else:
        g = torch.Generator(device=DEV).manual_seed(T + F)
        p = {"iid99": 0.01, "empty": 0.0, "full": 1.0}[kind]
        keep = torch.rand(T, F, device=DEV, generator=g) < p
        z = torch.where(keep, torch.rand(T, F, device=DEV, generator=g) + 0.01, 0).to(torch.bfloat16)
    zs = _pack(z)
    colmask = G.tile_colmask(zs)
    idx, kcount, colpref = G.ck_lists(colmask, T, F)
    _, kc2, _ = G.ck_lists(colmask, T, F, counts_only=True)
    want = _lists_reference(z)
    kc, ix = kcount.cpu().numpy(), idx.cpu().numpy()
    assert np.array_equal(kc, kc2.cpu().numpy())
    zn = z.float().cpu().numpy()
    for tm, cols in enumerate(want):
        assert kc[tm] == cols.size
        assert np.array_equal(ix[tm, :cols.size], cols)
        kp = -(-cols.size // 64) * 64
        pad = ix[tm, cols.size:kp]
        # the padding column is zero in every row of the tile
        assert np.all((pad >= 0) & (pad < F))
        assert not np.any(zn[tm * 128:(tm + 1) * 128][:, pad])
    # the compacted activation from the packed form, ReLU^2 and ReLU
    ro = G.tile_row_offsets(zs)
    a2 = (z.float() * z.float()).to(torch.bfloat16)
    for act, dense in ((1, a2), (0, z)):
        ac = G.ck_gather_packed(zs, ro, colmask, colpref, kcount, act).cpu()
        dn = dense.cpu()
        for tm, cols in enumerate(want):
            kp = -(-cols.size // 64) * 64
            rows = dn[tm * 128:(tm + 1) * 128]
            assert torch.equal(ac[tm * 128:(tm + 1) * 128, :cols.size].view(torch.int16),
                               rows[:, torch.from_numpy(cols).long()].view(torch.int16))
            assert not bool(ac[tm * 128:(tm + 1) * 128, cols.size:kp].float().abs().sum())
    # in-place compaction of a dense matrix whose zeros follow z's
    x = torch.where(z != 0, torch.randn(T, F, device=DEV), 0).to(torch.bfloat16)
    xc = G.ck_compact_rows_(x.clone(), idx, kcount).cpu()
    xn = x.cpu()
    for tm, cols in enumerate(want):
        kp = -(-cols.size // 64) * 64
        rows = slice(tm * 128, (tm + 1) * 128)
        if cols.size == F:  # identity list: rows untouched
            assert torch.equal(xc[rows], xn[rows])
            continue
        assert torch.equal(xc[rows, :cols.size].view(torch.int16),
                           xn[rows][:, torch.from_numpy(cols).long()].view(torch.int16))
        assert not bool(xc[rows, cols.size:kp].float().abs().sum())


@pytest.mark.parametrize("T,F,N", [(256, 1024, 256), (1024, 4096, 1024), (384, 512, 512)])
def test_compacted_gemm_matches_the_dense_product(T, F, N):
    """C = per tile ac[:, :Kp] @ B[idx[:Kp]] equals act(z) @ B, dense."""
    from autoresearch2_b200 import gemm as G
    z = bench.clustered_activation(T, F, DEV, seed=T + N)
    zs = _pack(z)
    colmask = G.tile_colmask(zs)
    idx, kcount, colpref = G.ck_lists(colmask, T, F)
    ac = G.ck_gather_packed(zs, G.tile_row_offsets(zs), colmask, colpref, kcount, 1)
    g = torch.Generator(device=DEV).manual_seed(5)
    B = (torch.randn(F, N, device=DEV, generator=g) / F ** 0.5).to(torch.bfloat16)
    out = G.ck_mm(ac, B, idx, kcount)
    a = (z.float() * z.float()).to(torch.bfloat16).float()
    close(out, a @ B.float(), what="ck_mm")
    # two calls in a row give the same bits (no state kept between calls)
    assert torch.equal(out, G.ck_mm(ac, B, idx, kcount))


@pytest.mark.parametrize("T,D,F", [(512, 256, 1024), (1024, 512, 2048)])
@pytest.mark.parametrize("act", ["relu", "relu2"])
def test_ffn_compacted_path_against_oracle(T, D, F, act):
    """FFNSparse / FFNSpRelu2 with the compacted-K products forced on: outputs
    and gradients against the float64 oracle, driven by the device mask."""
    import autoresearch2_b200 as sf
    sf.set_compact_k("on")
    prev_mma = sf.sparse_mma()
    sf.set_sparse_mma("off")
    try:
        g = torch.Generator().manual_seed(T + D + F)
        x = torch.randn(T, D, generator=g)
        W1 = torch.randn(F, D, generator=g) / D ** 0.5
        W2 = torch.randn(D, F, generator=g) / F ** 0.5
        b1 = torch.full((F,), -2.0)
        dout = torch.randn(T, D, generator=g)
        cast = [t.to(torch.bfloat16) for t in (x, W1, W2, b1, dout)]
        xg, W1g, W2g, b1g = (t.to(DEV).requires_grad_() for t in cast[:4])
        fn = sf.FFNSparse if act == "relu" else sf.FFNSpRelu2
        out = fn.apply(xg, W1g, W2g, None, b1g)
        assert sf.ffn.last_path() == "ck"
        mask = (out.grad_fn.z_sparse.to_dense() > 0).cpu().numpy()
        out.backward(cast[4].to(DEV))
    finally:
        sf.set_sparse_mma(prev_mma)
    bits = [oracle.f32_to_bf16(t.float().numpy()) for t in cast]
    r = oracle.ffn_fwd_bwd(bits[0], bits[1], bits[2], bits[4], act=act, b1=bits[3], code=oracle.BF16, mask=mask)
    for got, key in ((out, "out"), (xg.grad, "dx"), (W1g.grad, "dW1"), (W2g.grad, "dW2"), (b1g.grad, "db1")):
        close(got, torch.from_numpy(np.asarray(r[key], dtype=np.float64)), what=key)


@pytest.mark.parametrize("mode", ["off", "on"])
def test_clustered_workload_reduced_tokens(mode):
    """The large-FFN workload's shapes (d_model=8192, d_ff=28672) at 1024
    tokens with the clustered activation injected: the down-projection and
    the backward from the packed z, against float32 torch products."""
    import autoresearch2_b200 as sf
    sf.set_compact_k(mode)
    T, D, F = 1024, 8192, 28672
    x, W1, W2, z, dout = bench.make_clustered_inputs(T, D, F, DEV, seed=1)
    zs = _pack(z)
    zf = z.float()
    a = (zf * zf).to(torch.bfloat16).float()
    dA = (dout.float() @ W2.float()).to(torch.bfloat16).float()
    dpre = ((dA * 2.0).to(torch.bfloat16).float() * zf).to(torch.bfloat16).float()
    del dA
    # the second step reads the live fraction the first observed: the weight
    # gradients then skip the zero token blocks
    for step in range(2):
        out = sf.ffn.down_proj(zs, W2)
        assert sf.ffn.last_path() == ("ck" if mode == "on" else "dense")
        gx, gW1, gW2 = sf.ffn.packed_backward(dout, x, W1, W2, zs)
        torch.cuda.synchronize()
        close(out, a @ W2.float().T, what=f"out {step}")
        close(gW2, dout.float().T @ a, what=f"dW2 {step}")
        close(gx, dpre @ W1.float(), what=f"dx {step}")
        close(gW1, dpre.T @ x.float(), what=f"dW1 {step}")
    assert sf.ffn._token_skip(T, D, F, W2)


@pytest.mark.parametrize("p_cluster,expect", [(0.9, "ck"), (0.5, "dense")])
def test_auto_mode_follows_the_live_fraction(p_cluster, expect):
    """Auto: the first call observes the live fraction without waiting; the
    next calls take the compacted path when at most CK_AUTO_MAX_LIVE of the
    (tile, column) pairs are live (about 10% are with 90% of the clusters
    zero; about half with 50%)."""
    import autoresearch2_b200 as sf
    sf.set_compact_k("auto")
    T, D, F = 512, 256, 1024
    _, _, W2, _, _ = bench.make_clustered_inputs(T, D, F, DEV, seed=2)
    z = bench.clustered_activation(T, F, DEV, seed=2, p_cluster=p_cluster)
    zs = _pack(z)
    paths, outs = [], []
    for _ in range(3):
        outs.append(sf.ffn.down_proj(zs, W2).float())
        paths.append(sf.ffn.last_path())
        torch.cuda.synchronize()
    assert paths[0] == "dense" and paths[-1] == expect, paths
    close(outs[-1], outs[0], what="auto")
