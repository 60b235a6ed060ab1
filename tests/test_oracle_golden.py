"""Pins the CPU oracle against golden vectors from the reference's own code.

The fixtures under tests/golden/ were produced by running the reference's
Triton kernels under Triton's CPU interpreter (tests/golden/make_golden.py).
Masks, prefixes and unpacked tensors must match bit for bit; the FFN
arithmetic within the stated tolerances.
"""
import numpy as np
import pytest

import oracle
from conftest import golden, golden_names


@pytest.mark.parametrize("name", golden_names("flat_"))
def test_flat_pack_matches_reference(name):
    g = golden(name)
    vals, mask = oracle.flat_pack(g["dense"])
    np.testing.assert_array_equal(mask, g["packed_mask"])
    np.testing.assert_array_equal(vals.view(np.uint8), g["vals"].view(np.uint8))
    # the golden packer of old/bitpack/prepare.py:6-23 agrees as well
    nz = oracle.to_f64(g["dense"], oracle.dtype_code(g["dense"])).ravel() != 0
    np.testing.assert_array_equal(oracle.pack_bool_mask(nz), g["packed_mask"])
    # multi-threaded split gives the same bytes
    vals4, mask4 = oracle.flat_pack(g["dense"], nthreads=4)
    np.testing.assert_array_equal(mask4, mask)
    np.testing.assert_array_equal(vals4.view(np.uint8), vals.view(np.uint8))


@pytest.mark.parametrize("name", golden_names("flat_"))
def test_flat_unpack_matches_reference(name):
    g = golden(name)
    out = oracle.flat_unpack(g["vals"], g["packed_mask"], tuple(g["shape"]))
    np.testing.assert_array_equal(out.view(np.uint8), g["unpacked"].view(np.uint8))


@pytest.mark.parametrize("name", golden_names("tiled_"))
def test_tile_pack_matches_reference(name):
    g = golden(name)
    BM, BN = (int(v) for v in g["block"])
    off0 = int(g["start_offset"][0])
    arena = np.full_like(g["vals"], 0)
    arena[:] = g["vals"]  # untouched slots keep the reference's fill value
    arena[off0:off0 + int(g["prefix"][-1])] = 0
    bitmask, prefix, total = oracle.tile_pack(g["dense"], BM, BN, arena, off0)
    np.testing.assert_array_equal(bitmask, g["bitmask"])
    np.testing.assert_array_equal(prefix, g["prefix"])
    assert int(g["vals_offset"][0]) == off0
    assert int(g["offset_after"][0]) == off0 + total
    np.testing.assert_array_equal(arena.view(np.uint8), g["vals"].view(np.uint8))


@pytest.mark.parametrize("name", [n for n in golden_names("tiled_") if "unpacked" in golden(n)])
def test_tile_unpack_and_spAx_match_reference(name):
    g = golden(name)
    BM, BN = (int(v) for v in g["block"])
    M, N = (int(v) for v in g["shape"])
    off = int(g["vals_offset"][0])
    dense = oracle.tile_unpack(g["vals"], g["bitmask"], g["prefix"], off, (M, N), BM, BN)
    # spAx(x_sparse, I) is the reference's unpack (exact: one nonzero product per sum)
    np.testing.assert_array_equal(dense.view(np.uint8), g["unpacked"].view(np.uint8))
    code = oracle.dtype_code(g["dense"])
    # ... and it equals the packed input by value (-0.0 unpacks as +0.0)
    np.testing.assert_array_equal(oracle.to_f64(dense, code), oracle.to_f64(g["dense"], code))
    for key, sq in (("spAx", False), ("spAx_sq", True)):
        got = oracle.to_f64(oracle.spAx(g["vals"], g["bitmask"], g["prefix"], off, (M, N), BM, BN,
                                        g["spAx_W"], square=sq), code)
        ref = oracle.to_f64(g[key], code)
        tol = 1e-5 if code == oracle.F32 else 2e-2
        np.testing.assert_allclose(got, ref, rtol=tol, atol=tol * np.abs(ref).max())


@pytest.mark.parametrize("name", golden_names("tiled_"))
def test_mask_kernels_match_reference(name):
    g = golden(name)
    BM, BN = (int(v) for v in g["block"])
    got = oracle.mask_with_bitmask(g["grad"], g["bitmask"], BM, BN)
    np.testing.assert_array_equal(got.view(np.uint8), g["grad_masked"].view(np.uint8))
    if "grad_relu2" in g:
        off = int(g["vals_offset"][0])
        gr, vsq = oracle.grad_relu2(g["grad"], g["vals"], g["bitmask"], g["prefix"], off, BM, BN)
        np.testing.assert_array_equal(gr.view(np.uint8), g["grad_relu2"].view(np.uint8))
        np.testing.assert_array_equal(vsq.view(np.uint8), g["vals_squared"].view(np.uint8))


@pytest.mark.parametrize("name", golden_names("tiled128_"))
def test_tile128_variant_matches_reference(name):
    g = golden(name)
    M, N = (int(v) for v in g["shape"])
    arena = np.zeros(M * N, dtype=g["dense"].dtype)
    bitmask, prefix, total = oracle.tile_pack(g["dense"], 128, 128, arena, 0)
    np.testing.assert_array_equal(bitmask, g["bitmask"])
    np.testing.assert_array_equal(prefix, g["prefix"])
    np.testing.assert_array_equal(arena[:total].view(np.uint8), g["vals"].view(np.uint8))
    dense = oracle.tile_unpack(g["vals"], bitmask, prefix, 0, (M, N), 128, 128)
    np.testing.assert_array_equal(dense.astype(np.float32), g["unpacked_f32"])


@pytest.mark.parametrize("act", ["relu", "relu2"])
def test_ffn_matches_reference(act):
    g = golden(f"ffn_{act}")
    r = oracle.ffn_fwd_bwd(g["x"], g["W1"], g["W2"], g["dout"], act=act)
    for key, ref in (("out", "out"), ("dx", "dx"), ("dW1", "dW1"), ("dW2", "dW2")):
        want = g[ref].astype(np.float64)
        np.testing.assert_allclose(r[key], want, rtol=1e-5, atol=1e-5 * np.abs(want).max(),
                                   err_msg=f"{act}:{key}")
        dense = g[ref + "_dense"].astype(np.float64)
        np.testing.assert_allclose(r[key], dense, rtol=1e-5, atol=1e-5 * np.abs(dense).max())
    assert int(g["nnz"][0]) == int(r["mask"].sum())


def test_sp24_oracle_split_is_lossless():
    """2:4 part + overflow reproduce every non-zero of A (the split the sparse
    tensor-core path relies on), and every kept pair has idx0 < idx1."""
    rng = np.random.default_rng(4)
    for p_zero in (0.0, 0.5, 0.9):
        A = rng.standard_normal((256, 512)).astype(np.float32)
        A[rng.random(A.shape) < p_zero] = 0
        A_bits = oracle.f32_to_bf16(A)
        vals, nib, rows, cols, ov = oracle.sp24_compress(A_bits)
        full = oracle.sp24_project(vals, nib)
        full[rows, cols] = ov
        keep = (A_bits & 0x7FFF) != 0
        assert np.array_equal(full[keep], A_bits[keep])
        assert not np.any(full[~keep] & 0x7FFF)
        # kept slots carry the element's own bits, signed zeros included
        assert np.array_equal(full[full != 0], A_bits[full != 0])
        assert np.all((nib & 3) < (nib >> 2))
        meta = oracle.sp24_meta(nib)
        assert meta.shape == (2, 4, 128, 4)


@pytest.mark.parametrize("name", golden_names("codec15_"))
def test_codec15_matches_reference(name):
    g = golden(name)
    n = g["bits"].size
    comp = oracle.codec15_compress(g["bits"])
    np.testing.assert_array_equal(comp, g["compressed"])
    np.testing.assert_array_equal(oracle.codec15_uncompress(comp, n), g["restored"])
    if not name.startswith("codec15_raw"):  # non-negative data round-trips exactly
        np.testing.assert_array_equal(g["restored"], g["bits"])


def test_codec15_sign_lands_on_the_next_field():
    """A set sign bit of value i reaches bit 0 of value i + 1 exactly when the
    byte that holds stream bit 15 (i + 1) starts inside value i."""
    for i in range(16):
        bits = np.zeros(17, np.uint16)
        bits[i] = 0x8000
        got = oracle.codec15_uncompress(oracle.codec15_compress(bits), 17)
        want = np.zeros(17, np.uint16)
        if (15 * (i + 1)) % 8:
            want[i + 1] = 1
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("name", ["products_sparse_relu_Ax_f32", "products_full_matmul_f32"])
def test_relu_ax_pack_matches_reference(name):
    """relu(x @ W1.T) packed as (vals, meta) by the reference (its Triton
    product under the interpreter, or F.linear) against the oracle's float64
    product rounded to float32: mask and prefix bit for bit, values within
    1e-5 of the largest."""
    g = golden(name)
    vals, bitmask, prefix = oracle.relu_ax_pack(g["x"], g["W1"])
    np.testing.assert_array_equal(bitmask, g["bitmask"])
    np.testing.assert_array_equal(prefix, g["prefix"])
    np.testing.assert_allclose(vals, g["vals"], rtol=0, atol=1e-5 * np.abs(vals).max())


def test_relu_spAx_matches_reference():
    """Layer 2 of old/full_matmul: relu(unpack(vals, meta) @ W2.T) from the
    reference's own layer-1 values, within 1e-5 of the largest output."""
    g = golden("products_full_matmul_f32")
    M, N = g["x"].shape[0], g["W1"].shape[0]
    A = oracle.tile_unpack(g["vals"], g["bitmask"], g["prefix"], 0, (M, N), 128, 128)
    want = oracle.relu_matmul(A, np.ascontiguousarray(g["W2"]).T)
    np.testing.assert_allclose(g["y"], want, rtol=0, atol=1e-5 * np.abs(want).max())


def test_relu_sparse_Ax_matches_reference():
    """old/sparse_matmul: the reference's pack of A round-trips through the
    oracle, and relu(A @ x) (float32 operands, "ieee") is within 1e-5 of the
    largest output."""
    g = golden("products_relu_sparse_Ax_f32")
    A = g["A"]
    arena = np.zeros(A.size, dtype=np.float32)
    bitmask, prefix, total = oracle.tile_pack(A, 128, 128, arena, 0)
    np.testing.assert_array_equal(bitmask, g["bitmask"])
    np.testing.assert_array_equal(prefix, g["prefix"])
    np.testing.assert_array_equal(arena[:total].view(np.uint8), g["vals"].view(np.uint8))
    want = oracle.relu_matmul(A, g["x"])
    np.testing.assert_allclose(g["y"], want, rtol=0, atol=1e-5 * np.abs(want).max())
