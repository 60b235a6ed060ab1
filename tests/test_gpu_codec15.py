"""GPU parity of the 15-bit sign-strip codec (bitshifting/code.py) with the
reference's golden vectors and the oracle: every byte of the stream and
every restored word must match (integer work: bit-exact)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import golden, golden_names

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _status():
    yield
    import autoresearch2_b200 as sf
    sf.check_status()


def to_dev(bits, dtype=torch.bfloat16):
    return torch.from_numpy(np.asarray(bits, np.uint16).view(np.int16).copy()).to(DEV).view(dtype)


def words(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


@pytest.mark.parametrize("name", golden_names("codec15_"))
def test_codec15_matches_reference(name):
    from autoresearch2_b200 import bitshift
    g = golden(name)
    n = g["bits"].size
    dtype = torch.float16 if "f16" in name else torch.bfloat16
    stream = bitshift.compress_fn(to_dev(g["bits"], dtype))
    assert stream.numel() == bitshift.padded_bytes(n)
    np.testing.assert_array_equal(stream[:bitshift.compressed_bytes(n)].cpu().numpy(), g["compressed"])
    out = bitshift.uncompress_fn(stream, (n,), dtype)
    np.testing.assert_array_equal(words(out), g["restored"])


@pytest.mark.parametrize("n", [0, 1, 15, 16, 17, 4095, 4096, 4097, 531441, 1000003])
def test_codec15_random_words_match_oracle(n):
    """Every 16-bit pattern (sign bits, NaN and Inf patterns included)."""
    from autoresearch2_b200 import bitshift
    rng = np.random.default_rng(n)
    bits = rng.integers(0, 1 << 16, n, dtype=np.uint16)
    stream = bitshift.compress_fn(to_dev(bits))
    want = oracle.codec15_compress(bits)
    got = stream[:want.size].cpu().numpy()
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(words(bitshift.uncompress_fn(stream, (n,), torch.bfloat16)),
                                  oracle.codec15_uncompress(want, n))


@pytest.mark.parametrize("w_off,b_off", [(1, 0), (0, 3), (7, 5)])
def test_codec15_unaligned_buffers(w_off, b_off):
    """Word pointers off a 16-byte boundary (by w_off words) and byte pointers
    off it (by b_off bytes) take the scalar paths; the bytes outside the
    stream stay untouched."""
    from autoresearch2_b200 import _lib
    n = 3 * 4096 + 77
    nb = oracle.codec15_bytes(n)
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 1 << 16, n, dtype=np.uint16)
    src = torch.zeros(n + 16, dtype=torch.int16, device=DEV)
    src[w_off:w_off + n] = torch.from_numpy(bits.view(np.int16))
    dst = torch.full((nb + 32,), 0xA5, dtype=torch.uint8, device=DEV)
    st = _lib.stream_ptr(torch.device(DEV))
    vp = ctypes.c_void_p
    _lib.call("sffn_codec15_compress", vp(src.data_ptr() + 2 * w_off), n, vp(dst.data_ptr() + b_off), nb, st)
    got = dst.cpu().numpy()
    np.testing.assert_array_equal(got[b_off:b_off + nb], oracle.codec15_compress(bits))
    assert (got[:b_off] == 0xA5).all() and (got[b_off + nb:] == 0xA5).all()
    back = torch.full((n + 16,), -1, dtype=torch.int16, device=DEV)
    _lib.call("sffn_codec15_uncompress", vp(dst.data_ptr() + b_off), nb, n, vp(back.data_ptr() + 2 * w_off), st)
    b = back.cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(b[w_off:w_off + n], oracle.codec15_uncompress(got[b_off:b_off + nb], n))
    assert (b[:w_off] == 0xFFFF).all() and (b[w_off + n:] == 0xFFFF).all()


def test_codec15_round_trip_at_the_largest_size():
    """3^16 non-negative bf16 values (bitshifting/prepare.py:26's largest size)
    come back exactly; the stream is 15/16 of the data."""
    from autoresearch2_b200 import bitshift
    n = 3 ** 16
    g = torch.Generator(device=DEV).manual_seed(0)
    x = torch.randn(n, generator=g, device=DEV).to(torch.bfloat16).abs()
    stream = bitshift.compress_fn(x)
    assert bitshift.compressed_bytes(n) * 16 <= 15 * 2 * n + 16
    assert torch.equal(bitshift.uncompress_fn(stream, x.shape, torch.bfloat16), x)


def test_codec15_ops_and_short_stream():
    import autoresearch2_b200 as sf
    x = to_dev(np.arange(0, 3000, 7, dtype=np.uint16), torch.float16).reshape(3, -1)
    stream = torch.ops.sparseffn.codec15_compress(x)
    assert torch.equal(torch.ops.sparseffn.codec15_uncompress(stream, list(x.shape), torch.float16), x)
    with pytest.raises(ValueError, match="bytes"):
        sf.bitshift.uncompress_fn(stream[:10], x.shape, torch.float16)
    with pytest.raises(ValueError, match="16-bit"):
        sf.bitshift.compress_fn(torch.zeros(4, device=DEV))
