"""CPU-side checks of the C-ABI library: it loads without a GPU, exports every
entry point include/sparseffn.h declares, and its host-side argument checks
reject bad calls before touching the device."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sparseffn.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sffn_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from autoresearch2_b200 import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    syms = declared_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_every_symbol():
    from autoresearch2_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_library_is_built_for_sm100a_only():
    from autoresearch2_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)


def test_version_and_errors(lib):
    assert lib.sffn_version() >= 100
    assert lib.sffn_error_string(0) == b"ok"
    assert b"dtype" in lib.sffn_error_string(2)


def test_workspace_queries(lib):
    # max of the pack look-back states (8 B per 16K bf16 elements) and the
    # unpack counts + prefix (12 B per 16K elements, + 8 for the total)
    assert lib.sffn_flat_workspace_bytes(0) == 16
    assert lib.sffn_flat_workspace_bytes(8192) == 16 + 8
    assert lib.sffn_flat_workspace_bytes(8193) == 16 + 16
    assert lib.sffn_tile_workspace_bytes(130, 192, 64, 64) == 16 + 3 * 3 * 8


def test_host_side_rejections(lib):
    vp = ctypes.c_void_p
    dummy = vp(256)  # never dereferenced: every call below fails its host checks
    # unsupported dtype
    assert lib.sffn_flat_pack(dummy, 9, 10, dummy, dummy, 10, dummy, dummy, 64, dummy, None) == 2
    # negative size
    assert lib.sffn_flat_pack(dummy, 1, -1, dummy, dummy, 10, dummy, dummy, 64, dummy, None) == 1
    # misaligned dense pointer
    assert lib.sffn_flat_pack(vp(258), 1, 10, dummy, dummy, 10, dummy, dummy, 64, dummy, None) == 3
    # workspace too small
    assert lib.sffn_flat_pack(dummy, 1, 10 ** 6, dummy, dummy, 10, dummy, dummy, 8, dummy, None) == 4
    # unsupported tile shape
    assert lib.sffn_tile_pack(dummy, 1, 64, 64, 64, 48, 64, dummy, dummy, dummy, 10, dummy,
                              vp(512), dummy, 4096, dummy, None) == 6
    # cursor and vals_offset aliasing
    assert lib.sffn_tile_pack(dummy, 1, 64, 64, 64, 64, 64, dummy, dummy, dummy, 10, dummy,
                              dummy, dummy, 4096, dummy, None) == 1
    # unpack row range past the matrix
    assert lib.sffn_tile_unpack(dummy, 10, dummy, dummy, dummy, 1, 64, 64, 64, 64, 0, 2, 0, dummy,
                                1, 64, None) == 1
    # TF32 GEMM: empty shape, row stride below K, a row stride that is not 16 bytes, misaligned base
    i64 = ctypes.c_int64
    assert lib.sffn_gemm_tf32(dummy, i64(64), dummy, i64(64), dummy, i64(64), i64(0), i64(64), i64(64), 0,
                              dummy, None) == 1
    assert lib.sffn_gemm_tf32(dummy, i64(32), dummy, i64(64), dummy, i64(64), i64(64), i64(64), i64(64), 0,
                              dummy, None) == 1
    assert lib.sffn_gemm_tf32(dummy, i64(66), dummy, i64(64), dummy, i64(64), i64(64), i64(64), i64(64), 0,
                              dummy, None) == 3
    assert lib.sffn_gemm_tf32(vp(260), i64(64), dummy, i64(64), dummy, i64(64), i64(64), i64(64), i64(64), 0,
                              dummy, None) == 3
    # ReLU GEMM: empty shape, row stride below K
    assert lib.sffn_gemm_relu(dummy, i64(64), 0, dummy, i64(64), 0, dummy, 0, i64(64), i64(0), i64(64),
                              i64(64), None, None, 0, dummy, None) == 1
    assert lib.sffn_gemm_relu(dummy, i64(32), 0, dummy, i64(64), 0, dummy, 1, i64(64), i64(64), i64(64),
                              i64(64), None, None, 0, dummy, None) == 1
    assert lib.sffn_round_tf32(dummy, dummy, i64(-1), None) == 1
    assert lib.sffn_round_tf32(None, dummy, i64(4), None) == 1
    assert lib.sffn_round_tf32(None, None, i64(0), None) == 0


def test_codec15_host_checks(lib):
    vp = ctypes.c_void_p
    lib.sffn_codec15_bytes.restype = ctypes.c_int64
    lib.sffn_codec15_bytes.argtypes = [ctypes.c_int64]
    assert [lib.sffn_codec15_bytes(n) for n in (0, 1, 8, 16, 17, -1)] == [0, 2, 15, 30, 32, -1]
    words, stream = vp(1 << 20), vp(1 << 24)  # never dereferenced
    assert lib.sffn_codec15_compress(None, 0, None, 0, None) == 0  # empty: nothing to do
    assert lib.sffn_codec15_compress(words, -1, stream, 10, None) == 1
    assert lib.sffn_codec15_compress(None, 5, stream, 10, None) == 1
    assert lib.sffn_codec15_compress(words, 16, stream, 29, None) == 1  # stream needs 30 bytes
    assert lib.sffn_codec15_compress(vp((1 << 20) + 1), 16, stream, 30, None) == 3
    assert lib.sffn_codec15_compress(words, 16, vp((1 << 20) + 31), 30, None) == 1  # overlap
    assert lib.sffn_codec15_uncompress(stream, 31, 17, words, None) == 1  # stream needs 32 bytes
    assert lib.sffn_codec15_uncompress(stream, 30, 16, vp((1 << 24) - 2), None) == 1  # overlap
    assert lib.sffn_codec15_uncompress(stream, 30, 1 << 41, words, None) == 1  # beyond 2^40 words


def test_python_api_refuses_cpu_tensors():
    import torch
    import autoresearch2_b200 as sf
    with pytest.raises(ValueError, match="CUDA"):
        sf.bitsparse_pack(torch.zeros(4, 4))


def test_relu_products_refuse_cpu_tensors():
    """The (vals, meta) products and the TF32 / ReLU GEMM helpers raise on CPU
    tensors before any device call; an unknown input_precision is rejected."""
    import torch
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm
    x, W1 = torch.randn(64, 32), torch.randn(96, 32)
    meta = {"bitmask": torch.zeros(1024, dtype=torch.uint8), "prefix": torch.zeros(2, dtype=torch.int32),
            "grid_m": 1, "grid_n": 1, "BLOCK_M": 128, "BLOCK_N": 128, "shape": (64, 96)}
    calls = [lambda: sf.tiled.sparse_relu_Ax(W1, x), lambda: sf.tiled.sp_relu_Ax(W1, x),
             lambda: sf.tiled.relu_spAx(torch.zeros(4), meta, torch.randn(16, 96)),
             lambda: sf.tiled.relu_sparse_Ax(torch.zeros(4), meta, torch.randn(96, 8)),
             lambda: gemm.matmul_tf32(x, W1), lambda: gemm.round_tf32(x),
             lambda: gemm.mm_relu(x.bfloat16(), W1.T.bfloat16())]
    for c in calls:
        with pytest.raises(ValueError, match="CUDA"):
            c()


def test_launch_accounting():
    """Kernels counted per successful call (the bench's gpu_launches): the
    table's count, one launch per 1024-wide K chunk of the float32-output
    GEMM, two for the tile pack without values (count and scan), three with."""
    from autoresearch2_b200 import _lib
    vp = ctypes.c_void_p
    assert _lib._launches("sffn_gemm_bf16_f32out", [None] * 10 + [6 * 3072]) == 18
    assert _lib._launches("sffn_gemm_bf16_f32out", [None] * 10 + [100]) == 1
    assert _lib._launches("sffn_tile_pack", [None] * 9 + [None]) == 2
    assert _lib._launches("sffn_tile_pack", [None] * 9 + [vp(0)]) == 2
    assert _lib._launches("sffn_tile_pack", [None] * 9 + [vp(4096)]) == 3
    assert _lib._launches("sffn_ffn_up", []) == 1 and _lib._launches("sffn_version", []) == 0
    assert set(_lib.LAUNCHING) <= set(_lib.SIGNATURES)
