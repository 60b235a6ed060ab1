"""The no-allocation flat pack entry point, called through the C ABI.

sffn_flat_pack_noalloc serves callers that cannot allocate device memory --
plug-ins that are handed only their input and output buffers, programs whose
memory manager owns the device or runs to a fixed budget, and paths that must
not risk the synchronisation a cudaMalloc can cause.  It keeps its scratch in
a fixed array inside the library instead of taking a workspace.  These checks
compare it with the regular sffn_flat_pack (which takes a workspace) on two
calls in a row -- the second call finds the first call's state in the shared
array and must clear it -- and check that oversized inputs are refused.
Masks, values and counts are integer/byte results, so they must match exactly.

This file is collected last on purpose: it must pass in a fresh process (the
first call does the per-device set-up) and after every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _pack_both(d):
    from autoresearch2_b200 import _lib
    L = _lib.load()
    n = d.numel()
    code = _lib.dtype_code(d)
    st = _lib.stream_ptr(d.device)
    res = []
    for noalloc in (False, True):
        mask = torch.full(((n + 7) // 8,), 0xAB, dtype=torch.uint8, device=DEV)
        vals = torch.full((n,), 7, dtype=d.dtype, device=DEV)
        out = torch.zeros(2, dtype=torch.int64, device=DEV)  # nnz, status
        nnz_p = ctypes.c_void_p(out.data_ptr())
        status_p = ctypes.c_void_p(out.data_ptr() + 8)
        if noalloc:
            rc = L.sffn_flat_pack_noalloc(_lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), n,
                                          nnz_p, status_p, st)
        else:
            ws = _lib.workspace(L.sffn_flat_workspace_bytes(n), d.device)
            rc = L.sffn_flat_pack(_lib.ptr(d), code, n, _lib.ptr(mask), _lib.ptr(vals), n, nnz_p,
                                  _lib.ptr(ws), ws.numel(), status_p, st)
        assert rc == 0, L.sffn_error_string(rc)
        torch.cuda.synchronize()
        nnz, status = out.tolist()
        assert status == 0
        res.append((mask, vals[:nnz], nnz))
    return res


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_workspace_pack_on_two_calls(dtype):
    g = torch.Generator(device=DEV).manual_seed(11)
    # two calls in a row with different sizes and densities
    for rows, cols, p in ((1024, 4099, 0.3), (3000, 2048, 0.05)):
        keep = torch.rand(rows, cols, device=DEV, generator=g) < p
        d = torch.where(keep, torch.randn(rows, cols, device=DEV, generator=g),
                        torch.zeros((), device=DEV)).to(dtype)
        (m0, v0, n0), (m1, v1, n1) = _pack_both(d)
        assert n0 == n1 == int(keep.sum())
        assert torch.equal(m0, m1)
        assert torch.equal(v0.view(torch.uint8), v1.view(torch.uint8))


def test_noalloc_refuses_sizes_beyond_its_capacity():
    from autoresearch2_b200 import _lib
    L = _lib.load()
    too_many = 67_108_864 + 1
    dummy = torch.zeros(16, dtype=torch.uint8, device=DEV)
    out = torch.zeros(2, dtype=torch.int64, device=DEV)
    rc = L.sffn_flat_pack_noalloc(_lib.ptr(dummy), _lib.BF16, too_many, _lib.ptr(dummy),
                                  _lib.ptr(dummy), 0, ctypes.c_void_p(out.data_ptr()),
                                  ctypes.c_void_p(out.data_ptr() + 8), _lib.stream_ptr(DEV))
    assert rc == 8  # SFFN_ERR_TOO_LARGE
    assert b"capacity" in L.sffn_last_cuda_error()
